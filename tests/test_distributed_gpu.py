"""Multi-GPU tests (NCCL, one process per GPU; skipped with fewer than 2
GPUs): the sequence-sharded pscan (forward + backward through the real
all-gather and the device carry kernels) and channel sharding, against the
single-GPU result and the float64 oracle."""
import os
import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, mode, dtype_name):
    try:
        import sys
        sys.path.insert(0, REPO)
        import torch.distributed as dist

        import fpscan_b200 as fp
        import oracle
        from fpscan_b200.distributed import local_channels, seq_sharded_pscan

        os.environ["NCCL_NVLS_ENABLE"] = "0"  # no NVLink multicast objects in these tests
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, device_id=dev)
        dtype = getattr(torch, dtype_name)
        b, d, L = 2, 96, 8192 * world
        gen = torch.Generator(device=dev).manual_seed(1234)  # same full tensors on every rank
        g = (0.999 + 0.001 * torch.rand(b, d, L, generator=gen, device=dev)).to(dtype)
        x = (torch.randn(b, d, L, generator=gen, device=dev) / L).to(dtype)
        w = torch.randn(b, d, L, generator=gen, device=dev).to(dtype)
        tol = 1e-5 if dtype == torch.float32 else 1e-2
        if mode.startswith("seq"):
            Lr = L // world
            sl = slice(rank * Lr, (rank + 1) * Lr)
            gl = g[..., sl].contiguous().requires_grad_()
            xl = x[..., sl].contiguous().requires_grad_()
            y64 = oracle.scan_f64(g.double().cpu().numpy(), x.double().cpu().numpy())
            dg64, dt64 = oracle.scan_bwd_f64(g.double().cpu().numpy(), y64, w.double().cpu().numpy())
            if mode == "seq_dropout":
                # Failure injected on the host: after one healthy chained
                # forward (which builds the chain), rank 0 skips the next
                # call.  Rank 1's wait for rank 0's row states runs out
                # (limit 0.2 s): its rows come out NaN and the chain's status
                # check raises.  No kernel of either rank is left in flight.
                from fpscan_b200 import _lib
                from fpscan_b200.distributed import check_chains

                y = seq_sharded_pscan(gl.detach(), xl.detach(), mode="chain")
                errs = [oracle.normwise_error(y.double().cpu().numpy(), y64[..., sl])]
                check_chains(block=True)
                if rank == 1:
                    fp.set_wait_limit(0.2)
                    y = seq_sharded_pscan(gl.detach(), xl.detach(), mode="chain")
                    raised = False
                    try:
                        check_chains(block=True)
                    except fp.DeviceStatusError as exc:
                        raised = "neighbouring rank" in str(exc)
                    fp.set_wait_limit(2.0)
                    errs += [0.0 if raised else 1.0,
                             0.0 if bool(torch.isnan(y).all()) else 1.0,
                             float(_lib.device_status())]  # cleared by the check
            elif mode == "seq_multi":
                # 6 chained forwards in flight (more than the 4 ring slots:
                # the producer rank must wait for the consumer's acks), one
                # backward through all of them, repeated twice
                errs = []
                for _ in range(2):
                    ys = [seq_sharded_pscan(gl, xl * (k + 1), mode="chain") for k in range(6)]
                    loss = sum((yk * w[..., sl]).sum() for yk in ys)
                    dgl, dxl = torch.autograd.grad(loss, (gl, xl))
                    errs += [oracle.normwise_error(ys[5].detach().double().cpu().numpy() / 6,
                                                   y64[..., sl]),
                             oracle.normwise_error(dxl.double().cpu().numpy() / 21, dt64[..., sl]),
                             oracle.normwise_error(dgl.double().cpu().numpy() / 21,
                                                   dg64[..., sl])]
                from fpscan_b200 import _lib
                errs.append(float(_lib.device_status()))  # 0: no wait gave up
            else:
                m = {"seq": "auto", "seq_chain": "chain", "seq_allgather": "allgather"}[mode]
                y = seq_sharded_pscan(gl, xl, mode=m)
                dgl, dxl = torch.autograd.grad(y, (gl, xl), w[..., sl].contiguous())
                errs = [oracle.normwise_error(y.detach().double().cpu().numpy(), y64[..., sl]),
                        oracle.normwise_error(dxl.double().cpu().numpy(), dt64[..., sl]),
                        oracle.normwise_error(dgl.double().cpu().numpy(), dg64[..., sl])]
        else:
            gl, xl = local_channels(g, rank, world), local_channels(x, rank, world)
            yl = fp.pscan(gl.contiguous(), xl.contiguous())
            full = fp.scan_forward(g, x)
            errs = [float((yl - local_channels(full, rank, world)).abs().max().item())]
            tol = 0.0  # same kernel on the same rows: bit-identical
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, errs, tol, None))
    except Exception:
        q.put((rank, None, None, traceback.format_exc()))


def _run(mode, dtype_name, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, mode, dtype_name))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    for rank, errs, tol, tb in res:
        assert tb is None, f"rank {rank}:\n{tb}"
        assert max(errs) <= tol, (rank, errs)


needs2 = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")


@needs2
@pytest.mark.parametrize("dtype_name", ["float32", "bfloat16"])
def test_seq_sharded_nccl_matches_oracle(dtype_name):
    _run("seq", dtype_name)


@needs2
@pytest.mark.parametrize("mode", ["seq_chain", "seq_allgather"])
def test_seq_sharded_modes_match_oracle(mode):
    """Chained (carries rank to rank over NVLink inside the kernels) and
    all-gather (NCCL) sequence sharding, each forced."""
    _run(mode, "float32")


@needs2
def test_seq_sharded_chain_ring_backpressure():
    """More chained calls in flight than ring slots, twice over."""
    _run("seq_multi", "float32")


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs 4 GPUs")
@pytest.mark.parametrize("mode", ["seq_chain", "seq_multi"])
def test_seq_sharded_chain_4_ranks(mode):
    """The chain through two interior ranks (both links on each)."""
    _run(mode, "float32", world=4)


@needs2
def test_channel_sharded_nccl_bit_identical():
    _run("chan", "bfloat16")


@needs2
def test_seq_sharded_chain_rank_dropout_raises():
    """A rank that skips a chained call: its neighbour's bounded wait runs
    out, its rows are NaN and the chain's status check raises
    DeviceStatusError (instead of silently returning zeros)."""
    _run("seq_dropout", "float32")
