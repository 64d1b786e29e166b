"""Multi-rank logic on CPU with gloo (world 2 and 4): the sequence-sharded
carry exchange (forward and backward) against the full-sequence oracle, and
channel sharding reassembling the full result.  Device steps come from
tests/cpu_fake_ops.py; the collectives, combine order and autograd plumbing
are fpscan_b200.distributed's own."""
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(b, d, L, seed=0):
    gen = torch.Generator().manual_seed(seed)
    g = 0.95 + 0.05 * torch.rand(b, d, L, generator=gen, dtype=torch.float64)
    x = torch.randn(b, d, L, generator=gen, dtype=torch.float64)
    w = torch.randn(b, d, L, generator=gen, dtype=torch.float64)
    return g, x, w


def _seq_worker(rank, world, port, q):
    try:
        import sys
        sys.path.insert(0, REPO)
        sys.path.insert(0, os.path.join(REPO, "tests"))
        import oracle
        from cpu_fake_ops import CpuOps
        from fpscan_b200.distributed import seq_sharded_pscan

        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}",
                                rank=rank, world_size=world)
        b, d, L = 2, 3, 64 * world
        g, x, w = _inputs(b, d, L, seed=11)
        Lr = L // world
        sl = slice(rank * Lr, (rank + 1) * Lr)
        gl = g[..., sl].contiguous().requires_grad_()
        xl = x[..., sl].contiguous().requires_grad_()
        y = seq_sharded_pscan(gl, xl, ops=CpuOps())
        (y * w[..., sl]).sum().backward()
        y_ref = oracle.scan_f64(g.numpy(), x.numpy())
        dg_ref, dt_ref = oracle.scan_bwd_f64(g.numpy(), y_ref, w.numpy())
        errs = (oracle.normwise_error(y.detach().numpy(), y_ref[..., sl]),
                oracle.normwise_error(xl.grad.numpy(), dt_ref[..., sl]),
                oracle.normwise_error(gl.grad.numpy(), dg_ref[..., sl]))
        dist.destroy_process_group()
        q.put((rank, errs, None))
    except Exception:
        q.put((rank, None, traceback.format_exc()))


def _chan_worker(rank, world, port, q):
    try:
        import sys
        sys.path.insert(0, REPO)
        import oracle
        from fpscan_b200.distributed import local_channels

        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}",
                                rank=rank, world_size=world)
        b, d, L = 2, 5, 64  # 10 rows: uneven split over 4 ranks
        g, x, _ = _inputs(b, d, L, seed=5)
        gl, xl = local_channels(g, rank, world), local_channels(x, rank, world)
        yl = torch.from_numpy(oracle.scan_f64(gl.numpy(), xl.numpy()))
        parts = [None] * world
        dist.all_gather_object(parts, yl)
        y = torch.cat([p.reshape(-1, L) for p in parts]).reshape(b, d, L)
        err = oracle.normwise_error(y.numpy(), oracle.scan_f64(g.numpy(), x.numpy()))
        dist.destroy_process_group()
        q.put((rank, (err,), None))
    except Exception:
        q.put((rank, None, traceback.format_exc()))


def _dropout_worker(rank, world, port, q):
    """Rank 1 never joins the exchange (it leaves after setting up the
    process group); rank 0's sequence-sharded forward must end with an
    error from its collective within the process group's timeout instead
    of hanging or returning a result."""
    try:
        import datetime
        import sys
        import time
        sys.path.insert(0, REPO)
        sys.path.insert(0, os.path.join(REPO, "tests"))
        from cpu_fake_ops import CpuOps
        from fpscan_b200.distributed import seq_sharded_pscan

        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}",
                                rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=5))
        if rank == 1:
            q.put((rank, (0.0,), None))
            q.close()
            q.join_thread()
            os._exit(0)  # leaves without a word: no barrier, no destroy
        b, d, L = 2, 3, 64 * world
        g, x, _ = _inputs(b, d, L, seed=3)
        Lr = L // world
        t0 = time.time()
        try:
            seq_sharded_pscan(g[..., :Lr].contiguous(), x[..., :Lr].contiguous(), ops=CpuOps())
            outcome = 1.0  # returned a result: wrong
        except (RuntimeError, dist.DistError):
            outcome = 0.0 if time.time() - t0 < 60 else 1.0
        q.put((rank, (outcome,), None))
        q.close()
        q.join_thread()
        os._exit(0)
    except Exception:
        q.put((rank, None, traceback.format_exc()))


def _run(worker, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, errs, tb in results:
        assert tb is None, f"rank {rank} failed:\n{tb}"
    return results


@pytest.mark.parametrize("world", [2, 4])
def test_seq_sharded_exchange_matches_full_sequence(world):
    for rank, errs, _ in _run(_seq_worker, world):
        # carries travel as fp32 (as on the GPU path): agreement to fp32 rounding
        assert max(errs) < 1e-6, (rank, errs)


def test_channel_sharding_reassembles_full_scan():
    for rank, errs, _ in _run(_chan_worker, 4):
        assert errs[0] == 0.0


def test_chain_mode_selection_and_epochs():
    """Host logic of the chained sequence-sharded mode that needs no GPU:
    mode validation, when "auto" picks the chain, epoch counting (never 0,
    wraps at 2^32).  The chain itself runs in tests/test_distributed_gpu.py
    (2 GPUs, one process each)."""
    import sys
    sys.path.insert(0, REPO)
    from fpscan_b200 import distributed as fd

    x = torch.empty(1, 2, 8192)
    assert not fd.chain_supported(x)  # CPU tensors never chain
    with pytest.raises(ValueError):
        fd.seq_sharded_pscan(x, x, mode="ring")
    assert fd.RankChain._bump(0) == 1
    assert fd.RankChain._bump(41) == 42
    assert fd.RankChain._bump(0xFFFFFFFF) == 1  # 0 is reserved (mailbox words start at 0)


def test_rank_that_never_joins_ends_the_exchange_with_an_error():
    for rank, errs, _ in _run(_dropout_worker, 2):
        assert errs[0] == 0.0, rank
