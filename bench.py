"""Benchmark of the fpscan hot path on B200 (one process per GPU).

Default workload: pscan forward + backward, bf16,
batch 16 x dim 5120 x seqlen 16384, gates = exp(-softplus(z)), z ~ N(-1,1),
tokens, grad_out ~ N(0,1), seeded; the 81920 channels are split evenly over
the N ranks (fixed total work: strong scaling) with no communication.
A step is one PScan forward + backward (two kernels: scan, fused backward).

Metric: algorithmic HBM bytes / time, aggregated over all ranks, in GB/s:
3*N*s forward + 5*N*s backward (s = element size).  Every tensor is far
larger than L2 (126 MB), so no flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME]
    python bench.py --impl reference     # the reference's CPU path, timed on the host
    python bench.py --config anylen | channels_last --steps 20   # per-kernel tables

Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "scan HBM GB/s (% of B200 peak) and fwd+bwd p50 ms at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0

CONFIGS = {
    # channel-sharded bf16 fwd+bwd
    "shard_bd": dict(batch=16, dim=5120, seqlen=16384, dtype="bfloat16", gates="exp_softplus",
                     tokens_scale="unit"),
    # Mamba-like half fwd+bwd (single GPU, or channel-sharded)
    "halfbwd_bf16": dict(batch=8, dim=2048, seqlen=8192, dtype="bfloat16", gates="sigmoid",
                         tokens_scale="0.1"),
    "halfbwd_fp16": dict(batch=8, dim=2048, seqlen=8192, dtype="float16", gates="sigmoid",
                         tokens_scale="0.1"),
    # config 4 with the gate producer fused: the kernels read z and apply
    # exp(-softplus(z)) on load; the backward writes dz
    "shard_bd_gated": dict(batch=16, dim=5120, seqlen=16384, dtype="bfloat16",
                           gates="logits", tokens_scale="unit"),
    # the same at config-3 size (small enough for a full ncu capture)
    "halfbwd_gated": dict(batch=8, dim=2048, seqlen=8192, dtype="bfloat16", gates="logits",
                          tokens_scale="unit"),
    # sequence-sharded fp32 fwd+bwd, seqlen split over the ranks
    "shard_seq": dict(batch=4, dim=8192, seqlen=65536, dtype="float32", gates="0.999+0.001U",
                      tokens_scale="1/L"),
    # forward-only sweep, fp32, batch 2 x dim 256, seqlen 32..65536
    "fwd_sweep": dict(batch=2, dim=256, seqlen=65536, dtype="float32", gates="0.99+0.01U",
                      tokens_scale="1/L"),
    # beyond the reference (one GPU, per-kernel tables): any seqlen, and the
    # channel-last (batch, seqlen, dim) layout
    "anylen": dict(shapes=[(8, 2048, 8191, "bfloat16"), (16, 5120, 16383, "bfloat16"),
                           (8, 2048, 8191, "float32"), (2, 256, 100000, "float32")]),
    "channels_last": dict(shapes=[(8, 8192, 2048, "bfloat16"), (16, 16384, 5120, "bfloat16"),
                                  (8, 8192, 2048, "float32"), (4, 65536, 8192, "float32"),
                                  (2, 65536, 256, "float32"), (1, 100000, 512, "bfloat16")]),
}

# dram__bytes_read.sum + dram__bytes_write.sum per launch of the backward
# kernel, from one ncu capture of config 3 (134.2M elements: 1294.0 MB), scaled by the element count to the
# config-4 launch of each rank (traffic grows in proportion to the rows).
_CFG3_BWD_TRAFFIC_PER_ELEM = 1294.0e6 / (8 * 2048 * 8192)


def _peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def _dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.proc = None
        self.out = None
        bus = None
        try:
            p = torch.cuda.get_device_properties(device)
            bus = "%08X:%02X:%02X.0" % (p.pci_domain_id, p.pci_bus_id, p.pci_device_id)
        except Exception:
            pass
        self.cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                    "-lms", "50"] + ([f"--id={bus}"] if bus else [])

    def start(self):
        try:
            self.proc = subprocess.Popen(self.cmd, stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            parts = [s.strip() for s in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax),
                "reasons": sorted(reasons), "samples": len(sm)}


def _make_inputs(cfg, rows_lo, rows_hi, device, seed=0):
    """This rank's rows of the config's synthetic inputs (seeded per rank slice)."""
    dtype = getattr(torch, cfg["dtype"])
    L = cfg["seqlen"]
    n = rows_hi - rows_lo
    gen = torch.Generator(device=device).manual_seed(seed * 1000003 + rows_lo)
    shape = (1, n, L)
    z = torch.randn(shape, generator=gen, device=device)
    if cfg["gates"] == "exp_softplus":
        gates = torch.exp(-torch.nn.functional.softplus(z - 1.0)).to(dtype)
    elif cfg["gates"] == "logits":  # pre-activation z ~ N(-1, 1)
        gates = (z - 1.0).to(dtype)
    else:
        gates = torch.sigmoid(z + 2.0).to(dtype)
    del z
    scale = 0.1 if cfg["tokens_scale"] == "0.1" else 1.0
    tokens = (torch.randn(shape, generator=gen, device=device) * scale).to(dtype)
    grad_out = torch.randn(shape, generator=gen, device=device).to(dtype)
    return gates, tokens, grad_out


def _cpu_baseline(cfg, target_s=8.0):
    """Serial fp32 oracle (forward + fused backward), all host threads, on a
    bounded sample of the workload's rows, repeated for about target_s;
    GB/s by the same byte formula as the GPU line."""
    import oracle

    L = cfg["seqlen"]
    rows_total = cfg["batch"] * cfg["dim"]
    s = torch.empty((), dtype=getattr(torch, cfg["dtype"])).element_size()
    rng = np.random.default_rng(0)

    def make(rows):
        # gates in (0.27, 1) like exp(-softplus(N(-1,1))); timing does not
        # depend on the exact distribution
        g = (0.27 + 0.73 * rng.random((rows, L), dtype=np.float32)).astype(np.float32)
        x = rng.random((rows, L), dtype=np.float32) - 0.5
        go = rng.random((rows, L), dtype=np.float32) - 0.5
        return g, x, go

    rows = min(rows_total, 4096)
    g, x, go = make(rows)
    oracle.pscan_fwdbwd_f32(g, x, go)  # warm-up (first touch of the outputs)
    reps = 0
    t0 = time.perf_counter()
    while True:
        oracle.pscan_fwdbwd_f32(g, x, go)
        reps += 1
        dt = time.perf_counter() - t0
        if dt >= target_s:
            break
    rows_done = rows * reps
    return {"value": round(8 * rows_done * L * s / dt / 1e9, 3), "unit": "GB/s",
            "cores": oracle.num_threads(), "kind": "port",
            "sample": f"{rows} of {rows_total} rows x {L}, {reps} passes, fp32 serial forward + "
                      f"fused backward (oracle/scan_oracle.c, OpenMP over rows), {dt:.2f} s"}


def run_reference(args, cfg):
    """The reference's own CPU implementation of the path: parallel_scan_torch
    (Hillis-Steele, eval/baselines.py:40-61, restated in oracle/) forward plus
    torch autograd backward, all host threads, on a bounded sample of rows."""
    world, rank, _ = _dist_env()
    if rank != 0:
        return
    import oracle

    torch.set_num_threads(os.cpu_count() or 1)
    dtype = getattr(torch, cfg["dtype"])
    L = cfg["seqlen"]
    s = torch.empty((), dtype=dtype).element_size()
    gen = torch.Generator().manual_seed(0)

    def make(rows):
        z = torch.randn(1, rows, L, generator=gen)
        g = torch.exp(-torch.nn.functional.softplus(z - 1.0)).to(dtype).requires_grad_()
        x = torch.randn(1, rows, L, generator=gen).to(dtype).requires_grad_()
        go = torch.randn(1, rows, L, generator=gen).to(dtype)
        return g, x, go

    def step(g, x, go):
        y = oracle.parallel_scan_torch(g, x)
        torch.autograd.grad(y, (g, x), go)

    # Size the per-step sample: a warm call first (the first call pays
    # one-off allocation and thread start-up), then double the rows until a
    # step takes at least ~1 s of CPU work (and >= 1024 rows), or the whole
    # run would exceed the time budget.
    rows = 64
    g, x, go = make(rows)
    step(g, x, go)
    while True:
        g, x, go = make(rows)
        t0 = time.perf_counter()
        step(g, x, go)
        dt = time.perf_counter() - t0
        if rows >= 8192 or dt * 2 * (args.steps + args.warmup) > args.ref_budget_s:
            break
        if dt >= 1.0 and rows >= 1024:
            break
        rows *= 2
    g, x, go = make(rows)
    for _ in range(args.warmup):
        step(g, x, go)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step(g, x, go)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = 8 * rows * L * s * args.steps / total / 1e9
    sample = (f"{rows} of {cfg['batch'] * cfg['dim']} rows x {L} {cfg['dtype']} per step, "
              f"parallel_scan_torch forward + autograd backward on CPU")
    line = {
        "metric": METRIC, "value": round(value, 4), "unit": "GB/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": cfg["dtype"], "data": "synthetic",
        "config": _config_json(args, cfg, world),
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s",
                         "cores": torch.get_num_threads(), "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _config_json(args, cfg, world):
    return {"workload": f"{args.config}: pscan fwd+bwd {cfg['dtype']} batch={cfg['batch']} "
                        f"dim={cfg['dim']} seqlen={cfg['seqlen']}, channels split over {world} GPU(s)",
            "batch": cfg["batch"], "dim": cfg["dim"], "seqlen": cfg["seqlen"],
            "parallelism": f"channel-shard x{world}",
            "l2": "inputs larger than L2 (no flush)"}


def run_fpscan(args, cfg):
    import torch.distributed as dist

    import fpscan_b200
    from fpscan_b200 import _lib
    from fpscan_b200.distributed import channel_slice

    world, rank, local = _dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=device)
    _lib.load()

    rows_total = cfg["batch"] * cfg["dim"]
    lo, hi = channel_slice(rows_total, rank, world)
    L = cfg["seqlen"]
    dtype = getattr(torch, cfg["dtype"])
    s = torch.empty((), dtype=dtype).element_size()
    gates, tokens, grad_out = _make_inputs(cfg, lo, hi, device)
    gates.requires_grad_()
    tokens.requires_grad_()
    n_local = (hi - lo) * L

    gated = cfg["gates"] == "logits"

    def fwd(g, x):
        return fpscan_b200.pscan_gated(g, x, "exp_neg_softplus") if gated else fpscan_b200.pscan(g, x)

    def step():
        y = fwd(gates, tokens)
        torch.autograd.grad(y, (gates, tokens), grad_out)

    stream = torch.cuda.current_stream(device)
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()

    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    clocks = ClockSampler(local) if rank == 0 else None
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if clocks:
        clocks.start()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(args.steps):
        ev[i][0].record(stream)
        y = fwd(gates, tokens)
        ev[i][1].record(stream)
        torch.autograd.grad(y, (gates, tokens), grad_out)
        ev[i][2].record(stream)
    t_end.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clock_info = clocks.stop() if clocks else None
    elapsed_ms = t_start.elapsed_time(t_end)
    fwd_ms = [e[0].elapsed_time(e[1]) for e in ev]
    bwd_ms = [e[1].elapsed_time(e[2]) for e in ev]
    step_ms = [e[0].elapsed_time(e[2]) for e in ev]

    t = torch.tensor([elapsed_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    total_bytes = 8 * rows_total * L * s * args.steps
    value = total_bytes / (max_ms / 1e3) / 1e9

    peak, peak_kind = _peaks()
    bwd_mean = statistics.mean(bwd_ms)
    fwd_mean = statistics.mean(fwd_ms)
    achieved_bwd = 5 * n_local * s / (bwd_mean / 1e3) / 1e9
    achieved_fwd = 3 * n_local * s / (fwd_mean / 1e3) / 1e9
    traffic = (int(_CFG3_BWD_TRAFFIC_PER_ELEM * n_local)
               if cfg["dtype"] in ("bfloat16", "float16") else None)

    unfused = None
    if gated:
        # the same step composed from torch's activation + the plain scan:
        # what the fused path replaces (same seeds, device-timed, K steps)
        zf = gates.detach().float().requires_grad_()

        def step_unfused():
            g = torch.exp(-torch.nn.functional.softplus(zf)).to(gates.dtype)
            y = fpscan_b200.pscan(g, tokens)
            torch.autograd.grad(y, (zf, tokens), grad_out)

        for _ in range(3):
            step_unfused()
        ms_u = _timed_loop(step_unfused, args.steps, stream, world)
        unfused = {"ms_per_step": round(ms_u / args.steps, 4),
                   "gbs_same_bytes": round(8 * rows_total * L * s * args.steps / (ms_u / 1e3) / 1e9, 2),
                   "what": "torch exp(-softplus(z)) (fp32 z) + pscan fwd+bwd, autograd"}
        del zf

    e2e = None
    if not args.no_e2e:
        e2e = _e2e(args, cfg, gates.detach(), tokens.detach(), grad_out, device, world)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = _cpu_baseline(cfg)

    sweep = None
    if rank == 0 and world == 1 and not args.no_sweep:
        table, has_ref = _sweep_config2(device, 30, 3)
        sweep = {"what": "BASELINE config 2: scan_forward fp32 2x256xL, us per call and GB/s "
                         "(3*N*4 bytes), cold inputs (rotating sets), this library beside the "
                         "reference's own kernel", "reference_kernel_timed": has_ref,
                 "table": table}

    status = _lib.device_status()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3),
            "ms_per_step": round(max_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": cfg["dtype"],
            "data": "synthetic (seeded; BASELINE config distributions)",
            "config": _config_json(args, cfg, world),
            "pct_of_hbm_peak": round(100 * value / world / peak, 2),
            "fwd_bwd_p50_ms": round(statistics.median(step_ms), 4),
            "fwd_p50_ms": round(statistics.median(fwd_ms), 4),
            "bwd_p50_ms": round(statistics.median(bwd_ms), 4),
            "fwd_achieved_gbs": round(achieved_fwd, 1),
            "roofline": {"bound": "hbm", "kernel": "scan_bwd_kernel (fused backward)",
                         "achieved": round(achieved_bwd, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved_bwd / peak, 4), "peak_source": peak_kind,
                         "traffic": traffic,
                         "algorithmic_bytes_per_launch": 5 * n_local * s},
            "cpu_baseline": cpu,
            "unfused_gate_composition": unfused,
            "config2_sweep": sweep,
            "e2e": e2e,
            "gpu_launches": 2 * args.steps,
            "clocks": clock_info,
            "device_status": status,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _e2e(args, cfg, gates_d, tokens_d, grad_out_d, device, world):
    """Same metric through the public host-memory API
    (fpscan_b200.offload.scan_fwd_bwd_host): every step copies this step's
    inputs from pinned host memory to the device and all three results
    (y, grad_gates, grad_tokens) back, pipelined over row blocks."""
    import torch.distributed as dist

    from fpscan_b200.offload import scan_fwd_bwd_host

    g_h = gates_d.cpu().pin_memory()
    x_h = tokens_d.cpu().pin_memory()
    go_h = grad_out_d.cpu().pin_memory()
    outs = [torch.empty_like(g_h).pin_memory() for _ in range(3)]
    stream = torch.cuda.current_stream(device)

    def step():
        scan_fwd_bwd_host(g_h, x_h, go_h, *outs, device=device)

    step()
    torch.cuda.synchronize()
    k = max(1, min(args.steps, args.e2e_steps))
    if world > 1:
        dist.barrier()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(k):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    L = cfg["seqlen"]
    s = g_h.element_size()
    rows_total = cfg["batch"] * cfg["dim"]
    value = 8 * rows_total * L * s * k / (float(t.item()) / 1e3) / 1e9
    nbytes = g_h.numel() * s
    return {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 3 * nbytes,
            "d2h_bytes_per_step": 3 * nbytes, "steps": k,
            "path": "pinned host -> fpscan_b200.offload.scan_fwd_bwd_host (row blocks, "
                    "3 streams: H2D / kernels / D2H overlapped) -> pinned host"}


def _timed_loop(step, steps, stream, world):
    """Barrier + sync, K steps bracketed by CUDA events, max over ranks (ms)."""
    import torch.distributed as dist

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b)], dtype=torch.float64, device=stream.device)
    if world > 1:
        dist.barrier()
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_shard_seq(args, cfg):
    """every rank holds positions [r*L/N, (r+1)*L/N) of all
    4 x 8192 rows (fp32); one step = seq_sharded_pscan forward + backward
    (reduce, NCCL all-gather of the per-row carries, combine, scan -- both
    directions).  Credited bytes: 8*N*s of the whole sequence."""
    import torch.distributed as dist

    import fpscan_b200
    from fpscan_b200 import _lib
    from fpscan_b200.distributed import seq_sharded_pscan

    world, rank, local = _dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=device)
    _lib.load()
    B, D, L = cfg["batch"], cfg["dim"], cfg["seqlen"]
    Lr = L // world
    gen = torch.Generator(device=device).manual_seed(5 + rank)
    g = (0.999 + 0.001 * torch.rand(B, D, Lr, generator=gen, device=device)).requires_grad_()
    x = (torch.randn(B, D, Lr, generator=gen, device=device) / L).requires_grad_()
    go = torch.randn(B, D, Lr, generator=gen, device=device)

    def step():
        if world > 1:
            y = seq_sharded_pscan(g, x, mode=args.seq_mode)
        else:
            y = fpscan_b200.pscan(g, x)
        torch.autograd.grad(y, (g, x), go)

    for _ in range(args.warmup):
        step()
    stream = torch.cuda.current_stream(device)
    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
    ms = _timed_loop(step, args.steps, stream, world)
    clock_info = clocks.stop() if clocks else None
    s = 4
    value = 8 * B * D * L * s * args.steps / (ms / 1e3) / 1e9
    peak, peak_kind = _peaks()
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "float32", "data": "synthetic (seeded; BASELINE config 5 distributions)",
            "config": {"workload": f"shard_seq: pscan fwd+bwd fp32 batch={B} dim={D} seqlen={L}, "
                                   f"seqlen split over {world} GPU(s)",
                       "batch": B, "dim": D, "seqlen": L, "parallelism": f"seq-shard x{world}",
                       "seq_mode": args.seq_mode if world > 1 else "single GPU",
                       "l2": "inputs larger than L2 (no flush)"},
            "pct_of_hbm_peak": round(100 * value / world / peak, 2), "peak_source": peak_kind,
            "gpu_launches": (2 if world == 1 or args.seq_mode != "allgather" else 6) * args.steps,
            "clocks": clock_info, "device_status": _lib.device_status()}), flush=True)
    if world > 1:
        dist.destroy_process_group()


def _reference_extension():
    """The reference's own compiled extension (fpscan._C, unmodified, built
    for sm_100a by its setup.py into baseline/_ref), imported under a private
    name so it does not shadow this repository's ``fpscan`` package; None when
    it was not installed."""
    import glob
    import importlib.machinery
    import importlib.util

    paths = sorted(glob.glob(os.path.join(REPO, "baseline", "_ref", "fpscan", "_C*.so")))
    if not paths:
        return None
    try:
        loader = importlib.machinery.ExtensionFileLoader("fpscan_reference._C", paths[-1])
        spec = importlib.util.spec_from_file_location("fpscan_reference._C", paths[-1],
                                                      loader=loader)
        mod = importlib.util.module_from_spec(spec)
        loader.exec_module(mod)
        return mod
    except Exception:
        return None


def _sweep_config2(device, iters, warmup, seqlens=None, reps=5):
    """scan_forward, fp32, 2 x 256 channels, every seqlen
    32..65536, both directions, this library beside the reference's own
    kernel (fpscan._C from baseline/_ref, as eval/benchmark.py times it).
    Cold inputs: each call reads a different set of (gates, tokens, out)
    from a rotation whose sets together exceed 3x L2, so no flush kernel
    (and no write-back of a flush buffer) lands in the timed calls.  `iters`
    calls are queued behind a device-side sleep and run back to back between
    two CUDA events (single calls of a few microseconds are below the event
    timer's ~2 us resolution); the time per call is the median of `reps`
    such runs."""
    import fpscan_b200

    ref = _reference_extension()
    B, D = 2, 256
    l2 = 126 << 20
    impls = [("fpscan_b200", lambda g, x, o, r: fpscan_b200.scan_forward(g, x, r, o))]
    if ref is not None:
        impls.append(("reference", lambda g, x, o, r: ref.fullscan_forward(g, x, o, r)))
    table = []
    for lg in range(5, 17):
        L = 1 << lg
        if seqlens and L not in seqlens:
            continue
        per_set = 3 * B * D * L * 4
        nsets = max(2, -(-3 * l2 // per_set))
        gen = torch.Generator(device=device).manual_seed(L)
        g = 0.99 + 0.01 * torch.rand(nsets, B, D, L, generator=gen, device=device)
        x = torch.randn(nsets, B, D, L, generator=gen, device=device) / L
        o = torch.empty_like(x)
        row = {"seqlen": L, "rotating_sets": nsets}
        for name, fn in impls:
            for rev in (False, True):
                for i in range(warmup):
                    fn(g[i % nsets], x[i % nsets], o[i % nsets], rev)
                torch.cuda.synchronize()
                ts = []
                for rep in range(reps):
                    # a device-side sleep long enough for the host to queue
                    # all `iters` calls, so they run back to back
                    torch.cuda._sleep(iters * 40000)
                    a = torch.cuda.Event(enable_timing=True)
                    b = torch.cuda.Event(enable_timing=True)
                    a.record()
                    for i in range(iters):
                        k = (rep * iters + i) % nsets
                        fn(g[k], x[k], o[k], rev)
                    b.record()
                    b.synchronize()
                    ts.append(a.elapsed_time(b) / iters)
                p50 = statistics.median(ts)
                key = f"{name}_{'reverse' if rev else 'forward'}"
                row[f"{key}_us"] = round(p50 * 1e3, 3)
                row[f"{key}_gbs"] = round(3 * B * D * L * 4 / (p50 / 1e3) / 1e9, 1)
        if ref is not None:
            row["speedup_vs_reference_forward"] = round(
                row["reference_forward_us"] / row["fpscan_b200_forward_us"], 3)
        table.append(row)
        del g, x, o
        torch.cuda.empty_cache()
    return table, ref is not None


def run_fwd_sweep(args, cfg):
    """BASELINE config 2 on one GPU (_sweep_config2); `value` is this
    library's forward GB/s at seqlen 65536; the table has every row."""
    from fpscan_b200 import _lib

    world, rank, local = _dist_env()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    _lib.load()
    iters = max(args.steps, 20)
    table, has_ref = _sweep_config2(device, iters, args.warmup)
    peak, peak_kind = _peaks()
    last = table[-1]
    print(json.dumps({
        "metric": METRIC, "value": last["fpscan_b200_forward_gbs"], "unit": "GB/s", "n_gpus": 1,
        "steps": iters, "warmup": args.warmup,
        "ms_per_step": last["fpscan_b200_forward_us"] / 1e3, "higher_is_better": True,
        "scaling": "none", "vs_baseline": None, "dtype": "float32",
        "data": "synthetic (seeded; BASELINE config 2)",
        "config": {"workload": "fwd_sweep: scan_forward fp32 batch=2 dim=256 seqlen=32..65536",
                   "batch": 2, "dim": 256,
                   "l2": "cold: rotating input sets totalling > 3x L2, no flush kernel"},
        "pct_of_hbm_peak": round(100 * last["fpscan_b200_forward_gbs"] / peak, 2),
        "peak_source": peak_kind, "reference_kernel_timed": has_ref,
        "sweep": table}), flush=True)


def run_layout_table(args, kind):
    """One GPU: forward, reverse and fused-backward GB/s (algorithmic bytes:
    3*N*s and 5*N*s) of the any-seqlen or channel-last kernels at fixed
    shapes, CUDA events over K calls after W warm-up calls (every tensor is
    larger than L2 except the few-channel rows, noted in the table).  For the
    channel-last layout the reference's own recipe (transpose, last-axis
    scan, transpose back; here on this package's kernels) is timed beside it
    where the seqlen is one the reference accepts.  `value` = first row's
    forward+backward GB/s."""
    import fpscan_b200
    from fpscan_b200 import _lib, ops

    world, rank, local = _dist_env()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    _lib.load()

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        for _ in range(args.steps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / args.steps

    table = []
    for (d0, d1, d2, dt) in CONFIGS[kind]["shapes"][:args.max_shapes]:
        dtype = getattr(torch, dt)
        gen = torch.Generator(device=device).manual_seed(d0 + d1 + d2)
        shape = (d0, d1, d2)
        g = (0.9 + 0.1 * torch.rand(shape, generator=gen, device=device)).to(dtype)
        x = torch.randn(shape, generator=gen, device=device).to(dtype)
        go = torch.randn(shape, generator=gen, device=device).to(dtype)
        y = torch.empty_like(x)
        n, s = x.numel(), x.element_size()
        if kind == "anylen":
            fwd = lambda rev=False: fpscan_b200.scan_forward_anylen(g, x, reverse=rev, out=y)  # noqa: E731
            bwd = lambda: ops.scan_backward_anylen(g, y, go)  # noqa: E731
            layout = "(batch, dim, seqlen)"
        else:
            fwd = lambda rev=False: fpscan_b200.scan_forward_channels_last(g, x, reverse=rev, out=y)  # noqa: E731
            bwd = lambda: ops.scan_backward_channels_last(g, y, go)  # noqa: E731
            layout = "(batch, seqlen, dim)"
        ms_f, ms_r = timed(lambda: fwd()), timed(lambda: fwd(True))
        fwd()
        ms_b = timed(bwd)
        row = {"shape": list(shape), "layout": layout, "dtype": dt,
               "fwd_gbs": round(3 * n * s / ms_f / 1e6, 1), "rev_gbs": round(3 * n * s / ms_r / 1e6, 1),
               "bwd_gbs": round(5 * n * s / ms_b / 1e6, 1), "fwd_ms": round(ms_f, 4),
               "bwd_ms": round(ms_b, 4), "fwd_bwd_gbs": round(8 * n * s / (ms_f + ms_b) / 1e6, 1),
               "larger_than_l2": 3 * n * s > 126e6}
        if kind == "channels_last":
            row["kernel"] = ("streaming" if fpscan_b200.ops._lib.load().fpscan_cl_workspace_bytes(
                d0, d1, d2, ops.DTYPE_CODES[dtype], 0) <= 256 else "segmented")
            if d1 & (d1 - 1) == 0 and 32 <= d1 <= 65536 and 3 * n * s < 20e9:
                def recipe():
                    return fpscan_b200.scan_forward(g.mT.contiguous(), x.mT.contiguous()).mT.contiguous()
                row["reference_recipe_fwd_ms"] = round(timed(recipe), 4)
        table.append(row)
        del g, x, go, y
        torch.cuda.empty_cache()
    peak, peak_kind = _peaks()
    first = table[0]
    print(json.dumps({
        "metric": METRIC, "value": first["fwd_bwd_gbs"], "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(first["fwd_ms"] + first["bwd_ms"], 4), "higher_is_better": True,
        "scaling": "none", "vs_baseline": None, "dtype": first["dtype"],
        "data": "synthetic (seeded)",
        "config": {"workload": f"{kind}: forward / reverse / fused backward per shape",
                   "l2": "inputs larger than L2 except where larger_than_l2 is false"},
        "pct_of_hbm_peak": round(100 * first["fwd_bwd_gbs"] / peak, 2), "peak_source": peak_kind,
        "table": table, "device_status": _lib.device_status()}), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["fpscan", "reference"], default="fpscan")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="shard_bd")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true",
                    help="skip the config-2 seqlen sweep appended to the default run")
    ap.add_argument("--seq-mode", choices=["auto", "chain", "allgather"], default="auto",
                    help="shard_seq: carry exchange (chain: rank to rank over NVLink inside the "
                         "kernels; allgather: reduce + NCCL all-gather + scan)")
    ap.add_argument("--ref-budget-s", type=float, default=120.0,
                    help="--impl reference: size the per-step row sample so the run takes "
                         "about this many seconds")
    ap.add_argument("--max-shapes", type=int, default=None,
                    help="anylen / channels_last: only the first N shapes of the table")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    cfg = CONFIGS[args.config]
    if args.impl == "reference":
        # the reference's CPU path exists for the last-axis scan only
        run_reference(args, cfg if "dtype" in cfg else CONFIGS["shard_bd"])
    elif args.config == "shard_seq":
        run_shard_seq(args, cfg)
    elif args.config == "fwd_sweep":
        run_fwd_sweep(args, cfg)
    elif args.config in ("anylen", "channels_last"):
        run_layout_table(args, args.config)
    else:
        run_fpscan(args, cfg)


if __name__ == "__main__":
    main()
