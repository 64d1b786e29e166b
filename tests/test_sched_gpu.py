"""GPU tests of the dynamic row-unit scheduling of the streaming forward and
backward kernels (rows handed to CTAs through a per-launch counter instead
of one static tile per CTA).

* Bit-identical results: every row is still scanned by one CTA in chunk
  order, so the dynamic and the static tilings (FPSCAN_B200_STATIC_TILES=1,
  run in a child process) must agree bit for bit on every variant that
  schedules dynamically: forward, reverse, fused backward, gated forward and
  backward, scan with initial state, and the sequence-shard reduce / scan
  steps.  The plain forward and backward are also checked against the
  float64 oracle.
* Counter reset: a launch recorded into a CUDA graph keeps one counter word
  for every replay, so replays only give the right rows if each launch leaves
  its word at zero (output poisoned with NaN before every replay).
* Concurrent streams: launches in flight at the same time on different
  streams use different words.
"""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import fpscan_b200 as fpscan
import oracle
from fpscan_b200 import _lib
from fpscan_b200.distributed import CudaOps

from test_scan_gpu import _check

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))

# Shapes with more row units than resident CTAs (dynamic scheduling on), for
# one and several chunks per row, plus one with short rows packed per chunk.
CASES = [
    (torch.bfloat16, (4, 1024, 4096)),
    (torch.bfloat16, (2, 1024, 16384)),
    (torch.float32, (8, 1024, 1024)),
    (torch.float16, (32, 1024, 256)),
]


def _inputs(dtype, shape, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    g = torch.sigmoid(2 + torch.randn(shape, generator=gen, device="cuda"))
    x = 0.1 * torch.randn(shape, generator=gen, device="cuda")
    go = torch.randn(shape, generator=gen, device="cuda")
    z = torch.randn(shape, generator=gen, device="cuda") + 2
    h0 = torch.randn(shape[:2], generator=gen, device="cuda")
    return g.to(dtype), x.to(dtype), go.to(dtype), z.to(dtype), h0


def compute_all():
    """Every dynamically scheduled variant on every case: name -> tensor."""
    res = {}
    ops = CudaOps()
    for i, (dtype, shape) in enumerate(CASES):
        g, x, go, z, h0 = _inputs(dtype, shape, seed=100 + i)
        y = fpscan.scan_forward(g, x)
        res[f"{i}.fwd"] = y
        res[f"{i}.rev"] = fpscan.scan_forward(g, x, reverse=True)
        dg, dt = fpscan.scan_backward(g, y, go)
        res[f"{i}.dg"], res[f"{i}.dt"] = dg, dt
        res[f"{i}.init"] = fpscan.scan_forward(g, x, initial_state=h0)
        zz, xx = z.clone().requires_grad_(), x.clone().requires_grad_()
        yg = fpscan.pscan_gated(zz, xx)
        dz, dx = torch.autograd.grad(yg, (zz, xx), go)
        res[f"{i}.gated"], res[f"{i}.dz"], res[f"{i}.dx"] = yg.detach(), dz, dx
        g2, x2, go2, y2 = (t.reshape(-1, shape[-1]) for t in (g, x, go, y))
        carry = ops.fwd_reduce(g2, x2)
        res[f"{i}.carry"] = carry
        res[f"{i}.shard_scan"] = ops.fwd_scan(g2, x2, carry[1].contiguous())
        res[f"{i}.bwd_reduce"] = ops.bwd_reduce(g2, go2)
        sdg, sdt = ops.bwd_scan(g2, y2, go2, carry[0].contiguous(), carry[1].contiguous())
        res[f"{i}.shard_dg"], res[f"{i}.shard_dt"] = sdg, sdt
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    return {k: v.detach().cpu() for k, v in res.items()}


def test_dynamic_matches_static_bitwise(tmp_path):
    dyn = compute_all()
    path = tmp_path / "static.pt"
    code = (f"import sys, torch; sys.path.insert(0, {os.path.dirname(HERE)!r}); "
            f"sys.path.insert(0, {HERE!r})\n"
            "import test_sched_gpu as t\n"
            f"torch.save(t.compute_all(), {str(path)!r})\n")
    env = dict(os.environ, FPSCAN_B200_STATIC_TILES="1")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    static = torch.load(path)
    assert static.keys() == dyn.keys()
    bad = [k for k in dyn if not torch.equal(dyn[k], static[k])]
    assert not bad, f"dynamic and static tilings differ on {bad}"


@pytest.mark.parametrize("dtype,shape", CASES)
def test_dynamic_matches_oracle(dtype, shape):
    g, x, go, _, _ = _inputs(dtype, shape, seed=7)
    g64, x64 = g.double().cpu().numpy(), x.double().cpu().numpy()
    y = fpscan.scan_forward(g, x)
    y64 = oracle.scan_f64(g64, x64)
    _check(y, y64, dtype, "forward")
    _check(fpscan.scan_forward(g, x, reverse=True), oracle.scan_f64(g64, x64, True), dtype, "rev")
    dg, dt = fpscan.scan_backward(g, y, go)
    dg64, dt64 = oracle.scan_bwd_f64(g64, y64, go.double().cpu().numpy())
    _check(dt, dt64, dtype, "dtokens")
    _check(dg, dg64, dtype, "dgates")


def test_graph_replays_reuse_one_counter():
    """Replays of a captured forward + backward reuse their counter words:
    each launch must leave its word at zero for the next replay."""
    dtype, shape = torch.bfloat16, (4, 1024, 4096)
    g, x, go, _, _ = _inputs(dtype, shape, seed=3)
    ref_y = fpscan.scan_forward(g, x)
    ref_dg, ref_dt = fpscan.scan_backward(g, ref_y, go)
    y = torch.empty_like(x)
    dg, dt = torch.empty_like(x), torch.empty_like(x)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):  # first calls outside the capture
        fpscan.scan_forward(g, x, out=y)
        fpscan.scan_backward(g, y, go)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fpscan.scan_forward(g, x, out=y)
        a, b = fpscan.scan_backward(g, y, go)
        dg.copy_(a)
        dt.copy_(b)
    for _ in range(20):
        for t in (y, dg, dt):
            t.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(y, ref_y)
        assert torch.equal(dg, ref_dg) and torch.equal(dt, ref_dt)
    assert _lib.device_status() == 0


def test_concurrent_streams():
    dtype, shape = torch.bfloat16, (2, 1024, 4096)
    ins = [_inputs(dtype, shape, seed=50 + i) for i in range(4)]
    refs = [fpscan.scan_forward(g, x) for g, x, *_ in ins]
    streams = [torch.cuda.Stream() for _ in ins]
    outs = [torch.full_like(x, float("nan")) for _, x, *_ in ins]
    torch.cuda.synchronize()
    for _ in range(10):
        for (g, x, *_), s, o in zip(ins, streams, outs):
            with torch.cuda.stream(s):
                fpscan.scan_forward(g, x, out=o)
    torch.cuda.synchronize()
    for o, r in zip(outs, refs):
        assert torch.equal(o, r)
    assert _lib.device_status() == 0
