"""GPU parity tests of the channel-last scan (``scan_forward_channels_last``,
``pscan_channels_last``; C ABI ``fpscan_scan_fwd_cl`` / ``fpscan_scan_bwd_cl``):
(batch, seqlen, dim) tensors scanned along seqlen.

The reference supports this layout only through transposes around pscan
(README.md:94-99); the oracle here is the float64 serial scan of the
transposed tensors, and the same computation through this package's
last-axis kernels.  Tolerances as in test_scan_gpu.py.
"""
import numpy as np
import pytest
import torch

import fpscan_b200 as fpscan
import oracle

from test_scan_gpu import DTYPES, _check

pytestmark = pytest.mark.gpu
DEVICE = "cuda"


def _t64(t):
    """(B, L, D) tensor -> float64 numpy (B, D, L) for the oracle."""
    return t.detach().double().transpose(1, 2).contiguous().cpu().numpy()


def _from64(a):
    return np.ascontiguousarray(np.swapaxes(a, 1, 2))


def _inputs(shape, dtype, seed):
    gen = torch.Generator(device=DEVICE).manual_seed(seed)
    L = shape[1]
    g = 0.99 + 0.01 * torch.rand(shape, generator=gen, device=DEVICE)
    x = torch.randn(shape, generator=gen, device=DEVICE) / max(L, 32) ** 0.5
    go = torch.randn(shape, generator=gen, device=DEVICE)
    return g.to(dtype), x.to(dtype), go.to(dtype)


def _vec(dtype):
    return 4 if dtype == torch.float32 else 8


SHAPES = [  # (batch, seqlen, dim in 16-byte vectors)
    (2, 64, 32), (2, 1000, 32), (3, 333, 34), (1, 1, 32), (2, 65, 1), (1, 7, 5),
    (2, 4096, 64), (1, 12345, 33),
]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", SHAPES)
def test_channels_last_fwd_rev_bwd(dtype, shape):
    b, l, nv = shape
    shape = (b, l, nv * _vec(dtype))
    g, x, go = _inputs(shape, dtype, seed=l + nv)
    g64, x64 = _t64(g), _t64(x)
    for rev in (False, True):
        y = fpscan.scan_forward_channels_last(g, x, reverse=rev)
        _check(y, _from64(oracle.scan_f64(g64, x64, rev)), dtype, f"fwd rev={rev}")
    gg, xx = g.clone().requires_grad_(), x.clone().requires_grad_()
    y = fpscan.pscan_channels_last(gg, xx)
    dg, dt = torch.autograd.grad(y, (gg, xx), go)
    dg64, dt64 = oracle.scan_bwd_f64(g64, oracle.scan_f64(g64, x64), _t64(go))
    _check(dt, _from64(dt64), dtype, "dtokens")
    _check(dg, _from64(dg64), dtype, "dgates")


@pytest.mark.parametrize("shape", [(1, 100003, 128), (1, 70000, 256), (4, 20000, 4)])
def test_channels_last_few_columns_long(shape):
    """Few columns, long sequences: the time axis is cut into segments
    (reduce, compose, scan)."""
    dtype = torch.float32
    g, x, go = _inputs(shape, dtype, seed=shape[1])
    g64, x64 = _t64(g), _t64(x)
    _check(fpscan.scan_forward_channels_last(g, x), _from64(oracle.scan_f64(g64, x64)), dtype, "fwd")
    _check(fpscan.scan_forward_channels_last(g, x, reverse=True),
           _from64(oracle.scan_f64(g64, x64, True)), dtype, "rev")
    gg, xx = g.clone().requires_grad_(), x.clone().requires_grad_()
    dg, dt = torch.autograd.grad(fpscan.pscan_channels_last(gg, xx), (gg, xx), go)
    dg64, dt64 = oracle.scan_bwd_f64(g64, oracle.scan_f64(g64, x64), _t64(go))
    _check(dt, _from64(dt64), dtype, "dtokens")
    _check(dg, _from64(dg64), dtype, "dgates")


@pytest.mark.parametrize("dtype", DTYPES)
def test_channels_last_matches_transposed_pscan(dtype):
    """The reference's documented channel-last usage (README.md:94-99),
    pscan(g.mT.contiguous(), x.mT.contiguous()).mT, on this package's
    last-axis kernels, against the direct channel-last kernels."""
    b, l, d = 4, 8192, 1024
    g, x, go = _inputs((b, l, d), dtype, seed=9)
    y_cl = fpscan.scan_forward_channels_last(g, x)
    y_tr = fpscan.scan_forward(g.mT.contiguous(), x.mT.contiguous()).mT
    tol = 2e-6 if dtype == torch.float32 else 1e-2
    assert oracle.normwise_error(y_cl.double().cpu().numpy(), y_tr.double().cpu().numpy()) <= tol
    gg, xx = g.clone().requires_grad_(), x.clone().requires_grad_()
    d1 = torch.autograd.grad(fpscan.pscan_channels_last(gg, xx), (gg, xx), go)
    g2, x2 = g.mT.contiguous().requires_grad_(), x.mT.contiguous().requires_grad_()
    d2 = torch.autograd.grad(fpscan.pscan(g2, x2), (g2, x2), go.mT.contiguous())
    for u, v in zip(d1, d2):
        assert oracle.normwise_error(u.double().cpu().numpy(),
                                     v.mT.double().cpu().numpy()) <= tol
    # sampled channels against float64
    idx = [0, 517, 1023]
    ref = oracle.scan_f64(_t64(g[:, :, idx]), _t64(x[:, :, idx]))
    _check(y_cl[:, :, idx], _from64(ref), dtype, "sampled channels")


def test_channels_last_in_place_repeat_and_errors():
    g, x, _ = _inputs((2, 300, 64), torch.float32, seed=1)
    ref = _from64(oracle.scan_f64(_t64(g), _t64(x)))
    for _ in range(3):  # workspace reused across calls
        _check(fpscan.scan_forward_channels_last(g, x), ref, torch.float32, "repeat")
    xi = x.clone()
    fpscan.scan_forward_channels_last(g, xi, out=xi)
    _check(xi, ref, torch.float32, "in place")
    with pytest.raises(RuntimeError):  # dim not a multiple of 4 fp32 elements
        fpscan.scan_forward_channels_last(g[:, :, :63].contiguous(), x[:, :, :63].contiguous())
    with pytest.raises(RuntimeError):
        fpscan.scan_forward_channels_last(g.transpose(1, 2), x.transpose(1, 2))


_PATH_SCRIPT = r"""
import sys, numpy as np, torch
sys.path.insert(0, {repo!r}); sys.path.insert(0, {tests!r})
import fpscan_b200 as fpscan, oracle
from test_channels_last_gpu import _inputs, _t64, _from64, _vec
from test_scan_gpu import _check
for dtype in (torch.float32, torch.bfloat16, torch.float16):
    for (b, l, nv) in [(2, 1000, 32), (3, 333, 17), (1, 7, 9), (2, 4100, 64), (8, 300, 130)]:
        shape = (b, l, nv * _vec(dtype))
        g, x, go = _inputs(shape, dtype, seed=l + nv)
        g64, x64 = _t64(g), _t64(x)
        for rev in (False, True):
            _check(fpscan.scan_forward_channels_last(g, x, reverse=rev),
                   _from64(oracle.scan_f64(g64, x64, rev)), dtype, "fwd")
        gg, xx = g.clone().requires_grad_(), x.clone().requires_grad_()
        dg, dt = torch.autograd.grad(fpscan.pscan_channels_last(gg, xx), (gg, xx), go)
        dg64, dt64 = oracle.scan_bwd_f64(g64, oracle.scan_f64(g64, x64), _t64(go))
        _check(dt, _from64(dt64), dtype, "dtokens")
        _check(dg, _from64(dg64), dtype, "dgates")
from fpscan_b200 import _lib
assert _lib.device_status() == 0
print("ok")
"""


@pytest.mark.parametrize("path", ["stream", "split"])
def test_channels_last_both_paths(path):
    """One CTA per column and the segmented path (columns cut in time),
    each forced on the same cases in a fresh process (the choice is read
    once per process)."""
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    code = _PATH_SCRIPT.format(repo=os.path.dirname(here), tests=here)
    env = dict(os.environ, FPSCAN_B200_CL_PATH=path)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]


def test_channels_last_first_backward_on_autograd_thread():
    """The first channel-last launch of a process can come from autograd's
    backward worker thread, where no CUDA call has bound a context yet (the
    TMA descriptors are encoded against the current context): run it in a
    fresh process where the backward is the first launch of its kernel."""
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    code = (f"import sys; sys.path.insert(0, {os.path.dirname(here)!r}); import torch\n"
            "import fpscan_b200 as fp\n"
            "g = torch.rand(2, 64, 128, device='cuda').requires_grad_()\n"
            "x = torch.randn(2, 64, 128, device='cuda').requires_grad_()\n"
            "y = fp.pscan_channels_last(g, x)\n"
            "torch.autograd.grad(y.sum(), (g, x)); torch.cuda.synchronize(); print('ok')\n")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]
