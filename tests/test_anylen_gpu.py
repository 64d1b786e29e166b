"""GPU parity tests of the any-seqlen scan (``scan_forward_anylen``,
``pscan_anylen``; C ABI ``fpscan_scan_fwd_anylen`` / ``fpscan_scan_bwd_anylen``)
against the float64 oracle.

The reference limits seqlen to powers of two in [32, 65536]
(csrc/full_scan/full_scan.cu:207-233); these kernels take any seqlen >= 1, so
rows start at arbitrary element offsets, share 16-byte vectors with their
neighbours, and batch*dim*seqlen need not be a multiple of the vector width.
Tolerances are the ones of test_scan_gpu.py (reference tests/test_fpscan.py:
18-22 plus the normwise bound vs float64).
"""
import numpy as np
import pytest
import torch

import fpscan_b200 as fpscan
import oracle

from test_scan_gpu import DTYPES, _check, _np64

pytestmark = pytest.mark.gpu
DEVICE = "cuda"


def _inputs(shape, dtype, seed):
    gen = torch.Generator(device=DEVICE).manual_seed(seed)
    L = shape[-1]
    gates = 0.99 + 0.01 * torch.rand(shape, generator=gen, device=DEVICE)
    tokens = torch.randn(shape, generator=gen, device=DEVICE) / max(L, 32) ** 0.5
    go = torch.randn(shape, generator=gen, device=DEVICE)
    return gates.to(dtype), tokens.to(dtype), go.to(dtype)


ODD_SEQLENS = [1, 2, 3, 5, 7, 9, 17, 31, 33, 100, 255, 1000, 1023, 1025, 3000, 4097, 12345]


@pytest.mark.parametrize("seqlen", ODD_SEQLENS)
@pytest.mark.parametrize("dtype", DTYPES)
def test_anylen_fwd_rev_bwd(dtype, seqlen):
    shape = (3, 5, seqlen)  # 15 rows: element count odd for odd seqlen
    g, x, go = _inputs(shape, dtype, seed=seqlen)
    g64, x64 = _np64(g), _np64(x)
    for rev in (False, True):
        y = fpscan.scan_forward_anylen(g, x, reverse=rev)
        _check(y, oracle.scan_f64(g64, x64, rev), dtype, f"fwd rev={rev}")
    gg, xx = g.clone().requires_grad_(), x.clone().requires_grad_()
    y = fpscan.pscan_anylen(gg, xx)
    dg, dt = torch.autograd.grad(y, (gg, xx), go)
    y64 = oracle.scan_f64(g64, x64)
    dg64, dt64 = oracle.scan_bwd_f64(g64, y64, _np64(go))
    _check(dt, dt64, dtype, "dtokens")
    _check(dg, dg64, dtype, "dgates")


@pytest.mark.parametrize("shape", [(1, 1, 70001), (1, 2, 100003), (2, 1, 262147),
                                   (1, 1, 3 * 65536)])
def test_anylen_long_rows(shape):
    """Beyond the reference's 65536 limit (one CTA per row here)."""
    dtype = torch.float32
    g, x, go = _inputs(shape, dtype, seed=shape[-1])
    g64, x64 = _np64(g), _np64(x)
    _check(fpscan.scan_forward_anylen(g, x), oracle.scan_f64(g64, x64), dtype, "fwd")
    _check(fpscan.scan_forward_anylen(g, x, reverse=True), oracle.scan_f64(g64, x64, True), dtype,
           "rev")
    gg, xx = g.clone().requires_grad_(), x.clone().requires_grad_()
    dg, dt = torch.autograd.grad(fpscan.pscan_anylen(gg, xx), (gg, xx), go)
    dg64, dt64 = oracle.scan_bwd_f64(g64, oracle.scan_f64(g64, x64), _np64(go))
    _check(dt, dt64, dtype, "dtokens")
    _check(dg, dg64, dtype, "dgates")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", [(64, 300, 5), (8, 1000, 37), (4, 777, 129), (3, 2001, 1)])
def test_anylen_many_rows(dtype, shape):
    """Many short rows: several tiles per launch, rows straddling vectors,
    thread groups and chunks."""
    g, x, go = _inputs(shape, dtype, seed=sum(shape))
    g64, x64 = _np64(g), _np64(x)
    _check(fpscan.scan_forward_anylen(g, x), oracle.scan_f64(g64, x64), dtype, "fwd")
    _check(fpscan.scan_forward_anylen(g, x, reverse=True), oracle.scan_f64(g64, x64, True), dtype,
           "rev")
    gg, xx = g.clone().requires_grad_(), x.clone().requires_grad_()
    dg, dt = torch.autograd.grad(fpscan.pscan_anylen(gg, xx), (gg, xx), go)
    dg64, dt64 = oracle.scan_bwd_f64(g64, oracle.scan_f64(g64, x64), _np64(go))
    _check(dt, dt64, dtype, "dtokens")
    _check(dg, dg64, dtype, "dgates")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("seqlen", [32, 1024, 65536])
def test_anylen_agrees_with_pow2_path(dtype, seqlen):
    """On the reference's own seqlens both paths compute the same scan."""
    g, x, go = _inputs((2, 16, seqlen), dtype, seed=seqlen + 1)
    for rev in (False, True):
        a = fpscan.scan_forward_anylen(g, x, reverse=rev).double()
        b = fpscan.scan_forward(g, x, reverse=rev).double()
        assert oracle.normwise_error(a.cpu().numpy(), b.cpu().numpy()) <= (
            2e-6 if dtype == torch.float32 else 1e-2)
    y = fpscan.scan_forward(g, x)
    da = fpscan.ops.scan_backward_anylen(g, y, go)
    db = fpscan.ops.scan_backward(g, y, go)
    for u, v in zip(da, db):
        assert oracle.normwise_error(u.double().cpu().numpy(), v.double().cpu().numpy()) <= (
            2e-6 if dtype == torch.float32 else 1e-2)


def test_anylen_in_place_and_out():
    g, x, _ = _inputs((5, 7, 333), torch.float32, seed=3)
    ref = oracle.scan_f64(_np64(g), _np64(x))
    out = torch.empty_like(x)
    r = fpscan.scan_forward_anylen(g, x, out=out)
    assert r is out
    _check(out, ref, torch.float32, "out=")
    xi = x.clone()
    fpscan.scan_forward_anylen(g, xi, out=xi)
    _check(xi, ref, torch.float32, "in place")


def test_anylen_rows_isolated_from_nonfinite_neighbours():
    """A row that overflows to inf (or holds NaN) must not leak into the
    next row, which starts inside the same 16-byte vector."""
    shape = (1, 6, 13)
    g, x, go = _inputs(shape, torch.float32, seed=11)
    g[0, 1] = 1e30
    x[0, 1] = 1e30  # row 1 overflows to inf
    x[0, 3, 5] = float("nan")
    y = fpscan.scan_forward_anylen(g, x)
    yr = fpscan.scan_forward_anylen(g, x, reverse=True)
    g64, x64 = _np64(g), _np64(x)
    ref, refr = oracle.scan_f64(g64, x64), oracle.scan_f64(g64, x64, True)
    for r in (0, 2, 4, 5):
        np.testing.assert_allclose(_np64(y)[0, r], ref[0, r], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(_np64(yr)[0, r], refr[0, r], rtol=1e-5, atol=1e-6)
    gg, xx = g.clone().requires_grad_(), x.clone().requires_grad_()
    dg, dt = torch.autograd.grad(fpscan.pscan_anylen(gg, xx), (gg, xx), go)
    dg64, dt64 = oracle.scan_bwd_f64(g64, ref, _np64(go))
    for r in (0, 2, 4, 5):
        np.testing.assert_allclose(_np64(dt)[0, r], dt64[0, r], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(_np64(dg)[0, r], dg64[0, r], rtol=1e-5, atol=1e-6)


def test_anylen_linearity_large():
    """Size-independent property at a large odd shape: the scan is linear in
    tokens (bit-exact doubling is not guaranteed, so compare normwise)."""
    shape = (3, 1001, 9999)
    g, x, _ = _inputs(shape, torch.float32, seed=5)
    y1 = fpscan.scan_forward_anylen(g, x)
    y2 = fpscan.scan_forward_anylen(g, 2 * x)
    assert oracle.normwise_error((y2 / 2).double().cpu().numpy(), y1.double().cpu().numpy()) <= 1e-6
    rows = [0, 517, 3002]
    flat_g, flat_x = g.reshape(-1, shape[-1]), x.reshape(-1, shape[-1])
    ref = oracle.scan_f64(_np64(flat_g[rows])[None], _np64(flat_x[rows])[None])[0]
    got = y1.reshape(-1, shape[-1])[rows]
    _check(got, ref, torch.float32, "sampled rows")


def test_anylen_errors():
    g, x, _ = _inputs((2, 3, 10), torch.float32, seed=0)
    with pytest.raises(RuntimeError):
        fpscan.scan_forward_anylen(g.transpose(1, 2), x.transpose(1, 2))
    with pytest.raises(RuntimeError):
        fpscan.scan_forward_anylen(g, x[..., :9].contiguous())
    with pytest.raises(RuntimeError):
        fpscan.scan_forward_anylen(g[..., :0], x[..., :0])
    # the strict entry points keep the reference's power-of-two rule
    with pytest.raises(RuntimeError):
        fpscan.scan_forward(g, x)
