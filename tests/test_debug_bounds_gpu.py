"""The bounds-checking build (libfpscan_b200_debug.so, -DFPSCAN_DEBUG_BOUNDS),
a stand-in for the memory checkers that are closed on the GPU pool.

In that build every kernel checks each global access it computes itself --
bulk-copy sources with their halos, direct loads, vector and element
stores, carry arrays -- against its tensor's extent and alignment, skips one
outside and sets status bit 16.  These tests first show that the checker is
live (a probe address just past an extent sets the bit in the debug build
and not in the release build), then run every kernel family through the
debug build at edge shapes and require a clean status and results equal to
the float64 oracle.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

import oracle
from fpscan_b200 import _lib, build

pytestmark = pytest.mark.gpu
BOUNDS = 16
CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
TOL = {torch.float32: 1e-5, torch.float16: 1e-2, torch.bfloat16: 1e-2}


@pytest.fixture(scope="module")
def dbg():
    if not os.path.exists(build.DEBUG_LIB_PATH):
        pytest.skip("bounds-checking build not present (fpscan_b200.build.build_debug)")
    return _lib.open_library(build.DEBUG_LIB_PATH)


def _status(lib):
    v = ctypes.c_uint(0)
    torch.cuda.synchronize()
    _lib.check(lib.fpscan_device_status(ctypes.byref(v), 1), "fpscan_device_status")
    return int(v.value)


def _s():
    return torch.cuda.current_stream().cuda_stream


def _inputs(shape, dtype, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    g = (0.95 + 0.05 * torch.rand(shape, generator=gen, device="cuda")).to(dtype)
    x = (torch.randn(shape, generator=gen, device="cuda") / shape[-1] ** 0.5).to(dtype)
    go = torch.randn(shape, generator=gen, device="cuda").to(dtype)
    return g, x, go


def _np(t):
    return t.detach().double().cpu().numpy()


def test_checker_is_live(dbg):
    rel = _lib.load()
    _status(dbg)
    assert dbg.fpscan_debug_bounds(_s()) == 1
    assert _status(dbg) & BOUNDS
    _lib.device_status(clear=True)
    assert rel.fpscan_debug_bounds(_s()) == 0
    assert _lib.device_status(clear=True) == 0


@pytest.mark.parametrize("dtype,shape", [
    (torch.float32, (2, 3, 65536)), (torch.bfloat16, (1, 7, 64)), (torch.float16, (2, 2, 32)),
    (torch.float32, (64, 40, 512)), (torch.bfloat16, (1, 8, 65536))])
def test_forward_backward_and_split_paths(dbg, dtype, shape):
    b, d, L = shape
    code = CODES[dtype]
    g, x, go = _inputs(shape, dtype, seed=L + d)
    _status(dbg)
    y = torch.empty_like(x)
    for rev in (0, 1):
        ref = oracle.scan_f64(_np(g), _np(x), reverse=bool(rev))
        _lib.check(dbg.fpscan_scan_fwd(g.data_ptr(), x.data_ptr(), y.data_ptr(), b, d, L, code, rev,
                                       _s()), "fwd")
        assert oracle.normwise_error(_np(y), ref) <= TOL[dtype]
        need = dbg.fpscan_scan_fwd_workspace_bytes(b, d, L, code)
        ws = torch.zeros(max(need, 16), dtype=torch.uint8, device="cuda")
        _lib.check(dbg.fpscan_scan_fwd_ws(g.data_ptr(), x.data_ptr(), y.data_ptr(), b, d, L, code,
                                          rev, ws.data_ptr(), ws.numel(), _s()), "fwd_ws")
        assert oracle.normwise_error(_np(y), ref) <= TOL[dtype]
    _lib.check(dbg.fpscan_scan_fwd(g.data_ptr(), x.data_ptr(), y.data_ptr(), b, d, L, code, 0,
                                   _s()), "fwd")
    dg64, dt64 = oracle.scan_bwd_f64(_np(g), _np(y), _np(go))
    dg, dt = torch.empty_like(x), torch.empty_like(x)
    _lib.check(dbg.fpscan_scan_bwd(g.data_ptr(), y.data_ptr(), go.data_ptr(), dg.data_ptr(),
                                   dt.data_ptr(), b, d, L, code, _s()), "bwd")
    assert oracle.normwise_error(_np(dt), dt64) <= TOL[dtype]
    assert oracle.normwise_error(_np(dg), dg64) <= TOL[dtype]
    need = dbg.fpscan_scan_bwd_workspace_bytes(b, d, L, code)
    ws = torch.zeros(max(need, 16), dtype=torch.uint8, device="cuda")
    _lib.check(dbg.fpscan_scan_bwd_ws(g.data_ptr(), y.data_ptr(), go.data_ptr(), dg.data_ptr(),
                                      dt.data_ptr(), b, d, L, code, ws.data_ptr(), ws.numel(),
                                      _s()), "bwd_ws")
    assert oracle.normwise_error(_np(dt), dt64) <= TOL[dtype]
    assert oracle.normwise_error(_np(dg), dg64) <= TOL[dtype]
    assert _status(dbg) == 0


@pytest.mark.parametrize("dtype,shape", [(torch.bfloat16, (3, 7, 1001)),
                                         (torch.float32, (1, 3, 12345)),
                                         (torch.float16, (2, 1, 3))])
def test_any_seqlen(dbg, dtype, shape):
    b, d, L = shape
    code = CODES[dtype]
    g, x, go = _inputs(shape, dtype, seed=L)
    _status(dbg)
    y = torch.empty_like(x)
    _lib.check(dbg.fpscan_scan_fwd_anylen(g.data_ptr(), x.data_ptr(), y.data_ptr(), b, d, L, code,
                                          0, _s()), "fwd_anylen")
    assert oracle.normwise_error(_np(y), oracle.scan_f64(_np(g), _np(x))) <= TOL[dtype]
    dg, dt = torch.empty_like(x), torch.empty_like(x)
    _lib.check(dbg.fpscan_scan_bwd_anylen(g.data_ptr(), y.data_ptr(), go.data_ptr(), dg.data_ptr(),
                                          dt.data_ptr(), b, d, L, code, _s()), "bwd_anylen")
    dg64, dt64 = oracle.scan_bwd_f64(_np(g), _np(y), _np(go))
    assert oracle.normwise_error(_np(dt), dt64) <= TOL[dtype]
    assert oracle.normwise_error(_np(dg), dg64) <= TOL[dtype]
    assert _status(dbg) == 0


@pytest.mark.parametrize("dtype,shape", [(torch.bfloat16, (2, 777, 64)),
                                         (torch.float32, (1, 3001, 8))])
def test_channels_last(dbg, dtype, shape):
    b, L, d = shape
    code = CODES[dtype]
    g, x, go = _inputs(shape, dtype, seed=L + d)
    _status(dbg)

    def ws(bwd):
        n = dbg.fpscan_cl_workspace_bytes(b, L, d, code, bwd)
        return torch.zeros(max(n, 16), dtype=torch.uint8, device="cuda")

    def t(a):
        return np.ascontiguousarray(np.swapaxes(_np(a), 1, 2))

    y, w = torch.empty_like(x), ws(0)
    _lib.check(dbg.fpscan_scan_fwd_cl(g.data_ptr(), x.data_ptr(), y.data_ptr(), b, L, d, code, 0,
                                      w.data_ptr(), w.numel(), _s()), "fwd_cl")
    assert oracle.normwise_error(t(y), oracle.scan_f64(t(g), t(x))) <= TOL[dtype]
    dg, dt, w = torch.empty_like(x), torch.empty_like(x), ws(1)
    _lib.check(dbg.fpscan_scan_bwd_cl(g.data_ptr(), y.data_ptr(), go.data_ptr(), dg.data_ptr(),
                                      dt.data_ptr(), b, L, d, code, w.data_ptr(), w.numel(),
                                      _s()), "bwd_cl")
    dg64, dt64 = oracle.scan_bwd_f64(t(g), t(y), t(go))
    assert oracle.normwise_error(t(dt), dt64) <= TOL[dtype]
    assert oracle.normwise_error(t(dg), dg64) <= TOL[dtype]
    assert _status(dbg) == 0


def test_sequence_shard_carries(dbg):
    rows, L = 6, 4096
    g, x, go = _inputs((1, rows, L), torch.float32, seed=3)
    _status(dbg)
    ca = torch.empty(rows, device="cuda")
    cb = torch.empty(rows, device="cuda")
    _lib.check(dbg.fpscan_shard_fwd_reduce(g.data_ptr(), x.data_ptr(), ca.data_ptr(),
                                           cb.data_ptr(), rows, L, 0, _s()), "reduce")
    v = torch.empty(rows, device="cuda")
    _lib.check(dbg.fpscan_shard_bwd_reduce(g.data_ptr(), go.data_ptr(), v.data_ptr(), rows, L, 0,
                                           _s()), "bwd reduce")
    y64 = oracle.scan_f64(_np(g), _np(x))
    assert oracle.normwise_error(_np(cb), y64[0, :, -1]) <= 1e-5
    assert _status(dbg) == 0
