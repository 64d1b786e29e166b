"""Guard bands around the outputs of every kernel family (a stand-in for the
memory checkers that are closed on the GPU pool).

Each case calls one C-ABI entry point with its outputs placed inside larger
buffers whose bands before and after hold a canary bit pattern
(tests/guard.py), then checks that the bands are intact and that the
outputs match the float64 oracle.  The shapes are chosen to reach the edges
where a stray write would come from: partial last vectors and row heads in
the middle of a vector (any seqlen), rows outside [0, L) read through TMA
with zero fill (channel-last), halo vectors of the fused backward, short
rows packed several to a chunk, split-row look-back tiles, per-row carry
arrays of the sequence-shard steps.
"""
import numpy as np
import pytest
import torch

import oracle
from fpscan_b200 import _lib
from guard import guarded

pytestmark = pytest.mark.gpu

CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
NORM = {torch.float32: 1e-5, torch.float16: 1e-2, torch.bfloat16: 1e-2}


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


def _close(got, ref, dtype, what):
    err = oracle.normwise_error(_np(got), ref)
    assert err <= NORM[dtype], f"{what}: normwise error {err:.3e}"


@pytest.mark.parametrize("dtype,shape", [
    (torch.float32, (2, 3, 65536)),   # multi-chunk rows
    (torch.bfloat16, (3, 5, 4096)),
    (torch.float16, (1, 7, 64)),      # short rows packed into one chunk
    (torch.float32, (2, 2, 32)),      # direct-load variant
    (torch.float32, (64, 40, 512)),   # claimed row units
])
def test_forward_reverse_backward(dtype, shape):
    lib = _lib.load()
    b, d, L = shape
    g, x, go = _inputs(shape, dtype, seed=L + d)
    for rev in (0, 1):
        out = guarded(shape, dtype)
        _lib.check(lib.fpscan_scan_fwd(g.data_ptr(), x.data_ptr(), out.out.data_ptr(), b, d, L,
                                       CODES[dtype], rev, _s()), "fwd")
        out.check(f"fwd rev={rev}")
        _close(out.out, oracle.scan_f64(_np(g), _np(x), reverse=bool(rev)), dtype, "fwd")
    yf = guarded(shape, dtype)
    _lib.check(lib.fpscan_scan_fwd(g.data_ptr(), x.data_ptr(), yf.out.data_ptr(), b, d, L,
                                   CODES[dtype], 0, _s()), "fwd")
    y = yf.out
    dg, dt = guarded(shape, dtype), guarded(shape, dtype)
    _lib.check(lib.fpscan_scan_bwd(g.data_ptr(), y.data_ptr(), go.data_ptr(), dg.out.data_ptr(),
                                   dt.out.data_ptr(), b, d, L, CODES[dtype], _s()), "bwd")
    dg.check("bwd dgates")
    dt.check("bwd dtokens")
    dg64, dt64 = oracle.scan_bwd_f64(_np(g), _np(y), _np(go))
    _close(dt.out, dt64, dtype, "dtokens")
    _close(dg.out, dg64, dtype, "dgates")


@pytest.mark.parametrize("act", [1, 2, 3])
def test_gated_forward_backward(act):
    lib = _lib.load()
    dtype, shape = torch.bfloat16, (2, 16, 8192)
    b, d, L = shape
    gen = torch.Generator(device="cuda").manual_seed(act)
    z = (torch.randn(shape, generator=gen, device="cuda") * 0.5 + (-3.0 if act == 3 else 1.0)
         ).to(dtype)
    _, x, go = _inputs(shape, dtype, seed=act + 50)
    y = guarded(shape, dtype)
    _lib.check(lib.fpscan_scan_fwd_act(z.data_ptr(), x.data_ptr(), y.out.data_ptr(), b, d, L,
                                       CODES[dtype], 0, act, _s()), "fwd_act")
    y.check("fwd_act")
    dz, dt = guarded(shape, dtype), guarded(shape, dtype)
    _lib.check(lib.fpscan_scan_bwd_act(z.data_ptr(), y.out.data_ptr(), go.data_ptr(),
                                       dz.out.data_ptr(), dt.out.data_ptr(), b, d, L,
                                       CODES[dtype], act, _s()), "bwd_act")
    dz.check("bwd_act dz")
    dt.check("bwd_act dtokens")
    zf = z.double()
    gate = {1: torch.sigmoid(zf), 2: torch.exp(-torch.nn.functional.softplus(zf)),
            3: torch.exp(zf)}[act]
    _close(y.out, oracle.scan_f64(_np(gate), _np(x)), dtype, "gated forward")


def test_initial_state():
    lib = _lib.load()
    dtype, shape = torch.float32, (2, 5, 8192)
    b, d, L = shape
    g, x, _ = _inputs(shape, dtype, seed=9)
    h0 = torch.randn(b * d, device="cuda")
    for rev in (0, 1):
        y = guarded(shape, dtype)
        _lib.check(lib.fpscan_scan_fwd_init(g.data_ptr(), x.data_ptr(), y.out.data_ptr(),
                                            h0.data_ptr(), b, d, L, 0, rev, _s()), "fwd_init")
        y.check(f"fwd_init rev={rev}")
        gg, xx = _np(g).reshape(-1, L), _np(x).reshape(-1, L)
        if rev:
            gg, xx = gg[:, ::-1], xx[:, ::-1]
        acc = _np(h0).copy()
        ref = np.empty_like(xx)
        for t in range(L):
            acc = gg[:, t] * acc + xx[:, t]
            ref[:, t] = acc
        if rev:
            ref = ref[:, ::-1]
        _close(y.out.reshape(-1, L), ref, dtype, "init")


@pytest.mark.parametrize("dtype,shape", [
    (torch.bfloat16, (3, 7, 1001)),   # rows start mid-vector, partial last vector
    (torch.float32, (1, 3, 12345)),
    (torch.float16, (2, 1, 3)),       # fewer elements than one vector
    (torch.float32, (5, 1, 1)),
])
def test_any_seqlen_forward_backward(dtype, shape):
    lib = _lib.load()
    b, d, L = shape
    g, x, go = _inputs(shape, dtype, seed=L)
    for rev in (0, 1):
        y = guarded(shape, dtype)
        _lib.check(lib.fpscan_scan_fwd_anylen(g.data_ptr(), x.data_ptr(), y.out.data_ptr(), b, d,
                                              L, CODES[dtype], rev, _s()), "fwd_anylen")
        y.check(f"fwd_anylen rev={rev}")
        _close(y.out, oracle.scan_f64(_np(g), _np(x), reverse=bool(rev)), dtype, "anylen")
    yf = guarded(shape, dtype)
    _lib.check(lib.fpscan_scan_fwd_anylen(g.data_ptr(), x.data_ptr(), yf.out.data_ptr(), b, d, L,
                                          CODES[dtype], 0, _s()), "fwd_anylen")
    dg, dt = guarded(shape, dtype), guarded(shape, dtype)
    _lib.check(lib.fpscan_scan_bwd_anylen(g.data_ptr(), yf.out.data_ptr(), go.data_ptr(),
                                          dg.out.data_ptr(), dt.out.data_ptr(), b, d, L,
                                          CODES[dtype], _s()), "bwd_anylen")
    dg.check("bwd_anylen dgates")
    dt.check("bwd_anylen dtokens")
    dg64, dt64 = oracle.scan_bwd_f64(_np(g), _np(yf.out), _np(go))
    _close(dt.out, dt64, dtype, "anylen dtokens")
    _close(dg.out, dg64, dtype, "anylen dgates")


@pytest.mark.parametrize("dtype,shape", [
    (torch.bfloat16, (2, 777, 64)),    # streaming: seqlen not a multiple of the tile rows
    (torch.float32, (1, 3001, 8)),     # few columns: time-segmented
    (torch.float32, (4, 129, 256)),
])
def test_channels_last_forward_backward(dtype, shape):
    lib = _lib.load()
    b, L, d = shape
    g, x, go = _inputs(shape, dtype, seed=L + d)

    def ws(backward):
        n = lib.fpscan_cl_workspace_bytes(b, L, d, CODES[dtype], backward)
        return torch.zeros(max(n, 16), dtype=torch.uint8, device="cuda")

    def t(a):  # (b, L, d) -> rows along the last axis
        return np.ascontiguousarray(np.swapaxes(_np(a), 1, 2))

    for rev in (0, 1):
        y, w = guarded(shape, dtype), ws(0)
        _lib.check(lib.fpscan_scan_fwd_cl(g.data_ptr(), x.data_ptr(), y.out.data_ptr(), b, L, d,
                                          CODES[dtype], rev, w.data_ptr(), w.numel(), _s()),
                   "fwd_cl")
        y.check(f"fwd_cl rev={rev}")
        ref = oracle.scan_f64(t(g), t(x), reverse=bool(rev))
        err = oracle.normwise_error(t(y.out), ref)
        assert err <= NORM[dtype], err
    yf, w = guarded(shape, dtype), ws(0)
    _lib.check(lib.fpscan_scan_fwd_cl(g.data_ptr(), x.data_ptr(), yf.out.data_ptr(), b, L, d,
                                      CODES[dtype], 0, w.data_ptr(), w.numel(), _s()), "fwd_cl")
    dg, dt, w = guarded(shape, dtype), guarded(shape, dtype), ws(1)
    _lib.check(lib.fpscan_scan_bwd_cl(g.data_ptr(), yf.out.data_ptr(), go.data_ptr(),
                                      dg.out.data_ptr(), dt.out.data_ptr(), b, L, d, CODES[dtype],
                                      w.data_ptr(), w.numel(), _s()), "bwd_cl")
    dg.check("bwd_cl dgates")
    dt.check("bwd_cl dtokens")
    dg64, dt64 = oracle.scan_bwd_f64(t(g), t(yf.out), t(go))
    assert oracle.normwise_error(t(dt.out), dt64) <= NORM[dtype]
    assert oracle.normwise_error(t(dg.out), dg64) <= NORM[dtype]


def test_sequence_shard_steps():
    """Reduce, combine and scan-with-state steps of the all-gather mode (two
    shards emulated on one GPU), every output and carry array guarded."""
    lib = _lib.load()
    dtype, rows, L = torch.float32, 6, 4096
    g, x, go = _inputs((1, rows, 2 * L), dtype, seed=12)
    parts = [(g[..., :L].contiguous(), x[..., :L].contiguous(), go[..., :L].contiguous()),
             (g[..., L:].contiguous(), x[..., L:].contiguous(), go[..., L:].contiguous())]
    gathered = torch.empty(2, 2, rows, device="cuda")
    for r, (gr, xr, _) in enumerate(parts):
        ca, cb = guarded((rows,), torch.float32), guarded((rows,), torch.float32)
        _lib.check(lib.fpscan_shard_fwd_reduce(gr.data_ptr(), xr.data_ptr(), ca.out.data_ptr(),
                                               cb.out.data_ptr(), rows, L, 0, _s()), "reduce")
        ca.check("reduce A")
        cb.check("reduce B")
        gathered[r, 0], gathered[r, 1] = ca.out, cb.out
    init = guarded((rows,), torch.float32)
    _lib.check(lib.fpscan_carry_combine(gathered.data_ptr(), 2, 1, rows, 0, init.out.data_ptr(),
                                        _s()), "combine")
    init.check("combine")
    y1 = guarded((1, rows, L), dtype)
    g1, x1, go1 = parts[1]
    _lib.check(lib.fpscan_shard_fwd_scan(g1.data_ptr(), x1.data_ptr(), y1.out.data_ptr(),
                                         init.out.data_ptr(), rows, L, 0, _s()), "shard scan")
    y1.check("shard scan")
    y64 = oracle.scan_f64(_np(g), _np(x))
    _close(y1.out, y64[..., L:], dtype, "second shard")
    v = guarded((rows,), torch.float32)
    _lib.check(lib.fpscan_shard_bwd_reduce(g1.data_ptr(), go1.data_ptr(), v.out.data_ptr(), rows,
                                           L, 0, _s()), "bwd reduce")
    v.check("bwd reduce")
    y0 = torch.empty_like(x1)
    g0, x0, go0 = parts[0]
    _lib.check(lib.fpscan_scan_fwd(g0.data_ptr(), x0.data_ptr(), y0.data_ptr(), 1, rows, L, 0, 0,
                                   _s()), "fwd")
    dg, dt = guarded((1, rows, L), dtype), guarded((1, rows, L), dtype)
    zero = torch.zeros(rows, device="cuda")
    _lib.check(lib.fpscan_shard_bwd_scan(g0.data_ptr(), y0.data_ptr(), go0.data_ptr(),
                                         dg.out.data_ptr(), dt.out.data_ptr(), v.out.data_ptr(),
                                         zero.data_ptr(), rows, L, 0, _s()), "shard bwd scan")
    dg.check("shard bwd dgates")
    dt.check("shard bwd dtokens")
    dg64, dt64 = oracle.scan_bwd_f64(_np(g), y64, _np(go))
    _close(dt.out, dt64[..., :L], dtype, "first shard dtokens")
    _close(dg.out, dg64[..., :L], dtype, "first shard dgates")
