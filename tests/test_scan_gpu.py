"""GPU parity tests: fpscan_b200 (through its C ABI) against the CPU oracle,
the golden vectors made by the reference's own code, the reference's own CUDA
kernel (built from its sources into oracle/_ref) and size-independent
properties at the BASELINE configurations.

The first block mirrors the reference's tests/test_fpscan.py case for case
(same names, inputs, seeds and tolerances).  On top of the reference's
assert_close tolerances every comparison with the float64 oracle also checks
the normwise bound max|got-ref|/max|ref| <= 1e-5 (fp32) / 1e-2 (fp16, bf16).
"""
import json
import os

import numpy as np
import pytest
import torch

import fpscan_b200 as fpscan
import oracle
from fpscan_b200 import _lib

pytestmark = pytest.mark.gpu
DEVICE = "cuda"
HERE = os.path.dirname(os.path.abspath(__file__))

ALL_SEQLENS = [32, 64, 128, 256, 512, 1024, 2048, 4096, 8192, 16384, 32768, 65536]
HALF_SEQLENS = [32, 64, 128, 256, 512, 1024, 2048, 4096]
DTYPES = [torch.float32, torch.float16, torch.bfloat16]

# reference tests/test_fpscan.py:18-22
TOL = {
    torch.float32: dict(atol=2e-3, rtol=2e-3),
    torch.float16: dict(atol=3e-2, rtol=3e-2),
    torch.bfloat16: dict(atol=6e-2, rtol=6e-2),
}
# north-star normwise tolerance vs float64
NORM_TOL = {torch.float32: 1e-5, torch.float16: 1e-2, torch.bfloat16: 1e-2}


def _make_inputs(batch, dim, seqlen, dtype, seed=0):
    # reference tests/test_fpscan.py:25-29
    gen = torch.Generator(device=DEVICE).manual_seed(seed)
    gates = 0.99 + 0.01 * torch.rand(batch, dim, seqlen, generator=gen, device=DEVICE)
    tokens = torch.randn(batch, dim, seqlen, generator=gen, device=DEVICE) / seqlen
    return gates.to(dtype).contiguous(), tokens.to(dtype).contiguous()


def _np64(t):
    return t.detach().double().cpu().numpy()


def _check(got, ref, dtype, what=""):
    ref_t = torch.from_numpy(np.asarray(ref, dtype=np.float64))
    got_t = got.detach().double().cpu()
    torch.testing.assert_close(got_t, ref_t, **TOL[dtype])
    err = oracle.normwise_error(got_t.numpy(), ref_t.numpy())
    assert err <= NORM_TOL[dtype], f"{what} normwise error {err:.3e} > {NORM_TOL[dtype]}"


def _assert_normwise(got, ref, dtype, what=""):
    err = oracle.normwise_error(got.detach().double().cpu().numpy(), np.asarray(ref, np.float64))
    assert err <= NORM_TOL[dtype], f"{what} normwise error {err:.3e} > {NORM_TOL[dtype]}"


def _dtype_seqlens():
    for seqlen in ALL_SEQLENS:
        yield torch.float32, seqlen
    for seqlen in HALF_SEQLENS:
        yield torch.float16, seqlen
        yield torch.bfloat16, seqlen


# ----------------------------------------------------------------- reference test mirror
@pytest.mark.parametrize("dtype,seqlen", list(_dtype_seqlens()))
def test_forward_matches_oracle(dtype, seqlen):
    gates, tokens = _make_inputs(2, 4, seqlen, dtype, seed=seqlen)
    out = fpscan.scan_forward(gates, tokens)
    assert out.shape == tokens.shape
    assert out.dtype == dtype
    _check(out, oracle.scan_f64(_np64(gates), _np64(tokens)), dtype, "forward")


@pytest.mark.parametrize("seqlen", ALL_SEQLENS)
def test_reverse_matches_oracle(seqlen):
    gates, tokens = _make_inputs(2, 4, seqlen, torch.float32, seed=seqlen + 1)
    out = fpscan.scan_forward(gates, tokens, reverse=True)
    _check(out, oracle.scan_f64(_np64(gates), _np64(tokens), reverse=True), torch.float32)


@pytest.mark.parametrize("seqlen", [32, 256, 1024, 4096])
def test_agrees_with_torch_parallel_baseline(seqlen):
    gates, tokens = _make_inputs(2, 4, seqlen, torch.float32, seed=seqlen + 2)
    out = fpscan.scan_forward(gates, tokens)
    baseline = oracle.parallel_scan_torch(gates.double(), tokens.double())
    _check(out, baseline.cpu().numpy(), torch.float32)


@pytest.mark.parametrize("seqlen", [32, 128, 512, 2048, 8192])
def test_backward_matches_oracle(seqlen):
    gates, tokens = _make_inputs(2, 4, seqlen, torch.float32, seed=seqlen + 3)
    g = gates.clone().requires_grad_()
    x = tokens.clone().requires_grad_()
    grad_seed = torch.Generator(device=DEVICE).manual_seed(seqlen + 4)
    weight = torch.randn(*tokens.shape, generator=grad_seed, device=DEVICE)
    out = fpscan.pscan(g, x)
    (out * weight).sum().backward()
    y64 = oracle.scan_f64(_np64(gates), _np64(tokens))
    dg, dt = oracle.scan_bwd_f64(_np64(gates), y64, _np64(weight))
    _check(g.grad, dg, torch.float32, "dgates")
    _check(x.grad, dt, torch.float32, "dtokens")


def test_non_power_of_two_seqlen_raises():
    gates, tokens = _make_inputs(1, 1, 32, torch.float32)
    with pytest.raises(RuntimeError):
        fpscan.scan_forward(gates[..., :30].contiguous(), tokens[..., :30].contiguous())


def test_non_contiguous_raises():
    gates, tokens = _make_inputs(2, 4, 64, torch.float32)
    with pytest.raises(RuntimeError):
        fpscan.scan_forward(gates.transpose(1, 2), tokens.transpose(1, 2))


# ----------------------------------------------------------------- beyond the reference's tests
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("seqlen", [32, 512, 8192, 65536])
def test_reverse_half(dtype, seqlen):
    gates, tokens = _make_inputs(2, 3, seqlen, dtype, seed=seqlen + 9)
    out = fpscan.scan_forward(gates, tokens, reverse=True)
    _check(out, oracle.scan_f64(_np64(gates), _np64(tokens), reverse=True), dtype, "reverse")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("seqlen", [32, 64, 256, 1024, 2048, 4096, 16384, 65536])
def test_backward_all_dtypes(dtype, seqlen):
    gates, tokens = _make_inputs(3, 5, seqlen, dtype, seed=seqlen + 13)
    gen = torch.Generator(device=DEVICE).manual_seed(seqlen)
    go = torch.randn(3, 5, seqlen, generator=gen, device=DEVICE).to(dtype)
    g = gates.clone().requires_grad_()
    x = tokens.clone().requires_grad_()
    y = fpscan.pscan(g, x)
    dg_t, dt_t = torch.autograd.grad(y, (g, x), go)
    y64 = oracle.scan_f64(_np64(gates), _np64(tokens))
    _check(y, y64, dtype, "y")
    dg, dt = oracle.scan_bwd_f64(_np64(gates), y64, _np64(go))
    _check(dt_t, dt, dtype, "dtokens")
    _check(dg_t, dg, dtype, "dgates")


@pytest.mark.parametrize("batch,dim", [(1, 1), (1, 3), (3, 5), (2, 37), (5, 300)])
@pytest.mark.parametrize("seqlen", [32, 128, 1024, 4096])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_ragged_row_counts(batch, dim, seqlen, dtype):
    # row counts that leave partial tiles / partial chunks
    gates, tokens = _make_inputs(batch, dim, seqlen, dtype, seed=batch * 1000 + dim)
    for rev in (False, True):
        out = fpscan.scan_forward(gates, tokens, reverse=rev)
        _check(out, oracle.scan_f64(_np64(gates), _np64(tokens), reverse=rev), dtype)


@pytest.mark.parametrize("name", [c["name"] for c in json.load(
    open(os.path.join(HERE, "golden", "golden_meta.json")))["cases"]])
def test_golden_vectors(name):
    gold = np.load(os.path.join(HERE, "golden", "golden.npz"))
    dtype = getattr(torch, name.split("_")[1])
    g = torch.from_numpy(gold[f"{name}/gates"]).to(DEVICE, dtype)
    x = torch.from_numpy(gold[f"{name}/tokens"]).to(DEVICE, dtype)
    _check(fpscan.scan_forward(g, x), gold[f"{name}/y"], dtype, name)
    if f"{name}/y_rev" in gold.files:
        _check(fpscan.scan_forward(g, x, reverse=True), gold[f"{name}/y_rev"], dtype, name)
    if f"{name}/dgates" in gold.files:
        go = torch.from_numpy(gold[f"{name}/grad_out"]).to(DEVICE, dtype)
        gg, xx = g.clone().requires_grad_(), x.clone().requires_grad_()
        dg, dt = torch.autograd.grad(fpscan.pscan(gg, xx), (gg, xx), go)
        _check(dt, gold[f"{name}/dtokens"], dtype, name + " dtokens")
        _check(dg, gold[f"{name}/dgates"], dtype, name + " dgates")


def test_out_argument_and_in_place():
    gates, tokens = _make_inputs(2, 4, 1024, torch.float32, seed=3)
    ref = oracle.scan_f64(_np64(gates), _np64(tokens))
    out = torch.empty_like(tokens)
    assert fpscan.scan_forward(gates, tokens, out=out) is out
    _check(out, ref, torch.float32)
    t2 = tokens.clone()
    fpscan.scan_forward(gates, t2, out=t2)  # in place over tokens
    _check(t2, ref, torch.float32)


def test_empty_batch():
    g = torch.empty(0, 4, 64, device=DEVICE)
    assert fpscan.scan_forward(g, g).shape == (0, 4, 64)


def test_first_gate_is_ignored_like_reference():
    # reference kernel forces the first gate to 1 (csrc/full_scan/full_scan.cu:96)
    gates, tokens = _make_inputs(2, 3, 4096, torch.float32, seed=1)
    gates[..., 0] = float("inf")
    out = fpscan.scan_forward(gates, tokens)
    g = _np64(gates)
    g[..., 0] = 0.0
    _check(out, oracle.scan_f64(g, _np64(tokens)), torch.float32)
    gates, tokens = _make_inputs(2, 3, 4096, torch.float32, seed=2)
    gates[..., -1] = float("nan")
    out = fpscan.scan_forward(gates, tokens, reverse=True)
    g = _np64(gates)
    g[..., -1] = 0.0
    _check(out, oracle.scan_f64(g, _np64(tokens), reverse=True), torch.float32)


def test_mismatched_dtype_raises():
    gates, tokens = _make_inputs(1, 2, 64, torch.float32)
    with pytest.raises(RuntimeError):
        fpscan.scan_forward(gates.half(), tokens)


def test_reference_extension_shim_contract():
    from fpscan_b200 import _C

    gates, tokens = _make_inputs(2, 4, 256, torch.float32, seed=4)
    out = torch.empty_like(tokens)
    ret = _C.fullscan_forward(gates, tokens, out, True)
    assert ret is out
    _check(out, oracle.scan_f64(_np64(gates), _np64(tokens), reverse=True), torch.float32)


# ----------------------------------------------------------------- vs the reference's kernel
_REF = oracle.load_reference_kernel()


@pytest.mark.skipif(_REF is None, reason="reference kernel not built (oracle/build_ref.py)")
@pytest.mark.parametrize("dtype,seqlen", [(torch.float32, L) for L in ALL_SEQLENS]
                         + [(torch.bfloat16, L) for L in (32, 1024, 8192)]
                         + [(torch.float16, L) for L in (64, 4096)])
def test_agrees_with_reference_kernel(dtype, seqlen):
    gates, tokens = _make_inputs(2, 8, seqlen, dtype, seed=seqlen + 21)
    for rev in (False, True):
        ref = torch.empty_like(tokens)
        _REF.fullscan_forward(gates, tokens, ref, rev)
        out = fpscan.scan_forward(gates, tokens, reverse=rev)
        torch.testing.assert_close(out.double(), ref.double(), **TOL[dtype])
        assert oracle.normwise_error(_np64(out), _np64(ref)) <= NORM_TOL[dtype]


@pytest.mark.skipif(_REF is None, reason="reference kernel not built (oracle/build_ref.py)")
@pytest.mark.parametrize("dtype,shape,cfg3", [
    (torch.bfloat16, (4, 64, 8192), False),
    (torch.float16, (8, 2048, 8192), True),   # BASELINE config 3, fp16
    (torch.bfloat16, (8, 2048, 8192), True),  # BASELINE config 3, bf16
])
def test_backward_agrees_with_reference_composition(dtype, shape, cfg3):
    """The fused backward against the reference's own backward composition
    (fpscan/ops.py:70-83: shift, reverse scan, multiply) run on the
    reference's kernel; config-3 cases use that config's distributions."""
    if cfg3:
        gen = torch.Generator(device=DEVICE).manual_seed(3)
        gates = torch.sigmoid(torch.randn(shape, generator=gen, device=DEVICE) + 2).to(dtype)
        tokens = (torch.randn(shape, generator=gen, device=DEVICE) * 0.1).to(dtype)
    else:
        gates, tokens = _make_inputs(*shape, dtype, seed=77)
    gen = torch.Generator(device=DEVICE).manual_seed(78)
    go = torch.randn(shape, generator=gen, device=DEVICE).to(dtype)

    def ref_scan(g, x, rev):
        o = torch.empty_like(x)
        _REF.fullscan_forward(g, x, o, rev)
        return o

    y_ref = ref_scan(gates, tokens, False)
    dg_ref, dt_ref = oracle.pscan_backward_formula(gates, y_ref, go, ref_scan)
    y = fpscan.scan_forward(gates, tokens)
    dg, dt = fpscan.scan_backward(gates, y, go)
    for a, b in ((y, y_ref), (dt, dt_ref), (dg, dg_ref)):
        assert oracle.normwise_error(_np64(a), _np64(b)) <= 1e-2


# ----------------------------------------------------------------- BASELINE configs, full size
def _sample_rows_check(gates, tokens, y, go=None, dg=None, dt=None, n=48, tol=1e-2, seed=0):
    """Compare n random rows of a full-size run with the float64 oracle."""
    L = tokens.shape[-1]
    rows = tokens.numel() // L
    idx = torch.randperm(rows, generator=torch.Generator().manual_seed(seed))[:n].to(DEVICE)

    def pick(t):
        return _np64(t.reshape(rows, L).index_select(0, idx))

    g64, x64 = pick(gates), pick(tokens)
    y64 = oracle.scan_f64(g64, x64)
    assert oracle.normwise_error(pick(y), y64) <= tol
    if go is not None:
        dg64, dt64 = oracle.scan_bwd_f64(g64, y64, pick(go))
        assert oracle.normwise_error(pick(dt), dt64) <= tol
        assert oracle.normwise_error(pick(dg), dg64) <= tol


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_config3_mamba_like_fwd_bwd(dtype):
    # batch 8, dim 2048, seqlen 8192, gates = sigmoid(N(2,1)).
    # Every row (16384) of the forward and the fused backward against the
    # float64 oracle, in blocks of rows.
    gen = torch.Generator(device=DEVICE).manual_seed(3)
    shape = (8, 2048, 8192)
    gates = torch.sigmoid(torch.randn(shape, generator=gen, device=DEVICE) + 2).to(dtype)
    tokens = (torch.randn(shape, generator=gen, device=DEVICE) * 0.1).to(dtype)
    go = torch.randn(shape, generator=gen, device=DEVICE).to(dtype)
    y = fpscan.scan_forward(gates, tokens)
    dg, dt = fpscan.scan_backward(gates, y, go)
    L = shape[-1]
    rows = gates.numel() // L
    worst = [0.0, 0.0, 0.0]
    for lo in range(0, rows, 2048):
        blk = slice(lo, lo + 2048)
        g64 = _np64(gates.view(rows, L)[blk])
        y64 = oracle.scan_f64(g64, _np64(tokens.view(rows, L)[blk]))
        dg64, dt64 = oracle.scan_bwd_f64(g64, y64, _np64(go.view(rows, L)[blk]))
        for i, (got, ref) in enumerate(((y, y64), (dt, dt64), (dg, dg64))):
            worst[i] = max(worst[i], oracle.normwise_error(_np64(got.view(rows, L)[blk]), ref))
    assert max(worst) <= 1e-2, worst


def test_config4_full_size_bf16():
    # BASELINE config 4 (single GPU, all channels): 16 x 5120 x 16384 bf16
    gen = torch.Generator(device=DEVICE).manual_seed(4)
    shape = (16, 5120, 16384)
    z = torch.randn(shape, generator=gen, device=DEVICE) - 1
    gates = torch.exp(-torch.nn.functional.softplus(z)).to(torch.bfloat16)
    del z
    tokens = torch.randn(shape, generator=gen, device=DEVICE).to(torch.bfloat16)
    go = torch.randn(shape, generator=gen, device=DEVICE).to(torch.bfloat16)
    y = fpscan.scan_forward(gates, tokens)
    dg, dt = fpscan.scan_backward(gates, y, go)
    _sample_rows_check(gates, tokens, y, go, dg, dt, seed=4)
    # linearity of the scan in tokens (size-independent property, fp32 check)
    y2 = fpscan.scan_forward(gates, (tokens.float() * 2).to(torch.bfloat16))
    assert torch.equal(y2, (y.float() * 2).to(torch.bfloat16))


def test_config5_2g_elements_fp32():
    # BASELINE config 5 on one GPU, forward and fused backward: 4 x 8192 x
    # 65536 fp32 = 2^31 elements per tensor (beyond 32-bit element offsets,
    # including the backward's halo offsets).  Sampled rows, plus the last two
    # rows, against float64.
    gen = torch.Generator(device=DEVICE).manual_seed(5)
    shape = (4, 8192, 65536)
    gates = 0.999 + 0.001 * torch.rand(shape, generator=gen, device=DEVICE)
    tokens = torch.randn(shape, generator=gen, device=DEVICE) / 65536
    go = torch.randn(shape, generator=gen, device=DEVICE)
    y = fpscan.scan_forward(gates, tokens)
    dg, dt = fpscan.scan_backward(gates, y, go)
    _sample_rows_check(gates, tokens, y, go, dg, dt, tol=1e-5, seed=5)
    g64, x64 = _np64(gates[-1, -2:]), _np64(tokens[-1, -2:])
    last = oracle.scan_f64(g64, x64)
    assert oracle.normwise_error(_np64(y[-1, -2:]), last) <= 1e-5
    dg64, dt64 = oracle.scan_bwd_f64(g64, last, _np64(go[-1, -2:]))
    assert oracle.normwise_error(_np64(dt[-1, -2:]), dt64) <= 1e-5
    assert oracle.normwise_error(_np64(dg[-1, -2:]), dg64) <= 1e-5


@pytest.mark.parametrize("dtype", DTYPES)
def test_reverse_equals_flipped_forward(dtype):
    gates, tokens = _make_inputs(4, 33, 2048, dtype, seed=8)
    a = fpscan.scan_forward(gates, tokens, reverse=True)
    b = fpscan.scan_forward(gates.flip(-1).contiguous(), tokens.flip(-1).contiguous()).flip(-1)
    # same arithmetic in mirrored order: bit-identical
    assert torch.equal(a, b)


# ----------------------------------------------------------------- sequence-shard kernels on one GPU
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("world,L", [(2, 4096), (4, 8192), (8, 65536), (8, 256)])
def test_seq_shard_kernels_emulated(dtype, world, L):
    """The shard entry points + carry combine, with ranks emulated in a loop on
    one GPU (the all-gather replaced by stacking), against the full scan."""
    from fpscan_b200.distributed import CudaOps

    ops = CudaOps()
    gates, tokens = _make_inputs(3, 7, L, dtype, seed=L + world)
    gen = torch.Generator(device=DEVICE).manual_seed(1)
    go = torch.randn(3, 7, L, generator=gen, device=DEVICE).to(dtype)
    Lr = L // world
    sl = [slice(r * Lr, (r + 1) * Lr) for r in range(world)]
    gs = [gates[..., s].contiguous() for s in sl]
    xs = [tokens[..., s].contiguous() for s in sl]
    gos = [go[..., s].contiguous() for s in sl]
    carries = torch.stack([ops.fwd_reduce(g, x) for g, x in zip(gs, xs)])
    ys, inits = [], []
    for r in range(world):
        init = ops.combine(carries, world, r, reverse=False)
        inits.append(init)
        ys.append(ops.fwd_scan_zero(gs[r], xs[r]) if r == 0 else ops.fwd_scan(gs[r], xs[r], init))
    vs = torch.stack([torch.stack([carries[r, 0], ops.bwd_reduce(gs[r], gos[r])])
                      for r in range(world)])
    dgs, dts = [], []
    for r in range(world):
        addend = ops.combine(vs, world, r, reverse=True)
        dg, dt = ops.bwd_scan(gs[r], ys[r], gos[r], addend, inits[r])
        dgs.append(dg)
        dts.append(dt)
    y64 = oracle.scan_f64(_np64(gates), _np64(tokens))
    dg64, dt64 = oracle.scan_bwd_f64(_np64(gates), y64, _np64(go))
    _check(torch.cat(ys, -1), y64, dtype, "y")
    _check(torch.cat(dts, -1), dt64, dtype, "dtokens")
    _check(torch.cat(dgs, -1), dg64, dtype, "dgates")


def test_device_status_clean():
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0


# ----------------------------------------------------------------- non-default kernel variants
_VARIANT_SCRIPT = r"""
import sys, torch
sys.path.insert(0, {repo!r})
import fpscan_b200 as fp, oracle
errs = []
for dtype in (torch.float32, torch.bfloat16):
    for (b, d, L) in ((2, 5, 32), (3, 7, 1024), (2, 3, 8192), (1, 2, 65536)):
        g = torch.Generator(device="cuda").manual_seed(L)
        gates = (0.9 + 0.1 * torch.rand(b, d, L, generator=g, device="cuda")).to(dtype)
        x = torch.randn(b, d, L, generator=g, device="cuda").to(dtype)
        go = torch.randn(b, d, L, generator=g, device="cuda").to(dtype)
        for rev in (False, True):
            y = fp.scan_forward(gates, x, reverse=rev)
            ref = oracle.scan_f64(gates.double().cpu().numpy(), x.double().cpu().numpy(), rev)
            errs.append(oracle.normwise_error(y.double().cpu().numpy(), ref))
        y = fp.scan_forward(gates, x)
        dg, dt = fp.scan_backward(gates, y, go)
        y64 = oracle.scan_f64(gates.double().cpu().numpy(), x.double().cpu().numpy())
        dg64, dt64 = oracle.scan_bwd_f64(gates.double().cpu().numpy(), y64, go.double().cpu().numpy())
        tol = 1e-5 if dtype == torch.float32 else 1e-2
        e = max(oracle.normwise_error(dt.double().cpu().numpy(), dt64),
                oracle.normwise_error(dg.double().cpu().numpy(), dg64))
        assert e <= tol, (dtype, b, d, L, e)
        assert max(errs) <= tol, (dtype, b, d, L, max(errs))
print("ok")
"""


@pytest.mark.parametrize("nv", ["1", "2", "4"])
def test_vector_width_variants(nv):
    """FPSCAN_B200_NV selects the 1/2/4-vector kernel variants (read once per
    process, so each runs in a child process)."""
    import subprocess
    import sys

    repo = os.path.dirname(HERE)
    env = dict(os.environ, FPSCAN_B200_NV=nv)
    r = subprocess.run([sys.executable, "-c", _VARIANT_SCRIPT.format(repo=repo)], env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr


# ----------------------------------------------------------------- split-row (few rows, long L) path
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("batch,dim,seqlen", [(2, 256, 65536), (1, 1, 65536), (1, 8, 65536),
                                              (2, 16, 32768), (1, 7, 65536), (1, 64, 65536),
                                              (2, 3, 8192)])
def test_split_row_path_vs_one_cta_per_row(dtype, batch, dim, seqlen):
    """fpscan_scan_fwd_ws (rows split across CTAs, decoupled look-back) against
    fpscan_scan_fwd (one CTA per row) and the oracle, three calls in a row on
    the same workspace (epoch-tagged status words are reused)."""
    lib = _lib.load()
    code = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[dtype]
    gates, tokens = _make_inputs(batch, dim, seqlen, dtype, seed=seqlen + dim)
    ws_bytes = lib.fpscan_scan_fwd_workspace_bytes(batch, dim, seqlen, code)
    ws = torch.zeros(max(ws_bytes, 16), dtype=torch.uint8, device=DEVICE)
    stream = torch.cuda.current_stream().cuda_stream
    for rev in (False, True):
        ref = oracle.scan_f64(_np64(gates), _np64(tokens), reverse=rev)
        plain = torch.empty_like(tokens)
        _lib.check(lib.fpscan_scan_fwd(gates.data_ptr(), tokens.data_ptr(), plain.data_ptr(), batch,
                                       dim, seqlen, code, int(rev), stream), "fwd")
        for _ in range(3):
            out = torch.full_like(tokens, float("nan"))
            _lib.check(lib.fpscan_scan_fwd_ws(gates.data_ptr(), tokens.data_ptr(), out.data_ptr(),
                                              batch, dim, seqlen, code, int(rev), ws.data_ptr(),
                                              ws.numel(), stream), "fwd_ws")
            _check(out, ref, dtype, f"split rev={rev}")
            assert oracle.normwise_error(_np64(out), _np64(plain)) <= NORM_TOL[dtype]
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0


def test_split_row_workspace_checks():
    lib = _lib.load()
    gates, tokens = _make_inputs(2, 4, 65536, torch.float32)
    need = lib.fpscan_scan_fwd_workspace_bytes(2, 4, 65536, 0)
    assert need > 0
    ws = torch.zeros(need, dtype=torch.uint8, device=DEVICE)
    out = torch.empty_like(tokens)
    s = torch.cuda.current_stream().cuda_stream
    assert lib.fpscan_scan_fwd_ws(gates.data_ptr(), tokens.data_ptr(), out.data_ptr(), 2, 4, 65536,
                                  0, 0, ws.data_ptr(), need - 16, s) == 1
    assert b"workspace" in lib.fpscan_last_error()
    assert lib.fpscan_scan_fwd_ws(gates.data_ptr(), tokens.data_ptr(), out.data_ptr(), 2, 4, 65536,
                                  0, 0, 0, 0, s) == 1
    # many rows: no workspace needed, plain kernel
    assert lib.fpscan_scan_fwd_workspace_bytes(64, 1024, 4096, 0) == 0


# ----------------------------------------------------------------- initial state
def _scan_init_f64(g, x, h0, reverse=False):
    g, x = np.asarray(g, np.float64), np.asarray(x, np.float64)
    if reverse:
        g, x = g[..., ::-1], x[..., ::-1]
    y = np.empty_like(x)
    acc = np.asarray(h0, np.float64).copy()
    for t in range(x.shape[-1]):
        acc = g[..., t] * acc + x[..., t]
        y[..., t] = acc
    return np.ascontiguousarray(y[..., ::-1]) if reverse else y


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("seqlen", [32, 256, 4096, 16384])
def test_initial_state_forward_and_reverse(dtype, seqlen):
    gates, tokens = _make_inputs(2, 5, seqlen, dtype, seed=seqlen + 31)
    h0 = torch.randn(2, 5, device=DEVICE)
    for rev in (False, True):
        y = fpscan.scan_forward(gates, tokens, reverse=rev, initial_state=h0)
        ref = _scan_init_f64(_np64(gates), _np64(tokens), _np64(h0), rev)
        _check(y, ref, dtype, f"init rev={rev}")
    # zero initial state == the reference's zero-state scan
    y0 = fpscan.scan_forward(gates, tokens, initial_state=torch.zeros(2, 5, device=DEVICE))
    _check(y0, oracle.scan_f64(_np64(gates), _np64(tokens)), dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("seqlen", [64, 8192])
def test_initial_state_gradients(dtype, seqlen):
    """Gradients w.r.t. gates, tokens and h0 against float64 autograd through
    the serial loop; the final state y[..., -1] also receives a gradient."""
    gates, tokens = _make_inputs(2, 3, seqlen, dtype, seed=seqlen + 41)
    h0 = torch.randn(2, 3, device=DEVICE)
    w = torch.randn(2, 3, seqlen, device=DEVICE)
    wf = torch.randn(2, 3, device=DEVICE)
    g = gates.clone().requires_grad_()
    x = tokens.clone().requires_grad_()
    h = h0.clone().requires_grad_()
    y = fpscan.pscan(g, x, initial_state=h)
    ((y.float() * w).sum() + (y[..., -1].float() * wf).sum()).backward()
    g64 = gates.double().cpu().requires_grad_()
    x64 = tokens.double().cpu().requires_grad_()
    h64 = h0.double().cpu().requires_grad_()
    acc, ys = h64, []
    for t in range(seqlen):
        acc = g64[..., t] * acc + x64[..., t]
        ys.append(acc)
    y64 = torch.stack(ys, -1)
    ((y64 * w.double().cpu()).sum() + (y64[..., -1] * wf.double().cpu()).sum()).backward()
    # With O(1) states and O(10) gradients, bf16 storage of y gives isolated
    # pointwise outliers in dgates (the reference stores y the same way), so
    # half types are held to the normwise bound only.
    check = _check if dtype == torch.float32 else (
        lambda got, ref, dt, what: _assert_normwise(got, ref, dt, what))
    check(y, y64.detach().numpy(), dtype, "y")
    check(x.grad, x64.grad.numpy(), dtype, "dtokens")
    check(g.grad, g64.grad.numpy(), dtype, "dgates")
    check(h.grad, h64.grad.numpy(), dtype, "dh0")


# ----------------------------------------------------------------- fused gate producers
_ACTS = {
    "sigmoid": (lambda z: 1 / (1 + np.exp(-z)), lambda g: g * (1 - g)),
    "exp_neg_softplus": (lambda z: np.exp(-np.logaddexp(0, z)), lambda g: -g * (1 - g)),
    "exp": (np.exp, lambda g: g),
}


@pytest.mark.parametrize("activation", sorted(_ACTS))
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("seqlen", [32, 1024, 16384])
def test_gated_scan_fwd_bwd(activation, dtype, seqlen):
    gen = torch.Generator(device=DEVICE).manual_seed(seqlen + 53)
    shape = (2, 5, seqlen)
    if activation == "exp":
        z = (-0.02 * torch.rand(shape, generator=gen, device=DEVICE)).to(dtype)
    elif activation == "sigmoid":
        z = (torch.randn(shape, generator=gen, device=DEVICE) + 4).to(dtype)
    else:
        z = (torch.randn(shape, generator=gen, device=DEVICE) - 4).to(dtype)
    x = (torch.randn(shape, generator=gen, device=DEVICE) * 0.1).to(dtype)
    go = torch.randn(shape, generator=gen, device=DEVICE).to(dtype)
    act, dact = _ACTS[activation]
    g64 = act(_np64(z))
    for rev in (False, True):
        y = fpscan.scan_forward_gated(z, x, activation, reverse=rev)
        _check(y, oracle.scan_f64(g64, _np64(x), rev), dtype, f"{activation} rev={rev}")
    zz, xx = z.clone().requires_grad_(), x.clone().requires_grad_()
    y = fpscan.pscan_gated(zz, xx, activation)
    dz, dt = torch.autograd.grad(y, (zz, xx), go)
    y64 = oracle.scan_f64(g64, _np64(x))
    dg64, dt64 = oracle.scan_bwd_f64(g64, y64, _np64(go))
    _check(dt, dt64, dtype, "dtokens")
    _assert_normwise(dz, dg64 * dact(g64), dtype, "dz")
    if dtype == torch.float32:
        _check(dz, dg64 * dact(g64), dtype, "dz")


def test_gated_scan_matches_unfused_composition():
    """Config-4 distributions at a small size: fused exp(-softplus) against
    torch's activation followed by the plain scan and backward."""
    gen = torch.Generator(device=DEVICE).manual_seed(7)
    shape = (4, 96, 16384)
    z = (torch.randn(shape, generator=gen, device=DEVICE) - 1).to(torch.bfloat16)
    x = torch.randn(shape, generator=gen, device=DEVICE).to(torch.bfloat16)
    go = torch.randn(shape, generator=gen, device=DEVICE).to(torch.bfloat16)
    zz = z.clone().requires_grad_()
    xx = x.clone().requires_grad_()
    y = fpscan.pscan_gated(zz, xx, "exp_neg_softplus")
    dz, dt = torch.autograd.grad(y, (zz, xx), go)
    z2 = z.float().clone().requires_grad_()
    x2 = x.clone().requires_grad_()
    g = torch.exp(-torch.nn.functional.softplus(z2)).to(torch.bfloat16)
    y2 = fpscan.pscan(g, x2)
    dz2, dt2 = torch.autograd.grad(y2, (z2, x2), go)
    for a, b in ((y, y2), (dt, dt2), (dz, dz2)):
        assert oracle.normwise_error(_np64(a), _np64(b)) <= 2e-2


def test_binding_and_ctypes_paths_agree(monkeypatch):
    """ops.py reaches the C ABI through the compiled binding (_ext.so) when it
    is built and through ctypes otherwise; both launch the same kernels."""
    from fpscan_b200 import ops
    assert ops._EXT is not None, "fpscan_b200/_ext.so not built (python -m fpscan_b200.build)"
    g, x = _make_inputs(3, 40, 4096, torch.bfloat16, seed=5)
    go = torch.randn_like(x)
    y1 = fpscan.scan_forward(g, x)
    r1 = fpscan.scan_forward(g, x, reverse=True)
    d1 = ops.scan_backward(g, y1, go)
    g1, x1 = g[:, :1].contiguous(), x[:, :1].contiguous()  # 3 rows: the split-row path
    s1 = fpscan.scan_forward(g1, x1)
    monkeypatch.setattr(ops, "_EXT", None)
    y2 = fpscan.scan_forward(g, x)
    r2 = fpscan.scan_forward(g, x, reverse=True)
    d2 = ops.scan_backward(g, y2, go)
    s2 = fpscan.scan_forward(g1, x1)
    for a, b in ((y1, y2), (r1, r2), (d1[0], d2[0]), (d1[1], d2[1]), (s1, s2)):
        assert torch.equal(a, b)
    with pytest.raises(RuntimeError):
        fpscan.scan_forward(g[..., :100].contiguous(), x[..., :100].contiguous())


# ----------------------------------------------------------------- guard bands, workspace path
@pytest.mark.parametrize("dtype,batch,dim,seqlen", [
    (torch.float32, 2, 256, 65536), (torch.float32, 1, 1, 65536), (torch.float32, 3, 1, 32768),
    (torch.float16, 1, 8, 65536), (torch.bfloat16, 1, 37, 65536), (torch.float32, 2, 3, 8192)])
def test_ws_path_guarded(dtype, batch, dim, seqlen):
    """fpscan_scan_fwd_ws (split rows with a decoupled look-back where the
    shape takes it) writes its output into a guard-banded buffer: against
    float64 in both directions, three calls in a row on one workspace, and no
    element outside the output touched."""
    from guard import guarded

    lib = _lib.load()
    code = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[dtype]
    gates, tokens = _make_inputs(batch, dim, seqlen, dtype, seed=seqlen + dim + batch)
    need = lib.fpscan_scan_fwd_workspace_bytes(batch, dim, seqlen, code)
    ws = torch.zeros(max(need, 16), dtype=torch.uint8, device=DEVICE)
    stream = torch.cuda.current_stream().cuda_stream
    for rev in (False, True):
        ref = oracle.scan_f64(_np64(gates), _np64(tokens), reverse=rev)
        for _ in range(3):
            g = guarded(tokens.shape, dtype)
            _lib.check(lib.fpscan_scan_fwd_ws(gates.data_ptr(), tokens.data_ptr(),
                                              g.out.data_ptr(), batch, dim, seqlen, code,
                                              int(rev), ws.data_ptr(), ws.numel(), stream),
                       "fwd_ws")
            g.check(f"fwd_ws rev={rev}")
            _check(g.out, ref, dtype, f"fwd_ws rev={rev}")
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0


# ----------------------------------------------------------------- split-row fused backward
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("batch,dim,seqlen", [(2, 4, 65536), (1, 1, 65536), (1, 64, 65536),
                                              (2, 3, 32768), (1, 5, 32768)])
def test_split_row_backward(dtype, batch, dim, seqlen):
    """fpscan_scan_bwd_ws (rows cut into segments processed from each row's
    end, decoupled look-back on the dtokens state) against fpscan_scan_bwd
    and float64, outputs guard-banded, three calls in a row on one
    workspace."""
    from guard import guarded

    lib = _lib.load()
    code = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[dtype]
    gates, tokens = _make_inputs(batch, dim, seqlen, dtype, seed=seqlen + dim + 7)
    gen = torch.Generator(device=DEVICE).manual_seed(dim)
    go = torch.randn(batch, dim, seqlen, generator=gen, device=DEVICE).to(dtype)
    y = fpscan.scan_forward(gates, tokens)
    need = lib.fpscan_scan_bwd_workspace_bytes(batch, dim, seqlen, code)
    assert need > 0  # these shapes take the split-row path
    ws = torch.zeros(need, dtype=torch.uint8, device=DEVICE)
    s = torch.cuda.current_stream().cuda_stream
    dg_p, dt_p = torch.empty_like(go), torch.empty_like(go)
    _lib.check(lib.fpscan_scan_bwd(gates.data_ptr(), y.data_ptr(), go.data_ptr(), dg_p.data_ptr(),
                                   dt_p.data_ptr(), batch, dim, seqlen, code, s), "bwd")
    y64 = oracle.scan_f64(_np64(gates), _np64(tokens))
    dg64, dt64 = oracle.scan_bwd_f64(_np64(gates), _np64(y), _np64(go))
    for _ in range(3):
        dg, dt = guarded(go.shape, dtype), guarded(go.shape, dtype)
        _lib.check(lib.fpscan_scan_bwd_ws(gates.data_ptr(), y.data_ptr(), go.data_ptr(),
                                          dg.out.data_ptr(), dt.out.data_ptr(), batch, dim,
                                          seqlen, code, ws.data_ptr(), ws.numel(), s), "bwd_ws")
        dg.check("split bwd dgates")
        dt.check("split bwd dtokens")
        _assert_normwise(dt.out, dt64, dtype, "split dtokens")
        _assert_normwise(dg.out, dg64, dtype, "split dgates")
        assert oracle.normwise_error(_np64(dt.out), _np64(dt_p)) <= NORM_TOL[dtype]
        assert oracle.normwise_error(_np64(dg.out), _np64(dg_p)) <= NORM_TOL[dtype]
    # the public API takes the same path
    gr, xr = gates.clone().requires_grad_(), tokens.clone().requires_grad_()
    dgr, dxr = torch.autograd.grad(fpscan.pscan(gr, xr), (gr, xr), go)
    _assert_normwise(dxr, dt64, dtype, "pscan dtokens")
    _assert_normwise(dgr, dg64, dtype, "pscan dgates")
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0
    del y64


def test_split_row_backward_workspace_checks():
    lib = _lib.load()
    assert lib.fpscan_scan_bwd_workspace_bytes(64, 1024, 4096, 0) == 0  # many rows: none
    gates, tokens = _make_inputs(1, 2, 65536, torch.float32)
    need = lib.fpscan_scan_bwd_workspace_bytes(1, 2, 65536, 0)
    assert need > 0
    ws = torch.zeros(need, dtype=torch.uint8, device=DEVICE)
    dg, dt = torch.empty_like(tokens), torch.empty_like(tokens)
    s = torch.cuda.current_stream().cuda_stream
    assert lib.fpscan_scan_bwd_ws(gates.data_ptr(), tokens.data_ptr(), tokens.data_ptr(),
                                  dg.data_ptr(), dt.data_ptr(), 1, 2, 65536, 0, ws.data_ptr(),
                                  need - 16, s) == 1
    assert b"workspace" in lib.fpscan_last_error()
    assert lib.fpscan_scan_bwd_ws(gates.data_ptr(), tokens.data_ptr(), tokens.data_ptr(),
                                  dg.data_ptr(), dg.data_ptr(), 1, 2, 65536, 0, ws.data_ptr(),
                                  need, s) == 1
    assert b"overlaps" in lib.fpscan_last_error()
