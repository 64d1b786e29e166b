"""fpscan_scan_fwd_noalloc: the scan for callers that cannot allocate device
memory (a host that owns every GPU allocation, a service that forbids
cudaMalloc/cudaFree while running, C code without a caching allocator).

Called through the C ABI, twice in a row per case (the library's fixed
scratch array is reused and keeps the previous call's contents), and
compared with the existing workspace entry point fpscan_scan_fwd_ws and with
the float64 oracle, within the normwise tolerance the other GPU tests use.
One case runs on a fresh non-blocking stream whose first call is the noalloc
call; one checks that device memory in use does not change across a call.
Collected last (file name) so that a run stopping at the first failure has
already run everything else.
"""
import numpy as np
import pytest
import torch

import oracle
from fpscan_b200 import _lib

pytestmark = pytest.mark.gpu

CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
NORM_TOL = {torch.float32: 1e-5, torch.float16: 1e-2, torch.bfloat16: 1e-2}
SCRATCH_BYTES = 256 + 16 * 512  # the library's fixed array: 512 split segments


def _inputs(b, d, L, dtype, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    g = (0.99 + 0.01 * torch.rand(b, d, L, generator=gen, device="cuda")).to(dtype)
    x = (torch.randn(b, d, L, generator=gen, device="cuda") / L).to(dtype)
    return g, x


def _noalloc(lib, gates, tokens, out, shape, code, rev, stream):
    b, d, L = shape
    _lib.check(lib.fpscan_scan_fwd_noalloc(gates.data_ptr(), tokens.data_ptr(), out.data_ptr(),
                                           b, d, L, code, rev, stream),
               "fpscan_scan_fwd_noalloc")


@pytest.mark.parametrize("dtype,shape", [
    (torch.float32, (1, 64, 65536)),    # split rows: 512 segments, the stated maximum
    (torch.bfloat16, (1, 3, 65536)),    # split rows, few segments
    (torch.float32, (1, 1, 65536)),     # split rows, one row
    (torch.float16, (4, 64, 1024)),     # no scratch needed: one CTA per row
])
def test_no_alloc_matches_workspace_entry(dtype, shape):
    lib = _lib.load()
    b, d, L = shape
    code = CODES[dtype]
    gates, tokens = _inputs(b, d, L, dtype, seed=L + d)
    stream = torch.cuda.current_stream().cuda_stream
    need = lib.fpscan_scan_fwd_workspace_bytes(b, d, L, code)
    ws = torch.zeros(max(need, 16), dtype=torch.uint8, device="cuda")
    g64 = gates.double().cpu().numpy()
    x64 = tokens.double().cpu().numpy()
    for rev in (0, 1):
        ref = torch.empty_like(tokens)
        _lib.check(lib.fpscan_scan_fwd_ws(gates.data_ptr(), tokens.data_ptr(), ref.data_ptr(), b, d, L,
                                          code, rev, ws.data_ptr(), ws.numel(), stream),
                   "fpscan_scan_fwd_ws")
        ref64 = ref.double().cpu().numpy()
        y64 = oracle.scan_f64(g64, x64, reverse=bool(rev))
        for _ in range(2):
            out = torch.full_like(tokens, float("nan"))
            _noalloc(lib, gates, tokens, out, shape, code, rev, stream)
            got = out.double().cpu().numpy()
            assert np.isfinite(got).all()
            assert oracle.normwise_error(got, ref64) <= NORM_TOL[dtype]
            assert oracle.normwise_error(got, y64) <= NORM_TOL[dtype]
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0


def test_no_alloc_on_a_fresh_nonblocking_stream_allocates_nothing():
    """The first call on a new non-blocking stream, then a second one,
    against the float64 oracle; device memory in use (driver's view and
    torch's allocator) is unchanged across the second call."""
    lib = _lib.load()
    shape = (1, 8, 65536)
    gates, tokens = _inputs(*shape, torch.float32, seed=7)
    y64 = oracle.scan_f64(gates.double().cpu().numpy(), tokens.double().cpu().numpy())
    outs = [torch.full_like(tokens, float("nan")) for _ in range(2)]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    torch.cuda.synchronize()
    with torch.cuda.stream(side):
        _noalloc(lib, gates, tokens, outs[0], shape, 0, 0, side.cuda_stream)
        side.synchronize()
        free0, _ = torch.cuda.mem_get_info()
        stats0 = torch.cuda.memory_stats().get("allocation.all.allocated", 0)
        _noalloc(lib, gates, tokens, outs[1], shape, 0, 0, side.cuda_stream)
        side.synchronize()
        free1, _ = torch.cuda.mem_get_info()
        stats1 = torch.cuda.memory_stats().get("allocation.all.allocated", 0)
    assert free1 == free0
    assert stats1 == stats0
    for out in outs:
        got = out.double().cpu().numpy()
        assert np.isfinite(got).all()
        assert oracle.normwise_error(got, y64) <= 1e-5
    assert _lib.device_status(clear=True) == 0


def test_no_alloc_rejects_shapes_beyond_its_scratch():
    """The limit is on split segments, whose number depends on the GPU (SM
    count, occupancy): the first rejected shape is searched for by calling
    the entry point on growing channel counts rather than fixed."""
    lib = _lib.load()
    L, dmax = 65536, 256
    gates, tokens = _inputs(1, dmax, L, torch.float32, seed=1)
    out = torch.empty_like(tokens)
    stream = torch.cuda.current_stream().cuda_stream
    for d in range(1, dmax + 1):
        rc = lib.fpscan_scan_fwd_noalloc(gates.data_ptr(), tokens.data_ptr(), out.data_ptr(), 1,
                                         d, L, 0, 0, stream)
        if rc != 0:
            assert rc == 1
            assert b"scratch" in lib.fpscan_last_error()
            break
    else:
        pytest.skip("no shape up to 256 channels needs more split segments than the scratch holds")
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0
