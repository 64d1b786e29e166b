"""fpscan_scan_fwd_noalloc: the scan for callers that cannot allocate device
memory (a host that owns every GPU allocation, a service that forbids
cudaMalloc/cudaFree while running, C code without a caching allocator).

Called through the C ABI, twice in a row per case (the library's fixed
scratch array is reused and keeps the previous call's contents), and
compared with the existing workspace entry point fpscan_scan_fwd_ws within
the normwise tolerance the other GPU tests use.  Collected last (file name)
so that a run stopping at the first failure has already run everything else.
"""
import numpy as np
import pytest
import torch

import oracle
from fpscan_b200 import _lib

pytestmark = pytest.mark.gpu

CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
NORM_TOL = {torch.float32: 1e-5, torch.float16: 1e-2, torch.bfloat16: 1e-2}


def _inputs(b, d, L, dtype, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    g = (0.99 + 0.01 * torch.rand(b, d, L, generator=gen, device="cuda")).to(dtype)
    x = (torch.randn(b, d, L, generator=gen, device="cuda") / L).to(dtype)
    return g, x


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
    assert (need > 0) == (L == 65536)  # the 65536 cases take the split path (scratch)
    ws = torch.zeros(max(need, 16), dtype=torch.uint8, device="cuda")
    for rev in (0, 1):
        ref = torch.empty_like(tokens)
        _lib.check(lib.fpscan_scan_fwd_ws(gates.data_ptr(), tokens.data_ptr(), ref.data_ptr(), b, d, L,
                                          code, rev, ws.data_ptr(), ws.numel(), stream),
                   "fpscan_scan_fwd_ws")
        ref64 = ref.double().cpu().numpy()
        for _ in range(2):
            out = torch.full_like(tokens, float("nan"))
            _lib.check(lib.fpscan_scan_fwd_noalloc(gates.data_ptr(), tokens.data_ptr(), out.data_ptr(),
                                                   b, d, L, code, rev, stream),
                       "fpscan_scan_fwd_noalloc")
            got = out.double().cpu().numpy()
            assert np.isfinite(got).all()
            assert oracle.normwise_error(got, ref64) <= NORM_TOL[dtype]
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0


def test_no_alloc_rejects_shapes_beyond_its_scratch():
    lib = _lib.load()
    gates, tokens = _inputs(1, 100, 65536, torch.float32, seed=1)  # 800 segments > 512
    assert lib.fpscan_scan_fwd_workspace_bytes(1, 100, 65536, 0) > 256 + 16 * 512
    out = torch.empty_like(tokens)
    rc = lib.fpscan_scan_fwd_noalloc(gates.data_ptr(), tokens.data_ptr(), out.data_ptr(), 1, 100,
                                     65536, 0, 0, torch.cuda.current_stream().cuda_stream)
    assert rc == 1
    assert b"scratch" in lib.fpscan_last_error()
