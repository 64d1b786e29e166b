"""Host-side logic that needs no GPU: the C ABI loads and exports every
declared symbol, argument validation (C and Python) mirrors the reference's
errors, channel partitioning."""
import ctypes
import glob
import os
import re

import pytest
import torch

import fpscan_b200
from fpscan_b200 import _lib, ops
from fpscan_b200.distributed import channel_slice

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    names = []
    for h in glob.glob(os.path.join(REPO, "include", "*.h")):
        names += re.findall(r"FPSCAN_API\s+[\w\s\*]+?\b(fpscan_\w+)\s*\(", open(h).read())
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    names = _declared_symbols()
    assert "fpscan_scan_fwd" in names and "fpscan_scan_bwd" in names
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"


def test_abi_version():
    assert _lib.load().fpscan_abi_version() == _lib.EXPECTED_ABI_VERSION


def _fwd(gates=16, tokens=16, out=16, b=1, d=1, l=32, dtype=0, rev=0):
    lib = _lib.load()
    return lib.fpscan_scan_fwd(gates, tokens, out, b, d, l, dtype, rev, None)


@pytest.mark.parametrize("l", [0, 16, 30, 48, 131072])
def test_c_abi_rejects_bad_seqlen(l):
    # csrc/full_scan/full_scan.cu:232: seqlen must be a power of 2 in [32, 65536]
    assert _fwd(l=l) == 1
    assert b"seqlen" in _lib.load().fpscan_last_error()


def test_c_abi_rejects_bad_dtype_null_and_misaligned():
    lib = _lib.load()
    assert _fwd(dtype=7) == 1 and b"dtype" in lib.fpscan_last_error()
    assert _fwd(gates=0) == 1 and b"NULL" in lib.fpscan_last_error()
    assert _fwd(tokens=24) == 1 and b"aligned" in lib.fpscan_last_error()
    assert _fwd(b=-1) == 1


def test_c_abi_rejects_partial_overlap():
    lib = _lib.load()
    assert _fwd(gates=4096, tokens=8192, out=8192 + 64, l=32) == 1
    assert b"overlap" in lib.fpscan_last_error()
    rc = lib.fpscan_scan_bwd(4096, 1 << 20, 2 << 20, 4096 + 16, 3 << 20, 1, 1, 32, 0, None)
    assert rc == 1 and b"overlap" in lib.fpscan_last_error()


def test_c_abi_empty_is_noop():
    # batch*dim == 0 launches nothing and succeeds (even without a GPU).
    assert _fwd(b=0) == 0
    assert _lib.load().fpscan_scan_bwd(0, 0, 0, 0, 0, 0, 4, 64, 0, None) == 0


def test_carry_combine_arg_checks():
    lib = _lib.load()
    assert lib.fpscan_carry_combine(16, 2, 2, 8, 0, 32, None) == 1
    assert lib.fpscan_carry_combine(16, 0, 0, 8, 0, 32, None) == 1


def test_python_rejects_cpu_tensors_like_reference():
    g = torch.rand(1, 1, 32)
    with pytest.raises(RuntimeError, match="CUDA"):
        fpscan_b200.scan_forward(g, g)


@pytest.mark.parametrize("case", ["pow2", "range", "shape", "dtype", "ndim", "out"])
def test_layout_validation(case):
    g = torch.rand(2, 3, 64)
    x = torch.rand(2, 3, 64)
    out = None
    if case == "pow2":
        g, x = g[..., :30].contiguous(), x[..., :30].contiguous()
    elif case == "range":
        g, x = torch.rand(1, 1, 16), torch.rand(1, 1, 16)
    elif case == "shape":
        x = torch.rand(2, 4, 64)
    elif case == "dtype":
        x = x.half()
    elif case == "ndim":
        g, x = g[0], x[0]
    elif case == "out":
        out = torch.empty(2, 3, 32)
    with pytest.raises(RuntimeError):
        ops.validate_layout(g, x, out)


def test_layout_validation_accepts_reference_shapes():
    for l in [32, 64, 4096, 65536]:
        t = torch.empty(1, 1, l)
        ops.validate_layout(t, t, torch.empty_like(t))


@pytest.mark.parametrize("rows,world", [(512, 1), (512, 8), (81920, 8), (7, 3), (3, 8)])
def test_channel_slice_partitions_rows(rows, world):
    spans = [channel_slice(rows, r, world) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == rows
    for (a, b), (c, d) in zip(spans, spans[1:]):
        assert b == c
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1


def test_reference_style_extension_shim():
    from fpscan_b200 import _C

    assert hasattr(_C, "fullscan_forward")


def test_anylen_validation_and_c_abi_checks():
    # any seqlen >= 1 is accepted by the *_anylen layer; 0 is not
    for l in [1, 3, 1000, 65537, 300001]:
        t = torch.empty(1, 1, l)
        ops.validate_layout(t, t, torch.empty_like(t), any_seqlen=True)
    t = torch.empty(1, 1, 0)
    with pytest.raises(RuntimeError):
        ops.validate_layout(t, t, any_seqlen=True)
    with pytest.raises(RuntimeError):  # strict path unchanged
        ops.validate_layout(torch.empty(1, 1, 1000), torch.empty(1, 1, 1000))
    lib = _lib.load()
    assert lib.fpscan_scan_fwd_anylen(16, 16, 16, 1, 1, 0, 0, 0, None) == 1
    assert b"seqlen" in lib.fpscan_last_error()
    assert lib.fpscan_scan_fwd_anylen(16, 24, 16, 1, 1, 7, 0, 0, None) == 1
    assert b"aligned" in lib.fpscan_last_error()
    assert lib.fpscan_scan_fwd_anylen(4096, 8192, 8192 + 64, 1, 1, 33, 0, 0, None) == 1
    assert b"overlap" in lib.fpscan_last_error()
    rc = lib.fpscan_scan_bwd_anylen(4096, 1 << 20, 2 << 20, 4096 + 16, 3 << 20, 1, 1, 33, 0, None)
    assert rc == 1 and b"overlap" in lib.fpscan_last_error()
    assert lib.fpscan_scan_fwd_anylen(0, 0, 0, 0, 4, 1000, 0, 0, None) == 0
    assert lib.fpscan_scan_bwd_anylen(0, 0, 0, 0, 0, 3, 0, 7, 2, None) == 0


def test_channels_last_validation_and_c_abi_checks():
    t = torch.empty(2, 10, 64)
    lib = _lib.load()
    # dim*itemsize must be a multiple of 16
    assert lib.fpscan_scan_fwd_cl(16, 16, 16, 1, 10, 6, 0, 0, 16, 1 << 20, None) == 1
    assert b"multiple" in lib.fpscan_last_error()
    assert lib.fpscan_scan_fwd_cl(16, 16, 16, 1, 0, 8, 0, 0, 16, 1 << 20, None) == 1
    assert b"seqlen" in lib.fpscan_last_error()
    need = lib.fpscan_cl_workspace_bytes(2, 1000, 256, 2, 0)
    # few columns (2 batches x 4 columns of 8 vectors): the segmented path sizes
    # its per-segment maps for ceil(2 * SMs / columns) segments (148 SMs assumed
    # without a GPU): columns x segments x 64 bf16 channels x (8 + 4) bytes
    n = 8 * 37 * 64
    assert need == (n * 8 + 255) // 256 * 256 + n * 4
    assert lib.fpscan_cl_workspace_bytes(2, 1000, 256, 2, 1) == need
    assert lib.fpscan_cl_workspace_bytes(16, 1000, 5120, 2, 0) == 256  # 1280 columns: no segments
    assert lib.fpscan_scan_fwd_cl(1 << 20, 2 << 20, 3 << 20, 2, 1000, 256, 2, 0, 4 << 20, need - 16,
                                  None) == 1
    assert b"workspace too small" in lib.fpscan_last_error()
    assert lib.fpscan_scan_fwd_cl(1 << 20, 2 << 20, 3 << 20, 2, 1000, 256, 2, 0, (3 << 20) + 64,
                                  need, None) == 1
    assert b"overlap" in lib.fpscan_last_error()
    rc = lib.fpscan_scan_bwd_cl(1 << 20, 2 << 20, 3 << 20, (1 << 20) + 16, 5 << 20, 2, 10, 256, 2,
                                6 << 20, 1 << 20, None)
    assert rc == 1 and b"overlap" in lib.fpscan_last_error()
    assert lib.fpscan_scan_fwd_cl(0, 0, 0, 0, 10, 256, 2, 0, 0, 0, None) == 0
    with pytest.raises(RuntimeError):
        ops.validate_channels_last(t, t)  # CPU tensors are rejected like the reference's


def test_link_abi_checks_without_gpu():
    """Chained sequence-sharding entry points: mailbox size and argument
    checks (all before any CUDA call)."""
    lib = _lib.load()
    rows, depth = 1000, 4
    ring = -(-depth * rows * 8 // 256) * 256
    one = -(-rows * 4 // 256) * 256
    assert lib.fpscan_link_bytes(rows, depth) == 2 * ring + 3 * one
    assert lib.fpscan_link_bytes(0, depth) == 0 and lib.fpscan_link_bytes(rows, 0) == 0
    mb = 1 << 20
    # neither neighbour
    assert lib.fpscan_shard_fwd_link(16, 16, 16, None, rows, 8192, 0, mb, None, None, 1, depth,
                                     None) == 1
    assert b"upstream or a downstream" in lib.fpscan_last_error()
    # epoch 0 is reserved
    assert lib.fpscan_shard_fwd_link(16, 16, 16, None, rows, 8192, 0, mb, mb, None, 0, depth,
                                     None) == 1
    assert b"epoch" in lib.fpscan_last_error()
    # local seqlen must exceed one chunk and be a power of two
    for L in (1024, 3000):
        assert lib.fpscan_shard_fwd_link(16, 16, 16, None, rows, L, 0, mb, mb, None, 1, depth,
                                         None) == 1
        assert b"seqlen" in lib.fpscan_last_error()
    # backward: y_prev required when there is an upstream rank
    assert lib.fpscan_shard_bwd_link(16, 16, 16, 16, 16, None, rows, 8192, 0, mb, mb, None, 1,
                                     depth, None) == 1
    assert b"y_prev" in lib.fpscan_last_error()


def test_bench_reference_arm_json_contract():
    """`bench.py --impl reference` (the reference's CPU path; runs without a
    GPU) prints one JSON line with the keys the benchmark contract names."""
    import json
    import subprocess
    import sys
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, os.path.join(repo, "bench.py"), "--impl", "reference",
                        "--steps", "1", "--warmup", "3", "--ref-budget-s", "2"],
                       capture_output=True, text=True,
                       timeout=600, cwd=repo)
    assert r.returncode == 0, r.stderr[-3000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["cores"] >= 1


def test_row_unit_planner(tmp_path):
    """plan_units (csrc/internal.h): static tiles without a counter or with
    fewer than two units per CTA slot, claimed units otherwise; every plan
    covers all rows and fits one wave (tests/plan_units_check.cpp)."""
    import shutil
    import subprocess
    here = os.path.dirname(os.path.abspath(__file__))
    csrc = os.path.join(os.path.dirname(here), "fpscan_b200", "csrc")
    cuda_inc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")
    gxx = shutil.which("g++")
    if gxx is None or not os.path.exists(os.path.join(cuda_inc, "cuda_runtime.h")):
        pytest.skip("needs g++ and the CUDA headers")
    exe = tmp_path / "plan_units_check"
    subprocess.run([gxx, "-std=c++17", "-O1", "-I", csrc, "-I", cuda_inc,
                    os.path.join(here, "plan_units_check.cpp"), "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-3000:]


def test_row_unit_claim_protocol(tmp_path):
    """The counter protocol of csrc/claim.h with CPU threads as CTAs
    (tests/claim_protocol_check.cpp): every unit processed exactly once and
    the counter word back at 0 after each launch, with aborting CTAs too."""
    import shutil
    import subprocess
    here = os.path.dirname(os.path.abspath(__file__))
    csrc = os.path.join(os.path.dirname(here), "fpscan_b200", "csrc")
    cuda_inc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")
    gxx = shutil.which("g++")
    if gxx is None or not os.path.exists(os.path.join(cuda_inc, "cuda_runtime.h")):
        pytest.skip("needs g++ and the CUDA headers")
    exe = tmp_path / "claim_protocol_check"
    subprocess.run([gxx, "-std=c++17", "-O1", "-pthread", "-I", csrc, "-I", cuda_inc,
                    os.path.join(here, "claim_protocol_check.cpp"), "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-3000:]


def test_nvtx_ranges_are_opt_in():
    """NVTX ranges wrap the forward, backward and sequence-shard steps only
    when FPSCAN_B200_NVTX=1; the range object is a no-op otherwise."""
    from fpscan_b200 import ops as o

    assert o.NVTX is False or os.environ.get("FPSCAN_B200_NVTX") == "1"
    with o.nvtx_range("fpscan.test"):
        pass
