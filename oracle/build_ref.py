"""ORACLE — build the reference's CUDA scan from its own sources (test only).

Compiles ``csrc/full_scan/full_scan.cu`` of the reference checkout (read in
place, never copied) together with oracle/ref_binding.cpp into
``oracle/_ref/fpscan_ref_ext.so`` for sm_100a, using the reference's nvcc
flags (setup.py:36-47).  Needs the reference checkout, so it runs in the build
container only; the built .so travels with the repository snapshot.
Usage: python oracle/build_ref.py [REFERENCE_ROOT]

The reference checkout is found from the argument, else the environment
variable FPSCAN_REFERENCE_ROOT, else BASELINE.json's ``reference_path``.
"""
from __future__ import annotations

import json
import os
import sys

ORACLE_DIR = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(ORACLE_DIR, "_ref")


def reference_root() -> str | None:
    """The reference checkout: $FPSCAN_REFERENCE_ROOT, else BASELINE.json's
    reference_path; None when neither names an existing directory."""
    root = os.environ.get("FPSCAN_REFERENCE_ROOT")
    if not root:
        try:
            with open(os.path.join(os.path.dirname(ORACLE_DIR), "BASELINE.json")) as f:
                root = json.load(f).get("reference_path")
        except (OSError, ValueError):
            root = None
    return root if root and os.path.isdir(root) else None


def build(ref_root: str | None = None, verbose: bool = False) -> str | None:
    ref_root = ref_root or reference_root()
    if ref_root is None:
        return None
    src = os.path.join(ref_root, "csrc", "full_scan", "full_scan.cu")
    if not os.path.exists(src):
        return None
    out = os.path.join(OUT_DIR, "fpscan_ref_ext.so")
    binding = os.path.join(ORACLE_DIR, "ref_binding.cpp")
    if os.path.exists(out) and os.path.getmtime(out) >= max(
            os.path.getmtime(src), os.path.getmtime(binding)):
        return out
    os.makedirs(OUT_DIR, exist_ok=True)
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    from torch.utils.cpp_extension import load

    load(
        name="fpscan_ref_ext",
        sources=[binding, src],
        extra_include_paths=[os.path.join(ref_root, "csrc")],
        extra_cflags=["-O3"],
        extra_cuda_cflags=[
            "-O3", "-lineinfo", "--use_fast_math", "-std=c++17",
            "-U__CUDA_NO_HALF_CONVERSIONS__", "-U__CUDA_NO_HALF_OPERATORS__",
            "-U__CUDA_NO_BFLOAT16_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
        ],
        build_directory=OUT_DIR,
        verbose=verbose,
        is_python_module=True,
    )
    return out


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else None, verbose=True))
