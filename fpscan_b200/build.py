"""Build libfpscan_b200.so in-tree with nvcc for sm_100a.

The library is a plain C-ABI shared object (no torch / pybind dependency):
every ``csrc/*.cu`` is compiled with relocatable device code (the device
status word is shared between translation units) and linked with the CUDA
runtime statically.  Rebuilds only when a source or header is newer than the
library.  Usage: ``python -m fpscan_b200.build [--force]``.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys
import tempfile

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_NAME = "libfpscan_b200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-rdc=true",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps():
    return (_sources() + glob.glob(os.path.join(CSRC, "*.cuh"))
            + glob.glob(os.path.join(CSRC, "*.h"))
            + glob.glob(os.path.join(REPO_DIR, "include", "*.h")) + [__file__])


def needs_build() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(p) > t for p in _deps())


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False,
          defines=(), out_path: str = LIB_PATH) -> str:
    """Compile the library if needed; returns its path.  `defines` (-D flags)
    and `out_path` build an alternative variant elsewhere (always rebuilt)."""
    if out_path == LIB_PATH and not defines and not force and not needs_build():
        return LIB_PATH
    nvcc = _nvcc()
    extra = (["-Xptxas", "-v"] if ptxas_verbose else []) + [f"-D{d}" for d in defines]
    with tempfile.TemporaryDirectory(prefix="fpscan_build_") as tmp:
        objs = []
        procs = []
        for src in _sources():
            obj = os.path.join(tmp, os.path.basename(src) + ".o")
            cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, *extra, "-I", CSRC,
                   "-I", os.path.join(REPO_DIR, "include"), "-c", src, "-o", obj]
            if verbose:
                print(" ".join(cmd))
            procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE,
                                                stderr=subprocess.STDOUT, text=True)))
            objs.append(obj)
        failed = []
        for src, p in procs:
            out, _ = p.communicate()
            if out and (verbose or ptxas_verbose or p.returncode):
                print(out, file=sys.stderr)
            if p.returncode:
                failed.append(src)
        if failed:
            raise RuntimeError(f"nvcc failed for {failed}")
        tmp_lib = os.path.join(tmp, LIB_NAME)
        cmd = [nvcc, *ARCH_FLAGS, "-rdc=true", "-shared", "-Xcompiler", "-fPIC",
               *objs, "-o", tmp_lib]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        os.makedirs(os.path.dirname(out_path), exist_ok=True)
        os.replace(tmp_lib, out_path)
    return out_path


# ---------------------------------------------------------------- bounds-checking build
DEBUG_LIB_PATH = os.path.join(PKG_DIR, "libfpscan_b200_debug.so")


def build_debug(force: bool = False, verbose: bool = False) -> str:
    """Compile libfpscan_b200_debug.so: the same library with
    -DFPSCAN_DEBUG_BOUNDS, whose kernels check every global access they
    compute themselves against its tensor's extent and record (and skip) one
    outside it in the device status word.  A test tool: the stand-in for the
    memory checkers that are closed on the GPU pool."""
    if (not force and os.path.exists(DEBUG_LIB_PATH)
            and all(os.path.getmtime(p) <= os.path.getmtime(DEBUG_LIB_PATH) for p in _deps())):
        return DEBUG_LIB_PATH
    return build(force=True, verbose=verbose, defines=("FPSCAN_DEBUG_BOUNDS",),
                 out_path=DEBUG_LIB_PATH)


# ---------------------------------------------------------------- torch binding
BINDING_SRC = os.path.join(PKG_DIR, "binding", "ext.cpp")
BINDING_PATH = os.path.join(PKG_DIR, "_ext.so")


def build_binding(force: bool = False, verbose: bool = False) -> str:
    """Compile fpscan_b200/_ext.so: the thin torch/pybind binding over the C
    ABI (fast path of ops.py for the reference's entry points).  Host code
    only (g++ against torch's headers); links libfpscan_b200.so by rpath."""
    # the library is linked by name (rpath): a rebuilt library needs no relink
    deps = [BINDING_SRC, os.path.join(REPO_DIR, "include", "fpscan_b200.h"), __file__]
    if (not force and os.path.exists(BINDING_PATH)
            and all(os.path.getmtime(d) <= os.path.getmtime(BINDING_PATH) for d in deps)):
        return BINDING_PATH
    import sysconfig

    import torch

    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    incs = [os.path.join(os.path.dirname(torch.__file__), "include"),
            os.path.join(os.path.dirname(torch.__file__), "include", "torch", "csrc", "api",
                         "include"),
            os.path.join(cuda_home, "include"), sysconfig.get_paths()["include"]]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    with tempfile.TemporaryDirectory(prefix="fpscan_bind_") as tmp:
        out = os.path.join(tmp, "_ext.so")
        cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-w",
               f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_ext",
               "-DTORCH_API_INCLUDE_EXTENSION_H", *[f"-I{i}" for i in incs], BINDING_SRC,
               "-o", out, f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
               "-ltorch_cuda", "-ltorch_python", f"-L{PKG_DIR}", "-lfpscan_b200",
               "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        os.replace(out, BINDING_PATH)
    return BINDING_PATH


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose="-v" in sys.argv,
                 ptxas_verbose="--ptxas" in sys.argv)
    print(path)
    print(build_binding(force="--force" in sys.argv, verbose="-v" in sys.argv))
