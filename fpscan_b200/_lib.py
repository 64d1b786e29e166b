"""ctypes binding of ``libfpscan_b200.so`` (the C ABI in include/fpscan_b200.h).

The shared object is built in-tree by ``python -m fpscan_b200.build``.  There
is no fallback: if the library is missing or fails to load, every op raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

LIB_PATH = _build.LIB_PATH

_c_i64 = ctypes.c_int64
_c_int = ctypes.c_int
_vp = ctypes.c_void_p

# name -> argtypes; every function returns int except fpscan_last_error
# (const char*) and fpscan_scan_fwd_workspace_bytes (int64).
SIGNATURES = {
    "fpscan_abi_version": [],
    "fpscan_scan_fwd": [_vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_int, _c_int, _vp],
    "fpscan_scan_fwd_workspace_bytes": [_c_i64, _c_i64, _c_i64, _c_int],
    "fpscan_scan_fwd_ws": [_vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_int, _c_int, _vp, _c_i64, _vp],
    "fpscan_scan_fwd_noalloc": [_vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_int, _c_int, _vp],
    "fpscan_scan_fwd_init": [_vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_int, _c_int, _vp],
    "fpscan_scan_fwd_act": [_vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_int, _vp],
    "fpscan_scan_bwd_act": [_vp, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_int, _c_int, _vp],
    "fpscan_scan_fwd_anylen": [_vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_int, _c_int, _vp],
    "fpscan_scan_bwd_anylen": [_vp, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_int, _vp],
    "fpscan_cl_workspace_bytes": [_c_i64, _c_i64, _c_i64, _c_int, _c_int],
    "fpscan_scan_fwd_cl": [_vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_int, _c_int, _vp, _c_i64, _vp],
    "fpscan_scan_bwd_cl": [_vp, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_int, _vp, _c_i64,
                           _vp],
    "fpscan_scan_bwd": [_vp, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_int, _vp],
    "fpscan_scan_bwd_workspace_bytes": [_c_i64, _c_i64, _c_i64, _c_int],
    "fpscan_scan_bwd_ws": [_vp, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_int, _vp, _c_i64,
                           _vp],
    "fpscan_shard_fwd_reduce": [_vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_int, _vp],
    "fpscan_shard_fwd_scan": [_vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_int, _vp],
    "fpscan_shard_bwd_reduce": [_vp, _vp, _vp, _c_i64, _c_i64, _c_int, _vp],
    "fpscan_shard_bwd_scan": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_int, _vp],
    "fpscan_carry_combine": [_vp, _c_int, _c_int, _c_i64, _c_int, _vp, _vp],
    "fpscan_link_bytes": [_c_i64, _c_int],
    "fpscan_link_create": [_c_i64, _c_int, ctypes.POINTER(_vp)],
    "fpscan_link_destroy": [_vp],
    "fpscan_link_ipc_handle": [_vp, ctypes.c_char_p],
    "fpscan_link_open": [ctypes.c_char_p, ctypes.POINTER(_vp)],
    "fpscan_link_close": [_vp],
    "fpscan_shard_fwd_link": [_vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_int, _vp, _vp, _vp,
                              ctypes.c_uint32, _c_int, _vp],
    "fpscan_shard_bwd_link": [_vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_int, _vp, _vp,
                              _vp, ctypes.c_uint32, _c_int, _vp],
    "fpscan_last_error": [],
    "fpscan_device_status": [ctypes.POINTER(ctypes.c_uint), _c_int],
    "fpscan_status_snapshot": [_vp, _vp],
    "fpscan_set_wait_limit_ns": [ctypes.c_uint64],
    "fpscan_debug_bounds": [_vp],
}

EXPECTED_ABI_VERSION = 1

_lock = threading.Lock()
_lib = None


class FpscanError(RuntimeError):
    """A C-ABI call returned a non-zero status."""


_RESTYPES = {"fpscan_last_error": ctypes.c_char_p,
             "fpscan_scan_fwd_workspace_bytes": ctypes.c_int64,
             "fpscan_scan_bwd_workspace_bytes": ctypes.c_int64,
             "fpscan_cl_workspace_bytes": ctypes.c_int64,
             "fpscan_link_bytes": ctypes.c_int64}


def open_library(path: str) -> ctypes.CDLL:
    """Load a build of the C ABI at `path` (e.g. the bounds-checking
    libfpscan_b200_debug.so) with the signatures set up; not cached."""
    lib = ctypes.CDLL(path)
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = _RESTYPES.get(name, ctypes.c_int)
    return lib


def load() -> ctypes.CDLL:
    """Load the library once (thread-safe) and set up its signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"fpscan_b200 CUDA library not found at {LIB_PATH}; build it with "
                "`python -m fpscan_b200.build` (needs nvcc for sm_100a)")
        lib = open_library(LIB_PATH)
        ver = lib.fpscan_abi_version()
        if ver != EXPECTED_ABI_VERSION:
            raise ImportError(f"libfpscan_b200 ABI version {ver}, expected {EXPECTED_ABI_VERSION}")
        _lib = lib
        return lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().fpscan_last_error().decode(errors="replace")
        raise FpscanError(f"{what}: {msg}")


def call(name: str, *args) -> None:
    lib = load()
    check(getattr(lib, name)(*args), name)


def device_status(clear: bool = True) -> int:
    """Synchronously read the current device's status word (0 = healthy)."""
    v = ctypes.c_uint(0)
    check(load().fpscan_device_status(ctypes.byref(v), 1 if clear else 0), "fpscan_device_status")
    return int(v.value)


STATUS_BITS = {
    1: "a kernel gave up waiting for its own copies to land",
    2: "a split-row scan gave up waiting for a preceding segment (look-back)",
    4: "a channel-last CTA found its staging buffer misaligned and skipped its work",
    8: "a chained sequence-sharded scan gave up waiting for a neighbouring rank",
    16: "a kernel skipped a global access outside its tensor (bounds-checking build)",
}


class DeviceStatusError(RuntimeError):
    """A bounded device-side wait ran out: results of the launches since the
    last check are not valid (the rows concerned hold NaN)."""


def describe_status(status: int) -> str:
    parts = [msg for bit, msg in STATUS_BITS.items() if status & bit]
    rest = status & ~sum(STATUS_BITS)
    if rest:
        parts.append(f"unknown bits 0x{rest:x}")
    return "; ".join(parts)


def raise_on_status(status: int, where: str = "") -> None:
    if status:
        raise DeviceStatusError(f"fpscan device status 0x{status:x}{' (' + where + ')' if where else ''}: "
                                f"{describe_status(status)}")


def check_device_status(where: str = "") -> None:
    """Synchronously read and clear the current device's status word; raise
    DeviceStatusError (a RuntimeError) if a bounded wait ran out."""
    raise_on_status(device_status(clear=True), where)


def set_wait_limit(seconds: float) -> None:
    """Limit of every bounded device-side wait on the current device
    (default 2 s; 1 ms .. 600 s)."""
    check(load().fpscan_set_wait_limit_ns(int(seconds * 1e9)), "fpscan_set_wait_limit_ns")
