"""Failure detection on one GPU, without faulting it: bounded device waits
that are made to run out on purpose, through the C ABI.

A chained sequence-sharded scan kernel is given an upstream (or downstream)
mailbox that nothing ever writes, with the wait limit set to 50 ms.  The
launch must return on its own within the limit (per row, rows waiting in
parallel), set the neighbour-timeout status bit, leave NaN -- never
plausible values -- in the rows that waited, and the Python layer must raise
DeviceStatusError.  The GPU context stays usable: a normal scan afterwards is
exact and leaves the status clean.
"""
import ctypes
import time

import numpy as np
import pytest
import torch

import fpscan_b200 as fp
import oracle
from fpscan_b200 import _lib

pytestmark = pytest.mark.gpu

LINK_TIMEOUT = 8


def _mailbox(lib, rows, depth=4):
    mb = ctypes.c_void_p()
    _lib.check(lib.fpscan_link_create(rows, depth, ctypes.byref(mb)), "fpscan_link_create")
    return mb.value


@pytest.fixture
def short_wait():
    fp.set_wait_limit(0.05)
    yield 0.05
    fp.set_wait_limit(2.0)


def _inputs(rows, L, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    g = 0.99 + 0.01 * torch.rand(1, rows, L, generator=gen, device="cuda")
    x = torch.randn(1, rows, L, generator=gen, device="cuda") / L
    return g, x


def test_upstream_rank_never_sends_forward(short_wait):
    lib = _lib.load()
    rows, L, depth = 3, 4096, 4
    local, upstream = _mailbox(lib, rows, depth), _mailbox(lib, rows, depth)
    g, x = _inputs(rows, L, 1)
    y = torch.zeros_like(x)
    rec = torch.zeros(rows, dtype=torch.float32, device="cuda")
    _lib.device_status(clear=True)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _lib.check(lib.fpscan_shard_fwd_link(g.data_ptr(), x.data_ptr(), y.data_ptr(), rec.data_ptr(),
                                         rows, L, 0, local, upstream, None, 1, depth,
                                         torch.cuda.current_stream().cuda_stream),
               "fpscan_shard_fwd_link")
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert elapsed < 1.5, elapsed
    assert torch.isnan(y).all()            # the rows that waited: NaN, not zeros
    assert torch.isnan(rec).all()
    with pytest.raises(fp.DeviceStatusError, match="neighbouring rank"):
        fp.check_device_status("upstream never sent")
    for mb in (local, upstream):
        lib.fpscan_link_destroy(mb)


def test_downstream_rank_never_sends_backward(short_wait):
    lib = _lib.load()
    rows, L, depth = 2, 8192, 4
    local, downstream = _mailbox(lib, rows, depth), _mailbox(lib, rows, depth)
    g, x = _inputs(rows, L, 2)
    y = fp.scan_forward(g, x)
    go = torch.randn_like(x)
    dg, dt = torch.zeros_like(x), torch.zeros_like(x)
    _lib.device_status(clear=True)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _lib.check(lib.fpscan_shard_bwd_link(g.data_ptr(), y.data_ptr(), go.data_ptr(), dg.data_ptr(),
                                         dt.data_ptr(), None, rows, L, 0, local, None, downstream,
                                         1, depth, torch.cuda.current_stream().cuda_stream),
               "fpscan_shard_bwd_link")
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 1.5
    assert torch.isnan(dt).all() and torch.isnan(dg).all()
    status = _lib.device_status(clear=True)
    assert status & LINK_TIMEOUT
    for mb in (local, downstream):
        lib.fpscan_link_destroy(mb)


def test_status_snapshot_is_asynchronous_and_clears(short_wait):
    """fpscan_status_snapshot reads and clears the status word on the stream,
    without a host synchronisation; a later healthy scan is exact."""
    lib = _lib.load()
    rows, L, depth = 1, 4096, 4
    local, upstream = _mailbox(lib, rows, depth), _mailbox(lib, rows, depth)
    g, x = _inputs(rows, L, 3)
    y = torch.empty_like(x)
    _lib.device_status(clear=True)
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.fpscan_shard_fwd_link(g.data_ptr(), x.data_ptr(), y.data_ptr(), None, rows, L,
                                         0, local, upstream, None, 1, depth, stream), "link")
    snap = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    _lib.check(lib.fpscan_status_snapshot(snap.data_ptr(), stream), "fpscan_status_snapshot")
    assert int(snap.item()) & LINK_TIMEOUT
    assert _lib.device_status(clear=True) == 0  # the snapshot cleared it
    # the context is healthy: an ordinary scan is exact
    y2 = fp.scan_forward(g, x)
    ref = oracle.scan_f64(g.double().cpu().numpy(), x.double().cpu().numpy())
    assert oracle.normwise_error(y2.double().cpu().numpy(), ref) <= 1e-5
    fp.check_device_status("after recovery")
    for mb in (local, upstream):
        lib.fpscan_link_destroy(mb)


def test_wait_limit_range_is_checked():
    with pytest.raises(RuntimeError):
        fp.set_wait_limit(1e-6)
    with pytest.raises(RuntimeError):
        fp.set_wait_limit(1e4)
