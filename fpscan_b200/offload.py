"""Scan forward + backward for tensors that live in host memory.

For callers whose (batch, dim, seqlen) tensors are in (pinned) host memory,
``scan_fwd_bwd_host`` streams row blocks through the GPU with three CUDA
streams so that host->device copies, the two kernels and device->host copies
of different blocks overlap (H2D and D2H use the two copy engines
concurrently; the kernels are far faster than PCIe):

    h2d stream:      [copy in 0][copy in 1][copy in 2] ...
    compute stream:            [fwd+bwd 0][fwd+bwd 1] ...
    d2h stream:                           [copy out 0][copy out 1] ...

``depth`` device buffer sets are recycled; block i reuses the set of block
i-depth once that block's results have left the device (event ordering, no
host synchronisation inside the loop).  Results are those of
``pscan``/``PScan.backward`` on the same data: y, grad_gates, grad_tokens.
The reference has no host-memory path; this is the call `bench.py` times as
its end-to-end figure.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from .ops import DTYPE_CODES, validate_layout

__all__ = ["scan_fwd_bwd_host"]


def _stream_ptr(s: torch.cuda.Stream) -> int:
    return s.cuda_stream


def scan_fwd_bwd_host(gates: torch.Tensor, tokens: torch.Tensor, grad_out: torch.Tensor,
                      y: Optional[torch.Tensor] = None, dgates: Optional[torch.Tensor] = None,
                      dtokens: Optional[torch.Tensor] = None, *,
                      device: Optional[torch.device] = None, block_bytes: int = 128 << 20,
                      depth: int = 3):
    """Forward scan and fused backward of host-resident tensors.

    gates, tokens, grad_out: (batch, dim, seqlen) contiguous CPU tensors
    (pin them for asynchronous copies).  y, dgates, dtokens: optional
    preallocated CPU outputs (allocated pinned when omitted).  Returns
    (y, dgates, dtokens).  Blocks until the results are in host memory.
    """
    for name, t in (("gates", gates), ("tokens", tokens), ("grad_out", grad_out)):
        if t.is_cuda:
            raise RuntimeError(f"{name} must be a host tensor (use pscan for device tensors)")
        if not t.is_contiguous():
            raise RuntimeError(f"{name} must be contiguous")
    validate_layout(gates, tokens)
    validate_layout(gates, grad_out)
    lib = _lib.load()
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    b, d, L = tokens.shape
    rows = b * d
    outs = []
    for t in (y, dgates, dtokens):
        if t is None:
            t = torch.empty_like(tokens, pin_memory=True)
        elif t.shape != tokens.shape or t.dtype != tokens.dtype or t.is_cuda or not t.is_contiguous():
            raise RuntimeError("outputs must be contiguous host tensors shaped like tokens")
        outs.append(t)
    if rows == 0:
        return tuple(outs)

    es = tokens.element_size()
    blk = max(1, min(rows, block_bytes // (L * es)))
    nblk = (rows + blk - 1) // blk
    depth = max(1, min(depth, nblk))
    code = DTYPE_CODES[tokens.dtype]
    host_in = [t.view(rows, L) for t in (gates, tokens, grad_out)]
    host_out = [t.view(rows, L) for t in outs]

    with torch.cuda.device(device):
        cur = torch.cuda.current_stream(device)
        s_in = torch.cuda.Stream(device)
        s_cmp = torch.cuda.Stream(device)
        s_out = torch.cuda.Stream(device)
        bufs = [[torch.empty(blk, L, dtype=tokens.dtype, device=device) for _ in range(6)]
                for _ in range(depth)]
        in_done = [torch.cuda.Event() for _ in range(depth)]
        cmp_done = [torch.cuda.Event() for _ in range(depth)]
        out_done = [None] * depth
        for q in (s_in, s_cmp, s_out):
            q.wait_stream(cur)  # the caller's pending work (e.g. buffer allocation)
        for i in range(nblk):
            slot = i % depth
            r0, r1 = i * blk, min(rows, (i + 1) * blk)
            n = r1 - r0
            g_d, x_d, go_d, y_d, dg_d, dt_d = (t[:n] for t in bufs[slot])
            with torch.cuda.stream(s_in):
                if out_done[slot] is not None:
                    s_in.wait_event(out_done[slot])
                for dst, src in zip((g_d, x_d, go_d), host_in):
                    dst.copy_(src[r0:r1], non_blocking=True)
                in_done[slot].record(s_in)
            s_cmp.wait_event(in_done[slot])
            _lib.check(lib.fpscan_scan_fwd(g_d.data_ptr(), x_d.data_ptr(), y_d.data_ptr(), 1, n, L,
                                           code, 0, _stream_ptr(s_cmp)), "fpscan_scan_fwd")
            _lib.check(lib.fpscan_scan_bwd(g_d.data_ptr(), y_d.data_ptr(), go_d.data_ptr(),
                                           dg_d.data_ptr(), dt_d.data_ptr(), 1, n, L, code,
                                           _stream_ptr(s_cmp)), "fpscan_scan_bwd")
            cmp_done[slot].record(s_cmp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(cmp_done[slot])
                for dst, src in zip(host_out, (y_d, dg_d, dt_d)):
                    dst[r0:r1].copy_(src, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(s_out)
                out_done[slot] = ev
        # Every block's copy-out depends on its kernels and copy-in, so this
        # covers all work issued above (and makes freeing `bufs` safe).
        s_out.synchronize()
    return tuple(outs)
