"""Multi-GPU scan: channel sharding and sequence sharding (one process per GPU).

The reference has no multi-GPU path; these two modes extend its API.

Channel sharding (``channel_slice`` / ``channel_sharded_pscan``): the
batch*dim rows are independent, so each rank scans its contiguous block of
rows with the single-GPU kernels and nothing is exchanged.

Sequence sharding (``seq_sharded_pscan``): rank r holds positions
[r*Lr, (r+1)*Lr) of every row.  A shard acts on its incoming state as an
affine map y_out = A*y_in + B, so:

forward
  1. reduce: per row (A_r = prod gates, B_r = local scan's last value)
     -- reads gates and tokens once, writes 2 floats per row;
  2. all_gather_into_tensor of the [2, rows] fp32 maps (NCCL over NVLink);
  3. combine maps of ranks < r into y_init (device kernel, no host sync);
  4. scan with initial state y_init.
backward (dtokens[t] = gates[t+1]*dtokens[t+1] + g[t], dgates[t] = dtokens[t]*y[t-1])
  1. reduce: per row v_r = gates_r[0] * dtokens_r[0] with nothing entering
     from the right; the map of shard r on the value entering it is
     (A_r, v_r) with the same A_r as the forward (so no gate halo is needed);
  2. all_gather of (A_r, v_r);
  3. combine maps of ranks > r into the value entering at the last element;
  4. fused backward with that addend and y_init (= y of the previous shard's
     last element) for dgates at the first position.

Chained mode (``seq_sharded_pscan(..., mode="chain")``, the default where it
applies): the reduce passes and the all-gathers disappear.  Each rank's scan
kernel waits, row by row, for the state entering the row from rank r-1 and
hands the row's final state to rank r+1 as soon as the row is done, through
per-rank mailboxes mapped into the neighbours with CUDA IPC (stores and
loads over NVLink; epoch-tagged words, bounded waits).  A wait that runs out
(a neighbour more than the wait limit behind) makes the rows concerned NaN
and sets a device status bit; every chained call queues a non-blocking read
of that bit, and the next chained call (or ``check_chains()``) raises
``DeviceStatusError``.
The ranks run as a pipeline one row apart, each reading its shard once:
forward 3*N*s and backward 5*N*s bytes per rank, as on one GPU.  The
backward chain runs the other way; the state each rank received in the
forward is y[-1] of its shard for dgates.  Needs one process per distinct
GPU of one node and a local seqlen larger than one chunk.

The device-side steps are behind ``LocalOps`` so the exchange logic can be
exercised on CPU ranks (gloo) with a CPU implementation injected by tests;
the default, ``CudaOps``, calls libfpscan_b200.so and is the only
implementation in this package.
"""
from __future__ import annotations

import socket
from typing import Optional

import torch
import torch.distributed as dist

from . import _lib
from .ops import DTYPE_CODES, nvtx_range, pscan, scan_backward, scan_forward, validate

import ctypes

__all__ = [
    "RankChain",
    "check_chains",
    "channel_slice",
    "channel_sharded_pscan",
    "seq_sharded_pscan",
    "SeqShardedPScan",
    "CudaOps",
]


# --------------------------------------------------------------------------- channel sharding
def channel_slice(rows: int, rank: int, world: int) -> tuple[int, int]:
    """[lo, hi) of the flattened batch*dim rows owned by ``rank``; the first
    ``rows % world`` ranks get one extra row."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"invalid rank {rank} for world {world}")
    base, extra = divmod(rows, world)
    lo = rank * base + min(rank, extra)
    hi = lo + base + (1 if rank < extra else 0)
    return lo, hi


def local_channels(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's rows of a (batch, dim, L) tensor, as a (1, rows_local, L) view."""
    b, d, l = x.shape
    lo, hi = channel_slice(b * d, rank, world)
    return x.reshape(1, b * d, l)[:, lo:hi]


def channel_sharded_pscan(gates_local: torch.Tensor, tokens_local: torch.Tensor) -> torch.Tensor:
    """Differentiable scan of this rank's channel block: no communication."""
    return pscan(gates_local, tokens_local)


# --------------------------------------------------------------------------- sequence sharding
class CudaOps:
    """Device steps of the sequence-sharded scan, on libfpscan_b200.so."""

    @staticmethod
    def _rows_len(x: torch.Tensor):
        return x.numel() // x.shape[-1], x.shape[-1]

    @staticmethod
    def _stream(x: torch.Tensor) -> int:
        return torch.cuda.current_stream(x.device).cuda_stream

    def fwd_reduce(self, gates, tokens):
        rows, L = self._rows_len(tokens)
        carry = torch.empty(2, rows, dtype=torch.float32, device=tokens.device)
        _lib.call("fpscan_shard_fwd_reduce", gates.data_ptr(), tokens.data_ptr(),
                  carry[0].data_ptr(), carry[1].data_ptr(), rows, L,
                  DTYPE_CODES[tokens.dtype], self._stream(tokens))
        return carry

    def fwd_scan(self, gates, tokens, y_init):
        rows, L = self._rows_len(tokens)
        out = torch.empty_like(tokens)
        _lib.call("fpscan_shard_fwd_scan", gates.data_ptr(), tokens.data_ptr(), out.data_ptr(),
                  y_init.data_ptr(), rows, L, DTYPE_CODES[tokens.dtype], self._stream(tokens))
        return out

    def fwd_scan_zero(self, gates, tokens):
        return scan_forward(gates, tokens)

    def bwd_reduce(self, gates, grad_out):
        rows, L = self._rows_len(grad_out)
        v = torch.empty(rows, dtype=torch.float32, device=grad_out.device)
        _lib.call("fpscan_shard_bwd_reduce", gates.data_ptr(), grad_out.data_ptr(), v.data_ptr(),
                  rows, L, DTYPE_CODES[grad_out.dtype], self._stream(grad_out))
        return v

    def bwd_scan(self, gates, y, grad_out, addend, y_prev):
        rows, L = self._rows_len(grad_out)
        dg = torch.empty_like(grad_out)
        dt = torch.empty_like(grad_out)
        _lib.call("fpscan_shard_bwd_scan", gates.data_ptr(), y.data_ptr(), grad_out.data_ptr(),
                  dg.data_ptr(), dt.data_ptr(), addend.data_ptr(), y_prev.data_ptr(), rows, L,
                  DTYPE_CODES[grad_out.dtype], self._stream(grad_out))
        return dg, dt

    def bwd_scan_zero(self, gates, y, grad_out):
        return scan_backward(gates, y, grad_out)

    def combine(self, gathered, world, rank, reverse):
        rows = gathered.shape[-1]
        out = torch.empty(rows, dtype=torch.float32, device=gathered.device)
        _lib.call("fpscan_carry_combine", gathered.data_ptr(), world, rank, rows,
                  1 if reverse else 0, out.data_ptr(), self._stream(gathered))
        return out


def _all_gather_maps(local: torch.Tensor, world: int, group) -> torch.Tensor:
    """[2, rows] fp32 per rank -> [world, 2, rows]."""
    flat = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype,
                       device=local.device)
    dist.all_gather_into_tensor(flat, local.contiguous(), group=group)
    return flat.view((world,) + tuple(local.shape))


def _validate_local(gates: torch.Tensor, tokens: torch.Tensor, on_cuda: bool) -> None:
    if on_cuda:
        validate(gates, tokens)
    else:
        if gates.shape != tokens.shape or gates.dtype != tokens.dtype:
            raise RuntimeError("gates and tokens must have the same shape and dtype")
    L = tokens.shape[-1]
    if L < 32 or L & (L - 1):
        raise RuntimeError(f"local seqlen must be a power of 2 >= 32 (got {L})")


class SeqShardedPScan(torch.autograd.Function):
    """Differentiable scan over sequences split along seqlen across ranks."""

    @staticmethod
    def forward(ctx, gates, tokens, group, ops):
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        with nvtx_range("fpscan.seq.forward.reduce"):
            carry = ops.fwd_reduce(gates, tokens)                # [2, rows]: (A_r, B_r)
        with nvtx_range("fpscan.seq.forward.exchange"):
            gathered = _all_gather_maps(carry, world, group)     # [world, 2, rows]
            y_init = ops.combine(gathered, world, rank, reverse=False)
        with nvtx_range("fpscan.seq.forward.scan"):
            if rank == 0:
                y = ops.fwd_scan_zero(gates, tokens)
            else:
                y = ops.fwd_scan(gates, tokens, y_init)
        ctx.save_for_backward(gates, y, carry[0].clone(), y_init)
        ctx.group, ctx.ops, ctx.world, ctx.rank = group, ops, world, rank
        return y

    @staticmethod
    def backward(ctx, grad_out):
        gates, y, a_local, y_init = ctx.saved_tensors
        ops, world, rank = ctx.ops, ctx.world, ctx.rank
        grad_out = grad_out.contiguous()
        with nvtx_range("fpscan.seq.backward.reduce"):
            v = ops.bwd_reduce(gates, grad_out)
        with nvtx_range("fpscan.seq.backward.exchange"):
            gathered = _all_gather_maps(torch.stack([a_local, v]), world, ctx.group)
            addend = ops.combine(gathered, world, rank, reverse=True)
        with nvtx_range("fpscan.seq.backward.scan"):
            if world == 1:
                dg, dt = ops.bwd_scan_zero(gates, y, grad_out)
            else:
                dg, dt = ops.bwd_scan(gates, y, grad_out, addend, y_init)
        return dg, dt, None, None


# --------------------------------------------------------------------------- chained mode
class RankChain:
    """Mailboxes linking this rank to ranks r-1 and r+1 (same rows on every
    rank).  Collective to construct: every rank of ``group`` must create its
    chain for the same ``rows`` in the same order.  ``depth`` ring slots per
    direction bound how many chained calls one rank may run ahead of its
    neighbour (the producer waits for the slot's previous use to be consumed)."""

    def __init__(self, rows: int, device: torch.device, group=None, depth: int = 4):
        self.lib = _lib.load()
        self.group, self.rows, self.depth = group, rows, depth
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        idx = torch.device(device).index
        # Linked kernels wait on one another: two ranks on one GPU would be
        # two such kernels on one device, which nothing schedules together.
        ids = [None] * self.world
        dist.all_gather_object(ids, (socket.gethostname(), _device_uuid(idx)), group=group)
        if len(set(ids)) != self.world:
            raise RuntimeError("chained sequence sharding needs one distinct GPU per rank")
        if len({h for h, _ in ids}) != 1:
            raise RuntimeError("chained sequence sharding needs all ranks on one node")
        with torch.cuda.device(idx):
            mb = ctypes.c_void_p()
            _lib.check(self.lib.fpscan_link_create(rows, depth, ctypes.byref(mb)),
                       "fpscan_link_create")
            self.local = mb.value
            h = ctypes.create_string_buffer(64)
            _lib.check(self.lib.fpscan_link_ipc_handle(self.local, h), "fpscan_link_ipc_handle")
            handles = [None] * self.world
            dist.all_gather_object(handles, h.raw, group=group)
            self.prev = self._open(handles[self.rank - 1]) if self.rank > 0 else None
            self.next = self._open(handles[self.rank + 1]) if self.rank < self.world - 1 else None
        self.device_index = idx
        self.fwd_epoch = 0
        self.bwd_epoch = 0
        # Failure detection: after every linked launch a read-and-clear of
        # the device status word is queued behind it (a 1-thread kernel into
        # _status_dev, copied to pinned host memory, and an event); the host
        # checks it once the event has completed -- at the next chained call
        # without blocking, or in check(block=True).
        self._status_dev = torch.zeros(1, dtype=torch.int32, device=device)
        self._pending: list = []

    def _open(self, handle: bytes) -> int:
        p = ctypes.c_void_p()
        _lib.check(self.lib.fpscan_link_open(ctypes.create_string_buffer(handle, 64),
                                             ctypes.byref(p)), "fpscan_link_open")
        return p.value

    @staticmethod
    def _bump(e: int) -> int:
        e = (e + 1) & 0xFFFFFFFF
        return e or 1

    def next_fwd_epoch(self) -> int:
        self.fwd_epoch = self._bump(self.fwd_epoch)
        return self.fwd_epoch

    def next_bwd_epoch(self) -> int:
        self.bwd_epoch = self._bump(self.bwd_epoch)
        return self.bwd_epoch

    def after_launch(self, where: str) -> None:
        """Queue the status check of the launch just issued on the current stream."""
        stream = torch.cuda.current_stream(self.device_index)
        host = torch.empty(1, dtype=torch.int32, pin_memory=True)
        _lib.check(self.lib.fpscan_status_snapshot(self._status_dev.data_ptr(), stream.cuda_stream),
                   "fpscan_status_snapshot")
        host.copy_(self._status_dev, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(stream)
        self._pending.append((ev, host, where))

    def check(self, block: bool = False) -> None:
        """Raise DeviceStatusError if a queued status check shows that a
        bounded wait ran out (a neighbouring rank fell behind by more than
        the wait limit; the rows concerned hold NaN).  With block=False only
        checks whose launches have completed are read."""
        keep = []
        for ev, host, where in self._pending:
            if block:
                ev.synchronize()
            if block or ev.query():
                status = int(host.item())
                if status:
                    self._pending = []
                    _lib.raise_on_status(status, f"rank {self.rank}, {where}")
            else:
                keep.append((ev, host, where))
        self._pending = keep

    def close(self) -> None:
        """Unmap the neighbours' mailboxes, then (after every rank has done
        the same) free this one.  Collective."""
        if self.local is None:
            return
        with torch.cuda.device(self.device_index):
            torch.cuda.synchronize()
            for p in (self.prev, self.next):
                if p:
                    self.lib.fpscan_link_close(p)
            dist.barrier(group=self.group)
            self.lib.fpscan_link_destroy(self.local)
        self.local = self.prev = self.next = None


def _device_uuid(idx: int) -> str:
    props = torch.cuda.get_device_properties(idx)
    return str(getattr(props, "uuid", idx))


_chains: dict = {}


def _chain_for(rows: int, device: torch.device, group) -> RankChain:
    key = (id(group), rows, device.index)
    ch = _chains.get(key)
    if ch is None:
        ch = _chains[key] = RankChain(rows, device, group)
    return ch


def chain_supported(tokens_local: torch.Tensor) -> bool:
    """Whether the chained mode applies: CUDA tensors whose local seqlen
    exceeds one chunk of the linked kernels (1024 fp32 / 2048 half elements
    forward; 2048 / 4096 backward)."""
    if not tokens_local.is_cuda:
        return False
    vec = 16 // tokens_local.element_size()
    return tokens_local.shape[-1] > 256 * vec * 2


class ChainedSeqShardedPScan(torch.autograd.Function):
    """Sequence-sharded scan with the row carries handed rank to rank over
    NVLink inside the scan kernels (no reduce pass, no collective)."""

    @staticmethod
    def forward(ctx, gates, tokens, chain):
        rows, L = tokens.numel() // tokens.shape[-1], tokens.shape[-1]
        code = DTYPE_CODES[tokens.dtype]
        y = torch.empty_like(tokens)
        y_init = (torch.empty(rows, dtype=torch.float32, device=tokens.device)
                  if chain.prev else None)
        chain.check(block=False)
        e = chain.next_fwd_epoch()
        with torch.cuda.device(tokens.device), nvtx_range("fpscan.chain.forward"):
            _lib.call("fpscan_shard_fwd_link", gates.data_ptr(), tokens.data_ptr(), y.data_ptr(),
                      y_init.data_ptr() if y_init is not None else None, rows, L, code,
                      chain.local, chain.prev, chain.next, e, chain.depth,
                      torch.cuda.current_stream(tokens.device).cuda_stream)
            chain.after_launch(f"forward epoch {e}")
        ctx.save_for_backward(gates, y, y_init if y_init is not None else y.new_empty(0))
        ctx.chain, ctx.has_init = chain, y_init is not None
        return y

    @staticmethod
    def backward(ctx, grad_out):
        gates, y, y_init = ctx.saved_tensors
        chain = ctx.chain
        grad_out = grad_out.contiguous()
        rows, L = grad_out.numel() // grad_out.shape[-1], grad_out.shape[-1]
        dg = torch.empty_like(grad_out)
        dt = torch.empty_like(grad_out)
        chain.check(block=False)
        e = chain.next_bwd_epoch()
        with torch.cuda.device(grad_out.device), nvtx_range("fpscan.chain.backward"):
            _lib.call("fpscan_shard_bwd_link", gates.data_ptr(), y.data_ptr(), grad_out.data_ptr(),
                      dg.data_ptr(), dt.data_ptr(), y_init.data_ptr() if ctx.has_init else None,
                      rows, L, DTYPE_CODES[grad_out.dtype], chain.local, chain.prev, chain.next,
                      e, chain.depth, torch.cuda.current_stream(grad_out.device).cuda_stream)
            chain.after_launch(f"backward epoch {e}")
        return dg, dt, None


def check_chains(block: bool = True) -> None:
    """Check every chain of this process (see RankChain.check): call it at a
    point where the host may wait, e.g. before the optimizer step, to raise
    for the step that failed rather than the next one."""
    for ch in list(_chains.values()):
        ch.check(block=block)


def seq_sharded_pscan(gates_local: torch.Tensor, tokens_local: torch.Tensor,
                      group: Optional[dist.ProcessGroup] = None, ops=None,
                      mode: str = "auto") -> torch.Tensor:
    """Differentiable scan of this rank's sequence shard ``(batch, dim, L/world)``.

    Rank r must hold positions [r*L/world, (r+1)*L/world) of every row, all
    ranks the same rows, and every rank must make the same calls in the same
    order.  ``mode``: "allgather" -- reduce, one all-gather of 2*rows fp32
    (NCCL), scan with the combined state, both directions; "chain" -- the
    carries pass rank to rank inside the scan kernels over NVLink (one
    distinct GPU per rank, one node, local seqlen above one chunk); "auto"
    -- "chain" where it applies, else "allgather".
    """
    if mode not in ("auto", "chain", "allgather"):
        raise ValueError(f"mode must be 'auto', 'chain' or 'allgather' (got {mode!r})")
    if ops is None:
        ops = CudaOps()
    _validate_local(gates_local, tokens_local, isinstance(ops, CudaOps))
    world = dist.get_world_size(group)
    use_chain = (mode == "chain" or (mode == "auto" and isinstance(ops, CudaOps)
                                     and world > 1 and chain_supported(tokens_local)))
    if use_chain:
        if not isinstance(ops, CudaOps) or not chain_supported(tokens_local) or world < 2:
            raise RuntimeError("chained mode needs CUDA shards on 2+ ranks with a local seqlen "
                               "above one chunk")
        rows = tokens_local.numel() // tokens_local.shape[-1]
        chain = _chain_for(rows, tokens_local.device, group)
        return ChainedSeqShardedPScan.apply(gates_local, tokens_local, chain)
    return SeqShardedPScan.apply(gates_local, tokens_local, group, ops)
