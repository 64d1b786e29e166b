"""Drop-in mirror of the reference's Python op layer (fpscan/ops.py).

Same public names, signatures and error type as the reference:

* ``scan_forward(gates, tokens, reverse=False, out=None)`` -- fpscan/ops.py:47-58
* ``PScan`` autograd function                              -- fpscan/ops.py:61-83
* ``pscan(gates, tokens)``                                 -- fpscan/ops.py:86-87

Tensors are ``(batch, dim, seqlen)``, contiguous, CUDA, float32 / float16 /
bfloat16, power-of-two seqlen in [32, 65536]; the scan runs along the last
axis with a zero initial state.  Invalid input raises ``RuntimeError`` as the
reference's TORCH_CHECKs do (csrc/full_scan/full_scan.h:7-15,
csrc/full_scan/full_scan.cu:181-182, 232, 240-256).  The work is done by
``libfpscan_b200.so`` on the caller's current CUDA stream; there is no CPU
path.
"""
from __future__ import annotations

import os
from typing import Optional

import torch

from . import _lib

__all__ = ["pscan", "scan_forward", "PScan", "pscan_gated", "scan_forward_gated",
           "pscan_anylen", "scan_forward_anylen", "pscan_channels_last",
           "scan_forward_channels_last"]

DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}

# NVTX ranges around the forward and backward (for nsys / ncu timelines):
# FPSCAN_B200_NVTX=1 turns them on; off, the ops pay nothing for them.
NVTX = os.environ.get("FPSCAN_B200_NVTX", "0") == "1"


class _Range:
    __slots__ = ("name",)

    def __init__(self, name: str):
        self.name = name

    def __enter__(self):
        if NVTX:
            torch.cuda.nvtx.range_push(self.name)

    def __exit__(self, *exc):
        if NVTX:
            torch.cuda.nvtx.range_pop()
        return False


def nvtx_range(name: str) -> _Range:
    """Context manager: an NVTX range named `name` when FPSCAN_B200_NVTX=1."""
    return _Range(name)
MIN_SEQLEN = 32
MAX_SEQLEN = 65536


def _check_input(x: torch.Tensor, name: str) -> None:
    # Order and wording follow CHECK_INPUT (csrc/full_scan/full_scan.h:7-15).
    if not isinstance(x, torch.Tensor):
        raise RuntimeError(f"{name} must be a torch.Tensor")
    if not x.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if not x.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
    if x.dtype not in DTYPE_CODES:
        raise RuntimeError(f"{name} must be float16 or bfloat16 or float32")


def validate(gates: torch.Tensor, tokens: torch.Tensor,
             out: Optional[torch.Tensor] = None, any_seqlen: bool = False) -> None:
    """Raise RuntimeError unless (gates, tokens[, out]) form a valid scan call."""
    _check_input(gates, "gates")
    _check_input(tokens, "tokens")
    validate_layout(gates, tokens, out, any_seqlen)


def validate_layout(gates: torch.Tensor, tokens: torch.Tensor,
                    out: Optional[torch.Tensor] = None, any_seqlen: bool = False) -> None:
    """Device-independent checks (shape, dtype, seqlen, out); CPU-testable.
    ``any_seqlen`` accepts every seqlen >= 1 (the *_anylen functions)."""
    if tokens.dim() != 3:
        raise RuntimeError(f"tokens must be 3-D (batch, dim, seqlen), got {tuple(tokens.shape)}")
    if gates.shape != tokens.shape:
        raise RuntimeError(
            f"gates {tuple(gates.shape)} and tokens {tuple(tokens.shape)} must have the same shape")
    if gates.dtype != tokens.dtype:
        raise RuntimeError(f"gates dtype {gates.dtype} must equal tokens dtype {tokens.dtype}")
    if gates.device != tokens.device:
        raise RuntimeError("gates and tokens must be on the same device")
    seqlen = tokens.shape[-1]
    if any_seqlen:
        if seqlen < 1:
            raise RuntimeError(f"seqlen must be >= 1 (got {seqlen})")
    elif seqlen & (seqlen - 1) or not MIN_SEQLEN <= seqlen <= MAX_SEQLEN:
        raise RuntimeError(
            f"seqlen must be a power of 2, >= {MIN_SEQLEN}, <= {MAX_SEQLEN} (got {seqlen})")
    if out is not None:
        if out.shape != tokens.shape or out.dtype != tokens.dtype or out.device != tokens.device:
            raise RuntimeError("out must match tokens in shape, dtype and device")
        if not out.is_contiguous():
            raise RuntimeError("out must be contiguous")


# ---- compiled binding (fpscan_b200/_ext.so, built by build.build_binding):
# the reference's entry points through a thin C++ layer over the same C ABI;
# when it is absent the ctypes path below does the same work.
try:
    from . import _ext as _EXT
except ImportError:  # not built: ctypes path
    _EXT = None

# ---- launch path.  A call's host cost is on the critical path whenever the
# GPU waits for it (small tensors, back-to-back calls), so the common case
# avoids torch.cuda.device / Stream objects: the raw current stream and the
# current device come from torch's C bindings, the device is switched only
# when the tensors live elsewhere, and ctypes functions are looked up once.
_get_device = getattr(torch._C, "_cuda_getDevice", None) or torch.cuda.current_device
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None) or \
    (lambda idx: torch.cuda.current_stream(idx).cuda_stream)
_fns: dict = {}


def _fn(name: str):
    f = _fns.get(name)
    if f is None:
        f = _fns[name] = getattr(_lib.load(), name)
    return f


def _launch(dev: int, name: str, *args) -> None:
    """Call C-ABI entry point `name`(*args, stream) on device `dev` (its
    current stream); raise RuntimeError with the library's message on error."""
    f = _fns.get(name) or _fn(name)
    prev = _get_device()
    if prev == dev:
        rc = f(*args, _raw_stream(dev))
    else:
        torch.cuda.set_device(dev)
        try:
            rc = f(*args, _raw_stream(dev))
        finally:
            torch.cuda.set_device(prev)
    if rc:
        _lib.check(rc, name)


def _fast_valid(gates: torch.Tensor, tokens: torch.Tensor) -> bool:
    """True when (gates, tokens) certainly pass validate(); otherwise the
    caller runs validate() for the precise error."""
    try:
        if not (tokens.is_cuda and gates.is_cuda and tokens.dtype is gates.dtype
                and tokens.dtype in DTYPE_CODES and tokens.dim() == 3
                and gates.shape == tokens.shape and gates.device == tokens.device
                and tokens.is_contiguous() and gates.is_contiguous()):
            return False
    except AttributeError:
        return False
    seqlen = tokens.shape[2]
    return MIN_SEQLEN <= seqlen <= MAX_SEQLEN and not seqlen & (seqlen - 1)


# Split-row workspaces, one per (device, stream): calls ordered on one stream
# may share one; it is zeroed once when (re)allocated.
_workspaces: dict = {}


def _workspace(device: torch.device, stream: int, nbytes: int, kind: str = "split") -> torch.Tensor:
    # one workspace per kernel family: status words of different families
    # carry independent epochs and must not share memory
    key = (device.index, stream, kind)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


# workspace bytes of the split-row path, per (rows, seqlen, dtype, device)
_ws_need: dict = {}


def fullscan_forward(gates: torch.Tensor, tokens: torch.Tensor, out: torch.Tensor,
                     reverse: bool) -> torch.Tensor:
    """Same contract as the reference extension's ``fullscan_forward``
    (csrc/main.cpp:10 -> warpscan_fwd): validates, scans into ``out``, returns it.
    Few-channel, long-sequence shapes go to the split-row kernel, which needs
    a small per-stream workspace (kept here)."""
    if _EXT is not None:
        return _EXT.fullscan_forward(gates, tokens, out, bool(reverse))
    if not (_fast_valid(gates, tokens) and out.shape == tokens.shape
            and out.dtype is tokens.dtype and out.device == tokens.device and out.is_contiguous()):
        validate(gates, tokens, out)
    b, d, l = tokens.shape
    code = DTYPE_CODES[tokens.dtype]
    dev = tokens.get_device()
    key = (b * d, l, code, dev)
    ws_bytes = _ws_need.get(key)
    if ws_bytes is None:
        prev = _get_device()
        torch.cuda.set_device(dev)
        try:
            ws_bytes = _ws_need[key] = _lib.load().fpscan_scan_fwd_workspace_bytes(b, d, l, code)
        finally:
            torch.cuda.set_device(prev)
    if ws_bytes > 0:
        ws = _workspace(tokens.device, _raw_stream(dev), ws_bytes)
        _launch(dev, "fpscan_scan_fwd_ws", gates.data_ptr(), tokens.data_ptr(), out.data_ptr(),
                b, d, l, code, 1 if reverse else 0, ws.data_ptr(), ws.numel())
    else:
        _launch(dev, "fpscan_scan_fwd", gates.data_ptr(), tokens.data_ptr(), out.data_ptr(),
                b, d, l, code, 1 if reverse else 0)
    return out


def _check_state(state: torch.Tensor, tokens: torch.Tensor) -> torch.Tensor:
    if state.shape != tokens.shape[:2]:
        raise RuntimeError(f"initial_state must have shape {tuple(tokens.shape[:2])} "
                           f"(batch, dim), got {tuple(state.shape)}")
    if state.device != tokens.device:
        raise RuntimeError("initial_state must be on the device of tokens")
    return state.to(torch.float32).contiguous()


def scan_forward(gates: torch.Tensor, tokens: torch.Tensor, reverse: bool = False,
                 out: Optional[torch.Tensor] = None,
                 initial_state: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Linear-recurrence scan y[t] = gates[t]*y[t-1] + tokens[t] (no autograd).

    ``reverse=True`` scans from the end: y[t] = gates[t]*y[t+1] + tokens[t].
    ``out`` (optional) receives the result and is returned.
    ``initial_state`` (optional, shape (batch, dim)) replaces the zero state
    entering the first element in scan order (then that element's gate is
    used: y[0] = gates[0]*initial_state + tokens[0]).  The final state is
    the last element of the result in scan order.  The reference has only
    the zero state.
    """
    if initial_state is None and _EXT is not None:
        if out is None:
            return _EXT.scan_forward(gates, tokens, bool(reverse))
        return _EXT.fullscan_forward(gates, tokens, out, bool(reverse))
    if not _fns:
        _lib.load()  # fail loudly before allocating if the library is missing
    if out is None:
        out = torch.empty_like(tokens)
    if initial_state is None:
        return fullscan_forward(gates, tokens, out, reverse)
    validate(gates, tokens, out)
    h0 = _check_state(initial_state, tokens)
    b, d, l = tokens.shape
    _launch(tokens.get_device(), "fpscan_scan_fwd_init", gates.data_ptr(), tokens.data_ptr(),
            out.data_ptr(), h0.data_ptr(), b, d, l, DTYPE_CODES[tokens.dtype],
            1 if reverse else 0)
    return out


def scan_backward(gates: torch.Tensor, y: torch.Tensor, grad_output: torch.Tensor):
    """Fused gradient of ``y = scan_forward(gates, tokens)``: one launch
    returning ``(grad_gates, grad_tokens)``.  Equals the reference's
    PScan.backward composition (fpscan/ops.py:70-83)."""
    if _EXT is not None:
        return _EXT.scan_backward(gates, y, grad_output)
    if not (_fast_valid(gates, grad_output) and _fast_valid(gates, y)):
        validate(gates, grad_output)
        validate(gates, y)
    dgates = torch.empty_like(grad_output)
    dtokens = torch.empty_like(grad_output)
    b, d, l = grad_output.shape
    code = DTYPE_CODES[grad_output.dtype]
    dev = grad_output.get_device()
    key = (b * d, l, code, dev, "bwd")
    ws_bytes = _ws_need.get(key)
    if ws_bytes is None:
        prev = _get_device()
        torch.cuda.set_device(dev)
        try:
            ws_bytes = _ws_need[key] = _lib.load().fpscan_scan_bwd_workspace_bytes(b, d, l, code)
        finally:
            torch.cuda.set_device(prev)
    if ws_bytes > 0:  # few, long rows: the split-row backward
        ws = _workspace(grad_output.device, _raw_stream(dev), ws_bytes, kind="split_bwd")
        _launch(dev, "fpscan_scan_bwd_ws", gates.data_ptr(), y.data_ptr(), grad_output.data_ptr(),
                dgates.data_ptr(), dtokens.data_ptr(), b, d, l, code, ws.data_ptr(), ws.numel())
    else:
        _launch(dev, "fpscan_scan_bwd", gates.data_ptr(), y.data_ptr(), grad_output.data_ptr(),
                dgates.data_ptr(), dtokens.data_ptr(), b, d, l, code)
    return dgates, dtokens


class PScan(torch.autograd.Function):
    """Differentiable scan; saves (gates, out) like fpscan/ops.py:64-67 and
    computes both gradients in one fused kernel."""

    @staticmethod
    def forward(ctx, gates: torch.Tensor, tokens: torch.Tensor) -> torch.Tensor:
        if NVTX:
            with nvtx_range("fpscan.forward"):
                out = scan_forward(gates, tokens)
        else:
            out = scan_forward(gates, tokens)
        ctx.save_for_backward(gates, out)
        return out

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        gates, out = ctx.saved_tensors
        grad_output = grad_output.contiguous()
        if NVTX:
            with nvtx_range("fpscan.backward"):
                return scan_backward(gates, out, grad_output)
        return scan_backward(gates, out, grad_output)


class PScanWithState(torch.autograd.Function):
    """Differentiable scan with an initial state h0 (batch, dim):
    y[0] = gates[0]*h0 + tokens[0].  Gradients: the fused backward with h0
    as y[-1] gives grad_gates and grad_tokens; grad_h0 = gates[0]*grad_tokens[0]."""

    @staticmethod
    def forward(ctx, gates, tokens, h0):
        out = scan_forward(gates, tokens, initial_state=h0)
        h0f = _check_state(h0, tokens)
        ctx.save_for_backward(gates, out, h0f)
        ctx.h0_dtype = h0.dtype
        return out

    @staticmethod
    def backward(ctx, grad_output):
        gates, out, h0f = ctx.saved_tensors
        grad_output = grad_output.contiguous()
        validate(gates, grad_output)
        b, d, l = grad_output.shape
        dgates = torch.empty_like(grad_output)
        dtokens = torch.empty_like(grad_output)
        zero = torch.zeros_like(h0f)
        _launch(grad_output.get_device(), "fpscan_shard_bwd_scan", gates.data_ptr(),
                out.data_ptr(), grad_output.data_ptr(), dgates.data_ptr(), dtokens.data_ptr(),
                zero.data_ptr(), h0f.data_ptr(), b * d, l, DTYPE_CODES[grad_output.dtype])
        dh0 = (gates[..., 0].float() * dtokens[..., 0].float()).to(ctx.h0_dtype)
        return dgates, dtokens, dh0


def pscan(gates: torch.Tensor, tokens: torch.Tensor,
          initial_state: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Differentiable scan (fpscan/ops.py:86-87); ``initial_state`` (batch,
    dim), optional and differentiable, replaces the zero initial state."""
    if initial_state is None:
        return PScan.apply(gates, tokens)
    return PScanWithState.apply(gates, tokens, initial_state)


# --------------------------------------------------------------------------- fused gate producers
GATE_ACTIVATIONS = {"sigmoid": 1, "exp_neg_softplus": 2, "exp": 3}


def _act_code(activation: str) -> int:
    try:
        return GATE_ACTIVATIONS[activation]
    except KeyError:
        raise RuntimeError(f"activation must be one of {sorted(GATE_ACTIVATIONS)}, "
                           f"got {activation!r}") from None


def scan_forward_gated(z: torch.Tensor, tokens: torch.Tensor, activation: str = "sigmoid",
                       reverse: bool = False, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``scan_forward(act(z), tokens)`` with the gate activation applied
    inside the scan kernel (no separate pass over z).  ``activation``:
    "sigmoid", "exp_neg_softplus" (exp(-softplus(z)) = sigmoid(-z)) or "exp"."""
    code = _act_code(activation)
    validate(z, tokens, out)
    if out is None:
        out = torch.empty_like(tokens)
    b, d, l = tokens.shape
    _launch(tokens.get_device(), "fpscan_scan_fwd_act", z.data_ptr(), tokens.data_ptr(),
            out.data_ptr(), b, d, l, DTYPE_CODES[tokens.dtype], 1 if reverse else 0, code)
    return out


class PScanGated(torch.autograd.Function):
    """Differentiable scan of gates = act(z): one forward kernel, one fused
    backward kernel producing (grad_z, grad_tokens)."""

    @staticmethod
    def forward(ctx, z, tokens, activation):
        out = scan_forward_gated(z, tokens, activation)
        ctx.save_for_backward(z, out)
        ctx.code = _act_code(activation)
        return out

    @staticmethod
    def backward(ctx, grad_output):
        z, out = ctx.saved_tensors
        grad_output = grad_output.contiguous()
        validate(z, grad_output)
        dz = torch.empty_like(grad_output)
        dtokens = torch.empty_like(grad_output)
        b, d, l = grad_output.shape
        _launch(grad_output.get_device(), "fpscan_scan_bwd_act", z.data_ptr(), out.data_ptr(),
                grad_output.data_ptr(), dz.data_ptr(), dtokens.data_ptr(), b, d, l,
                DTYPE_CODES[grad_output.dtype], ctx.code)
        return dz, dtokens, None


def pscan_gated(z: torch.Tensor, tokens: torch.Tensor, activation: str = "sigmoid") -> torch.Tensor:
    """Differentiable ``pscan(act(z), tokens)`` with the gate producer fused
    into the scan kernels (forward and backward)."""
    return PScanGated.apply(z, tokens, activation)


# --------------------------------------------------------------------------- any seqlen
def scan_forward_anylen(gates: torch.Tensor, tokens: torch.Tensor, reverse: bool = False,
                        out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``scan_forward`` for any seqlen >= 1: not limited to the reference's
    powers of two in [32, 65536] (csrc/full_scan/full_scan.cu:207-233).
    Zero initial state; ``reverse`` and ``out`` as in ``scan_forward``."""
    _lib.load()
    validate(gates, tokens, out, any_seqlen=True)
    if out is None:
        out = torch.empty_like(tokens)
    b, d, l = tokens.shape
    _launch(tokens.get_device(), "fpscan_scan_fwd_anylen", gates.data_ptr(), tokens.data_ptr(),
            out.data_ptr(), b, d, l, DTYPE_CODES[tokens.dtype], 1 if reverse else 0)
    return out


def scan_backward_anylen(gates: torch.Tensor, out: torch.Tensor, grad_output: torch.Tensor):
    """Fused backward of ``pscan_anylen``: returns (grad_gates, grad_tokens)."""
    validate(gates, grad_output, any_seqlen=True)
    validate(out, grad_output, any_seqlen=True)
    dgates = torch.empty_like(grad_output)
    dtokens = torch.empty_like(grad_output)
    b, d, l = grad_output.shape
    _launch(grad_output.get_device(), "fpscan_scan_bwd_anylen", gates.data_ptr(), out.data_ptr(),
            grad_output.data_ptr(), dgates.data_ptr(), dtokens.data_ptr(), b, d, l,
            DTYPE_CODES[grad_output.dtype])
    return dgates, dtokens


class PScanAnyLen(torch.autograd.Function):
    """``PScan`` for any seqlen >= 1."""

    @staticmethod
    def forward(ctx, gates, tokens):
        out = scan_forward_anylen(gates, tokens)
        ctx.save_for_backward(gates, out)
        return out

    @staticmethod
    def backward(ctx, grad_output):
        gates, out = ctx.saved_tensors
        return scan_backward_anylen(gates, out, grad_output.contiguous())


def pscan_anylen(gates: torch.Tensor, tokens: torch.Tensor) -> torch.Tensor:
    """Differentiable ``pscan`` for any seqlen >= 1 (e.g. 1000, 3, 200000)."""
    return PScanAnyLen.apply(gates, tokens)


# --------------------------------------------------------------------------- channel-last layout
def validate_channels_last(gates: torch.Tensor, tokens: torch.Tensor,
                           out: Optional[torch.Tensor] = None) -> None:
    """Checks for (batch, seqlen, dim) tensors scanned along seqlen."""
    _check_input(gates, "gates")
    _check_input(tokens, "tokens")
    if tokens.dim() != 3:
        raise RuntimeError(f"tokens must be 3-D (batch, seqlen, dim), got {tuple(tokens.shape)}")
    if gates.shape != tokens.shape or gates.dtype != tokens.dtype or gates.device != tokens.device:
        raise RuntimeError("gates and tokens must have the same shape, dtype and device")
    if tokens.shape[1] < 1:
        raise RuntimeError(f"seqlen must be >= 1 (got {tokens.shape[1]})")
    vec = 16 // tokens.element_size()
    if tokens.shape[2] % vec:
        raise RuntimeError(f"dim must be a multiple of {vec} for {tokens.dtype} (got {tokens.shape[2]})")
    if out is not None:
        if out.shape != tokens.shape or out.dtype != tokens.dtype or out.device != tokens.device:
            raise RuntimeError("out must match tokens in shape, dtype and device")
        if not out.is_contiguous():
            raise RuntimeError("out must be contiguous")


def _cl_workspace(t: torch.Tensor, backward: bool) -> torch.Tensor:
    b, l, d = t.shape
    nbytes = _fn("fpscan_cl_workspace_bytes")(b, l, d, DTYPE_CODES[t.dtype], 1 if backward else 0)
    return _workspace(t.device, _raw_stream(t.get_device()), nbytes, kind="channels_last")


def scan_forward_channels_last(gates: torch.Tensor, tokens: torch.Tensor, reverse: bool = False,
                               out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Scan along dim 1 of (batch, seqlen, dim) tensors:
    y[:, t] = gates[:, t] * y[:, t-1] + tokens[:, t] (zero initial state).

    Replaces the reference's documented channel-last usage
    ``scan_forward(g.mT.contiguous(), x.mT.contiguous()).mT.contiguous()``
    (README.md:94-99) without the transposes.  Any seqlen >= 1; dim must be a
    multiple of 16 bytes' worth of elements."""
    _lib.load()
    validate_channels_last(gates, tokens, out)
    if out is None:
        out = torch.empty_like(tokens)
    b, l, d = tokens.shape
    if b == 0 or d == 0:
        return out
    ws = _cl_workspace(tokens, False)
    _launch(tokens.get_device(), "fpscan_scan_fwd_cl", gates.data_ptr(), tokens.data_ptr(),
            out.data_ptr(), b, l, d, DTYPE_CODES[tokens.dtype], 1 if reverse else 0,
            ws.data_ptr(), ws.numel())
    return out


def scan_backward_channels_last(gates: torch.Tensor, out: torch.Tensor,
                                grad_output: torch.Tensor):
    """Fused backward of ``pscan_channels_last``: (grad_gates, grad_tokens)."""
    validate_channels_last(gates, grad_output)
    validate_channels_last(out, grad_output)
    dgates = torch.empty_like(grad_output)
    dtokens = torch.empty_like(grad_output)
    b, l, d = grad_output.shape
    if b == 0 or d == 0:
        return dgates, dtokens
    ws = _cl_workspace(grad_output, True)
    _launch(grad_output.get_device(), "fpscan_scan_bwd_cl", gates.data_ptr(), out.data_ptr(),
            grad_output.data_ptr(), dgates.data_ptr(), dtokens.data_ptr(), b, l, d,
            DTYPE_CODES[grad_output.dtype], ws.data_ptr(), ws.numel())
    return dgates, dtokens


class PScanChannelsLast(torch.autograd.Function):
    """``PScan`` on (batch, seqlen, dim) tensors."""

    @staticmethod
    def forward(ctx, gates, tokens):
        out = scan_forward_channels_last(gates, tokens)
        ctx.save_for_backward(gates, out)
        return out

    @staticmethod
    def backward(ctx, grad_output):
        gates, out = ctx.saved_tensors
        return scan_backward_channels_last(gates, out, grad_output.contiguous())


def pscan_channels_last(gates: torch.Tensor, tokens: torch.Tensor) -> torch.Tensor:
    """Differentiable scan along dim 1 of (batch, seqlen, dim) tensors."""
    return PScanChannelsLast.apply(gates, tokens)
