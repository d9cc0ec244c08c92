"""Python surface of the fused multi-head MLP, call-compatible with dtadpole/flashMLP.

    Z = X @ W1,  H = act(Z),  O = H @ W2          per head
    X: (H, B, D)   W1: (H, D, E)   W2: (H, E, D)   O: (H, B, D)

`flashmlp_fwd`, `flashmlp_bwd`, `FlashMLPFunction` and `FlashMLP` keep the reference's
names, signatures, shape assertions (and their messages) and return conventions
(flashmlp.py:428-616). Their compute goes through libflashmlp_b200.so (hand-written
sm_100a kernels); there is no other compute path.
"""
from __future__ import annotations

import contextlib
import ctypes
import threading
from typing import Tuple

import numpy as np
import torch

from . import _lib

_ACT_CODES = {
    "leaky_relu": _lib.FMLP_ACT_LEAKY_RELU,
    "silu": _lib.FMLP_ACT_SILU,
    "sigmoid": _lib.FMLP_ACT_SIGMOID,
}


def activation_code(activation: str) -> int:
    """Maps an activation name to the C ABI code. Like the reference, any other string
    (including "") means no activation (flashmlp.py:146-147)."""
    return _ACT_CODES.get(activation, _lib.FMLP_ACT_LINEAR)


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return _lib.FMLP_DTYPE_BF16
    if t.dtype == torch.float16:
        return _lib.FMLP_DTYPE_F16
    if t.dtype == torch.float32:  # TF32 tensor-core products, as tl.dot on fp32 tensors
        return _lib.FMLP_DTYPE_F32
    raise TypeError(
        f"flashmlp_b200 supports torch.bfloat16, torch.float16 and torch.float32 tensors, got {t.dtype}"
    )


def _check_tensors(*ts: torch.Tensor) -> torch.device:
    dev = ts[0].device
    if dev.type != "cuda":
        raise RuntimeError("flashmlp_b200 kernels need CUDA tensors (there is no CPU path)")
    for t in ts[1:]:
        if t.device != dev:
            raise RuntimeError(f"all tensors must be on {dev}, got one on {t.device}")
        if t.dtype != ts[0].dtype:
            raise TypeError(f"all tensors must share one dtype, got {ts[0].dtype} and {t.dtype}")
    _dtype_code(ts[0])
    return dev


def _ptr(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def _on_device(dev: torch.device):
    """torch.cuda.device(dev), or nothing when dev is already the current device (the
    common case; the context manager costs microseconds per call at small shapes)."""
    if dev.index is None or dev.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(dev)


# fmlp_bwd_workspace_size per (device, shape, dtype): it depends only on those (the SM
# count enters the split rule), and the lookup is on the per-call host path
_WS_FULL = {}


_WS_LIMIT = threading.local()


@contextlib.contextmanager
def backward_workspace_limit(nbytes):
    """Within this context (per thread) the backward entry points ask the library for at
    most `nbytes` of workspace, never less than fmlp_bwd_workspace_size_min. The library
    then runs the dZ-store mode in head groups whose dZ^T tiles fit in it (one group
    reuses the workspace after the other), or the recompute mode if fewer than
    min(H, 4) heads' tiles fit. `None` lifts the limit: the fastest mode, whose transient
    is 2*H*E*B bytes (8 GiB for 32 heads with B = 65536 and E = 2048) plus split partials,
    in groups of at most 8 GiB."""
    prev = getattr(_WS_LIMIT, "v", None)
    _WS_LIMIT.v = None if nbytes is None else max(0, int(nbytes))
    try:
        yield
    finally:
        _WS_LIMIT.v = prev


@contextlib.contextmanager
def low_memory_backward(enabled: bool = True):
    """Within this context (per thread) the backward entry points ask the library for its
    least workspace (fmlp_bwd_workspace_size_min), which selects the recompute mode: the dX
    programs recompute Z and dH rather than read the dZ^T tiles that the dW programs store
    in the dZ-store mode. It saves that transient at the cost of the recomputed products.
    Equivalent to backward_workspace_limit(0)."""
    with backward_workspace_limit(0 if enabled else getattr(_WS_LIMIT, "v", None)):
        yield


def _bwd_workspace_bytes(L, H: int, B: int, D: int, E: int, dt: int) -> int:
    key = (torch.cuda.current_device(), H, B, D, E, dt)
    full = _WS_FULL.get(key)
    if full is None:
        full = _WS_FULL[key] = int(L.fmlp_bwd_workspace_size(H, B, D, E, dt))
    lim = getattr(_WS_LIMIT, "v", None)
    if lim is None or lim >= full:
        return full
    return max(int(L.fmlp_bwd_workspace_size_min(H, B, D, E, dt)), lim)


def flashmlp_fwd(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                 activation: str = "") -> torch.Tensor:
    """Forward pass; drop-in for flashmlp.py:428-477.

    Args:
        x: (H, B, D); w1: (H, D, E); w2: (H, E, D); activation: "silu", "leaky_relu",
        "sigmoid" or "" (anything else is linear).
    Returns:
        O of shape (H, B, D), same dtype as x.
    """
    assert x.shape[0] == w1.shape[0], "Number of heads must match"
    assert x.shape[0] == w2.shape[0], "Number of heads must match"
    assert x.shape[2] == w1.shape[1], "Hidden dimension mismatch"
    assert w1.shape[2] == w2.shape[1], "Intermediate dimension mismatch"
    assert x.shape[2] == w2.shape[2], "Output dimension mismatch"

    H, B, D = x.shape
    E = w1.shape[2]

    x = x.reshape(H * B, D)
    w1 = w1.reshape(D * H, E)
    w2 = w2.reshape(E * H, D)

    assert x.is_contiguous(), "Input X must be contiguous"
    assert w1.is_contiguous(), "Weight W1 must be contiguous"
    assert w2.is_contiguous(), "Weight W2 must be contiguous"

    dev = _check_tensors(x, w1, w2)
    o = torch.empty_like(x)
    L = _lib.lib()
    with _on_device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        rc = L.fmlp_fwd(x.data_ptr(), w1.data_ptr(), w2.data_ptr(), o.data_ptr(), H, B, D, E,
                        _dtype_code(x), activation_code(activation), stream)
    _lib.check(rc, "fmlp_fwd")
    return o.reshape(H, B, D)


def flashmlp_bwd(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                 do: torch.Tensor, activation: str = "") -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Backward pass; drop-in for flashmlp.py:480-538. Recomputes Z and H from X, W1 and W2.

    Returns:
        (dx, dw1, dw2) with the shapes of (x, w1, w2).
    """
    assert x.shape[2] == w1.shape[1], "Hidden dimension mismatch"
    assert w1.shape[2] == w2.shape[1], "Intermediate dimension mismatch"
    assert x.shape[2] == w2.shape[2], "Output dimension mismatch"
    assert x.shape == do.shape, "Gradient shape mismatch"

    H, B, D = x.shape
    E = w1.shape[2]

    x = x.reshape(H * B, D)
    w1 = w1.reshape(D * H, E)
    w2 = w2.reshape(E * H, D)
    do = do.reshape(H * B, D).contiguous()

    assert x.is_contiguous(), "Input X must be contiguous"
    assert w1.is_contiguous(), "Weight W1 must be contiguous"
    assert w2.is_contiguous(), "Weight W2 must be contiguous"
    assert do.is_contiguous(), "Gradient dO must be contiguous"

    dev = _check_tensors(x, w1, w2, do)
    dx = torch.empty_like(x)
    dw1 = torch.empty_like(w1)
    dw2 = torch.empty_like(w2)
    L = _lib.lib()
    dt = _dtype_code(x)
    with _on_device(dev):
        # scratch: the dZ^T tiles of the dZ-store mode and/or the fp32 dW partial sums of
        # split dW programs
        ws_bytes = _bwd_workspace_bytes(L, H, B, D, E, dt)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes else None
        stream = torch.cuda.current_stream(dev).cuda_stream
        rc = L.fmlp_bwd(x.data_ptr(), w1.data_ptr(), w2.data_ptr(), do.data_ptr(), dx.data_ptr(),
                        dw1.data_ptr(), dw2.data_ptr(), ws.data_ptr() if ws is not None else None, ws_bytes,
                        H, B, D, E, dt, activation_code(activation), stream)
    _lib.check(rc, "fmlp_bwd")
    return dx.reshape(H, B, D), dw1.reshape(H, D, E), dw2.reshape(H, E, D)


def flashmlp_bwd_dw_f32(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, do: torch.Tensor,
                        activation: str = "", dw_out: torch.Tensor = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Backward with dW as unrounded fp32 sums over this call's rows (fmlp_bwd_dw_f32).

    Returns (dx, dw) with dx like flashmlp_bwd's and dw a flat fp32 tensor holding dW1
    (H, D, E) followed by dW2 (H, E, D); `dw_out` (2*H*D*E fp32, contiguous) is filled
    instead of a new tensor when given. Used by the batch-sharded step, whose ranks add
    their fp32 partials before any rounding."""
    assert x.shape[2] == w1.shape[1], "Hidden dimension mismatch"
    assert w1.shape[2] == w2.shape[1], "Intermediate dimension mismatch"
    assert x.shape[2] == w2.shape[2], "Output dimension mismatch"
    assert x.shape == do.shape, "Gradient shape mismatch"
    H, B, D = x.shape
    E = w1.shape[2]
    x = x.contiguous()
    w1 = w1.contiguous()
    w2 = w2.contiguous()
    do = do.contiguous()
    dev = _check_tensors(x, w1, w2, do)
    dx = torch.empty_like(x)
    n = 2 * H * D * E
    if dw_out is None:
        dw_out = torch.empty(n, dtype=torch.float32, device=dev)
    elif dw_out.dtype != torch.float32 or dw_out.numel() != n or not dw_out.is_contiguous() or dw_out.device != dev:
        raise ValueError(f"dw_out must be a contiguous float32 tensor of {n} elements on {dev}")
    L = _lib.lib()
    dt = _dtype_code(x)
    with torch.cuda.device(dev):
        ws_bytes = _bwd_workspace_bytes(L, H, B, D, E, dt)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes else None
        stream = torch.cuda.current_stream(dev).cuda_stream
        rc = L.fmlp_bwd_dw_f32(_ptr(x), _ptr(w1), _ptr(w2), _ptr(do), _ptr(dx), _ptr(dw_out),
                               _ptr(ws) if ws is not None else None, ws_bytes, H, B, D, E, dt,
                               activation_code(activation), ctypes.c_void_p(stream))
    _lib.check(rc, "fmlp_bwd_dw_f32")
    return dx, dw_out


def flashmlp_fwd_shared_x(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                          activation: str = "") -> torch.Tensor:
    """Mean over heads of the MLP of one shared input: x (B, D) -> (B, D),
    (1/H) * sum_h act(x @ w1[h]) @ w2[h] (fmlp_fwd_shared_x). Equals
    flashmlp_fwd(x.expand(H, B, D), w1, w2).mean(0) -- the reference's FlashMLP on a 2-D
    input, flashmlp.py:603-614 -- without materialising the expanded x or the per-head
    outputs; the head sum is accumulated in fp32 and rounded once. Needs D <= 128."""
    assert x.dim() == 2 and x.shape[1] == w1.shape[1], "Hidden dimension mismatch"
    assert w1.shape[0] == w2.shape[0], "Number of heads must match"
    assert w1.shape[2] == w2.shape[1], "Intermediate dimension mismatch"
    assert x.shape[1] == w2.shape[2], "Output dimension mismatch"
    H, D, E = w1.shape
    B = x.shape[0]
    x, w1, w2 = x.contiguous(), w1.contiguous(), w2.contiguous()
    dev = _check_tensors(x, w1, w2)
    o = torch.empty_like(x)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        rc = _lib.lib().fmlp_fwd_shared_x(_ptr(x), _ptr(w1), _ptr(w2), _ptr(o), H, B, D, E, _dtype_code(x),
                                          activation_code(activation), ctypes.c_void_p(stream))
    _lib.check(rc, "fmlp_fwd_shared_x")
    return o


def flashmlp_bwd_shared_x(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, do: torch.Tensor,
                          activation: str = "") -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Backward of flashmlp_fwd_shared_x (fmlp_bwd_shared_x): do (B, D) is the gradient of
    the head mean; returns dx (B, D) (summed over heads), dw1 (H, D, E), dw2 (H, E, D)."""
    assert x.dim() == 2 and x.shape == do.shape, "Gradient shape mismatch"
    assert x.shape[1] == w1.shape[1], "Hidden dimension mismatch"
    assert w1.shape[2] == w2.shape[1], "Intermediate dimension mismatch"
    H, D, E = w1.shape
    B = x.shape[0]
    x, w1, w2, do = x.contiguous(), w1.contiguous(), w2.contiguous(), do.contiguous()
    dev = _check_tensors(x, w1, w2, do)
    dx = torch.empty_like(x)
    dw1 = torch.empty_like(w1)
    dw2 = torch.empty_like(w2)
    L = _lib.lib()
    dt = _dtype_code(x)
    with torch.cuda.device(dev):
        ws_bytes = _bwd_workspace_bytes(L, H, B, D, E, dt)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes else None
        stream = torch.cuda.current_stream(dev).cuda_stream
        rc = L.fmlp_bwd_shared_x(_ptr(x), _ptr(w1), _ptr(w2), _ptr(do), _ptr(dx), _ptr(dw1), _ptr(dw2),
                                 _ptr(ws) if ws is not None else None, ws_bytes, H, B, D, E, dt,
                                 activation_code(activation), ctypes.c_void_p(stream))
    _lib.check(rc, "fmlp_bwd_shared_x")
    return dx, dw1, dw2


class FlashMLPSharedInputFunction(torch.autograd.Function):
    """Autograd for the head mean of a shared (B, D) input; saves only x, W1 and W2."""

    @staticmethod
    def forward(ctx, x, w1, w2, activation=""):
        o = flashmlp_fwd_shared_x(x, w1, w2, activation)
        ctx.save_for_backward(x, w1, w2)
        ctx.activation = activation
        return o

    @staticmethod
    def backward(ctx, do):
        x, w1, w2 = ctx.saved_tensors
        dx, dw1, dw2 = flashmlp_bwd_shared_x(x, w1, w2, do, ctx.activation)
        return dx, dw1, dw2, None


class FlashMLPFunction(torch.autograd.Function):
    """Autograd wrapper; saves only X, W1 and W2 (flashmlp.py:545-557)."""

    @staticmethod
    def forward(ctx, x, w1, w2, activation=""):
        o = flashmlp_fwd(x, w1, w2, activation)
        ctx.save_for_backward(x, w1, w2)
        ctx.activation = activation
        return o

    @staticmethod
    def backward(ctx, do):
        x, w1, w2 = ctx.saved_tensors
        dx, dw1, dw2 = flashmlp_bwd(x, w1, w2, do, ctx.activation)
        return dx, dw1, dw2, None


class FlashMLP(torch.nn.Module):
    """Multi-head MLP module (flashmlp.py:564-616).

    Parameters `w1` (H, D, E) and `w2` (H, E, D) are initialised like the reference,
    randn / sqrt(E) and randn / sqrt(D), so state dicts interchange. A 2-D input (B, D) is
    broadcast to every head and the output is averaged over heads; for 16-bit inputs with
    D <= 128 this runs on the shared-input kernels (no (H, B, D) copies of x, dO or dX; the
    head mean is accumulated in fp32), otherwise on the per-head kernels with the expanded
    input, as in the reference (flashmlp.py:603-614). float32 parameters run on the TF32
    kernels (D <= 128).
    """

    def __init__(self, num_heads: int, hidden_dim: int, intermediate_dim: int,
                 activation: str = "silu", dtype=torch.float16, device="cuda"):
        super().__init__()
        self.num_heads = num_heads
        self.hidden_dim = hidden_dim
        self.intermediate_dim = intermediate_dim
        self.activation = activation
        self.w1 = torch.nn.Parameter(
            torch.randn(num_heads, hidden_dim, intermediate_dim, dtype=dtype, device=device)
            / np.sqrt(intermediate_dim)
        )
        self.w2 = torch.nn.Parameter(
            torch.randn(num_heads, intermediate_dim, hidden_dim, dtype=dtype, device=device)
            / np.sqrt(hidden_dim)
        )

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        squeeze_output = x.dim() == 2
        if squeeze_output and x.shape[-1] <= 128 and self.num_heads > 0 and x.dtype != torch.float32:
            return FlashMLPSharedInputFunction.apply(x, self.w1, self.w2, self.activation)
        if squeeze_output:
            x = x.unsqueeze(0).expand(self.num_heads, -1, -1)
        o = FlashMLPFunction.apply(x, self.w1, self.w2, self.activation)
        if squeeze_output:
            o = o.mean(dim=0)
        return o
