"""FP8 (e4m3) forward of the fused multi-head MLP (fmlp_fwd_fp8 in the C ABI).

Not part of the reference, whose kernels run in fp16, bf16 and fp32; this is the same
forward, O = act(X W1) W2 per head, with 8-bit operands on the B200's kind::f8f6f4 tensor
cores and per-tensor scales, the usual FP8 inference recipe:

    Z  = (X8 @ W1_8) * x_scale * w1_scale          fp32 accumulation
    H8 = e4m3(act(Z) / h_scale)                    round to nearest even, saturating at 448
    O  = (H8 @ W2_8) * h_scale * w2_scale          rounded once to bf16 or fp16

The kernel takes the weights transposed (W1^T (H, E, D), W2^T (H, D, E)) so that every
shared-memory operand is K-major; `prepare_fp8_weights` quantizes reference-layout
weights and transposes them once. Forward only: there is no FP8 backward.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from .api import _ptr, activation_code

E4M3_MAX = 448.0


def quantize_e4m3(t: torch.Tensor, scale: float | None = None):
    """(t8, scale) with t ~= scale * t8.float(): per-tensor scale amax / 448 unless given
    (1.0 for an all-zero tensor), values saturated to +-448 before the cast."""
    if scale is None:
        amax = float(t.detach().abs().max()) if t.numel() else 0.0
        scale = amax / E4M3_MAX if amax > 0 else 1.0
    t8 = (t.detach().float() / scale).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return t8, float(scale)


@dataclass
class Fp8Weights:
    w1t: torch.Tensor  # (H, E, D) float8_e4m3fn, W1^T
    w2t: torch.Tensor  # (H, D, E) float8_e4m3fn, W2^T
    w1_scale: float
    w2_scale: float


def prepare_fp8_weights(w1: torch.Tensor, w2: torch.Tensor, w1_scale: float | None = None,
                        w2_scale: float | None = None) -> Fp8Weights:
    """Quantize reference-layout weights w1 (H, D, E), w2 (H, E, D) to e4m3 and store them
    transposed for fmlp_fwd_fp8."""
    assert w1.dim() == 3 and w2.dim() == 3, "weights are (H, D, E) and (H, E, D)"
    assert w1.shape[0] == w2.shape[0], "Number of heads must match"
    assert w1.shape[2] == w2.shape[1], "Intermediate dimension mismatch"
    assert w1.shape[1] == w2.shape[2], "Output dimension mismatch"
    w1q, s1 = quantize_e4m3(w1, w1_scale)
    w2q, s2 = quantize_e4m3(w2, w2_scale)
    return Fp8Weights(w1q.transpose(1, 2).contiguous(), w2q.transpose(1, 2).contiguous(), s1, s2)


def flashmlp_fwd_fp8(x8: torch.Tensor, weights: Fp8Weights, activation: str = "", x_scale: float = 1.0,
                     h_scale: float = 1.0, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """FP8 forward: x8 (H, B, D) float8_e4m3fn with x ~= x_scale * x8; returns O (H, B, D)
    in out_dtype (torch.bfloat16 or torch.float16). h_scale sets the e4m3 range of the
    activations (H8 = act(Z) / h_scale); pick it so that max |act(Z)| / h_scale stays near
    448. Needs D % 16 == 0, D <= 128, E % 16 == 0."""
    w1t, w2t = weights.w1t, weights.w2t
    assert x8.dim() == 3 and w1t.dim() == 3 and w2t.dim() == 3, "x8 (H,B,D), w1t (H,E,D), w2t (H,D,E)"
    H, B, D = x8.shape
    E = w1t.shape[1]
    assert w1t.shape == (H, E, D), "w1t must be W1^T of shape (H, E, D)"
    assert w2t.shape == (H, D, E), "w2t must be W2^T of shape (H, D, E)"
    for t in (x8, w1t, w2t):
        if t.dtype != torch.float8_e4m3fn:
            raise TypeError(f"fmlp_fwd_fp8 takes torch.float8_e4m3fn tensors, got {t.dtype}")
        if t.device.type != "cuda" or t.device != x8.device:
            raise RuntimeError("fmlp_fwd_fp8 needs all tensors on one CUDA device (there is no CPU path)")
    if out_dtype == torch.bfloat16:
        oc = _lib.FMLP_DTYPE_BF16
    elif out_dtype == torch.float16:
        oc = _lib.FMLP_DTYPE_F16
    else:
        raise TypeError(f"out_dtype must be torch.bfloat16 or torch.float16, got {out_dtype}")
    x8, w1t, w2t = x8.contiguous(), w1t.contiguous(), w2t.contiguous()
    dev = x8.device
    o = torch.empty((H, B, D), dtype=out_dtype, device=dev)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        rc = _lib.lib().fmlp_fwd_fp8(_ptr(x8), _ptr(w1t), _ptr(w2t), _ptr(o), H, B, D, E, float(x_scale),
                                     float(weights.w1_scale), float(weights.w2_scale), float(h_scale),
                                     activation_code(activation), oc, ctypes.c_void_p(stream))
    _lib.check(rc, "fmlp_fwd_fp8")
    return o
