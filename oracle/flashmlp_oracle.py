"""CPU oracle for the fused multi-head MLP — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this
module, and only as the checker (or as the timed CPU baseline); the product path
(flashmlp_b200) never does.

It restates, in numpy float32, the algorithm of dtadpole/flashMLP (flashmlp.py):

  * `fwd_kernel` / `bwd_kernel` follow the Triton kernels' rounding points:
      Z = X @ W1 in fp32 (flashmlp.py:137, :212, :294)
      H = act(Z) rounded to the input dtype (flashmlp.py:140-147, :214-221, :296-303)
      dH = dO @ W2^T in fp32 (flashmlp.py:224, :306)
      dZ = dH * act'(Z) rounded to the input dtype, with act' using the rounded H for
           silu and sigmoid (flashmlp.py:43-46, :227-235, :312-320); for sigmoid,
           (1 - sig) is itself a 16-bit value (sig is the 16-bit H, flashmlp.py:232-233)
      O, dX, dW1, dW2 accumulate in fp32 and are rounded once (flashmlp.py:150-158, :238,
           :309, :323, :393, :420-421)
  * `fwd_fp32` / `bwd_fp32` follow the reference's PyTorch path `flashmlp_torch_fwd` /
    `flashmlp_torch_bwd` (flashmlp.py:671-723) evaluated in fp32, with no intermediate
    rounding.

Inputs are float32 arrays whose values are already representable in the 16-bit dtype
(use round_to(x, dtype) first). Heads are independent, so large cases may be sliced by
head. Parity of this oracle is pinned against fixtures generated from the reference
itself (tests/golden/make_golden.py: the reference's PyTorch functions in fp32 and its
Triton kernels under the Triton CPU interpreter in fp16).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def round_bf16(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16, returned as float32."""
    a = np.ascontiguousarray(a, dtype=F32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = r.view(F32)
    return np.where(np.isnan(a), a, out).astype(F32)


def round_f16(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> float16, returned as float32."""
    return np.asarray(a, dtype=F32).astype(np.float16).astype(F32)


def round_to(a: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return round_bf16(a)
    if dtype == "f16":
        return round_f16(a)
    if dtype == "f32":
        return np.asarray(a, dtype=F32)
    raise ValueError(dtype)


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """float32 holding bf16 values -> uint16 bit patterns (for compact fixtures)."""
    return (np.ascontiguousarray(round_bf16(a)).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(F32)


def sigmoid(z: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        return (F32(1.0) / (F32(1.0) + np.exp(-z, dtype=F32))).astype(F32)


def activate(z: np.ndarray, activation: str) -> np.ndarray:
    """flashmlp.py:27-46 and the inline sigmoid at :145; unknown names are linear."""
    if activation == "leaky_relu":
        return np.where(z >= 0, z, F32(0.01) * z).astype(F32)
    if activation == "silu":
        return (z * sigmoid(z)).astype(F32)
    if activation == "sigmoid":
        return sigmoid(z)
    return z.astype(F32)


def _t(a: np.ndarray) -> np.ndarray:
    return np.swapaxes(a, -1, -2)


def fwd_kernel(x, w1, w2, activation: str, dtype: str) -> np.ndarray:
    """O as the fused forward kernel computes it (flashmlp.py:132-158)."""
    z = np.matmul(x, w1, dtype=F32)
    h = round_to(activate(z, activation), dtype)
    return round_to(np.matmul(h, w2, dtype=F32), dtype)


def dz_kernel(z, h, dh, activation: str, dtype: str) -> np.ndarray:
    """dZ rounded to the input dtype (flashmlp.py:227-235, :312-320); h is the rounded H."""
    if activation == "leaky_relu":
        dz = dh * np.where(z >= 0, F32(1.0), F32(0.01))
    elif activation == "silu":
        s = sigmoid(z)
        dz = dh * (s + h * (F32(1.0) - s))
    elif activation == "sigmoid":
        dz = (dh * h) * round_to(F32(1.0) - h, dtype)
    else:
        dz = dh
    return round_to(dz.astype(F32), dtype)


def bwd_kernel(x, w1, w2, do, activation: str, dtype: str):
    """(dX, dW1, dW2) as the unified backward kernel computes them (flashmlp.py:165-421)."""
    z = np.matmul(x, w1, dtype=F32)
    h = round_to(activate(z, activation), dtype)
    dh = np.matmul(do, _t(w2), dtype=F32)
    dz = dz_kernel(z, h, dh, activation, dtype)
    dx = round_to(np.matmul(dz, _t(w1), dtype=F32), dtype)
    dw1 = round_to(np.matmul(_t(x), dz, dtype=F32), dtype)
    dw2 = round_to(np.matmul(_t(h), do, dtype=F32), dtype)
    return dx, dw1, dw2


def fwd_fp32(x, w1, w2, activation: str) -> np.ndarray:
    """flashmlp_torch_fwd (flashmlp.py:671-686) in fp32."""
    return np.matmul(activate(np.matmul(x, w1, dtype=F32), activation), w2, dtype=F32)


def bwd_fp32(x, w1, w2, do, activation: str):
    """flashmlp_torch_bwd (flashmlp.py:689-723) in fp32, forward recomputed."""
    z = np.matmul(x, w1, dtype=F32)
    h = activate(z, activation)
    dh = np.matmul(do, _t(w2), dtype=F32)
    dw2 = np.matmul(_t(h), do, dtype=F32)
    if activation == "leaky_relu":
        dz = dh * np.where(z >= 0, F32(1.0), F32(0.01))
    elif activation == "silu":
        s = sigmoid(z)
        dz = dh * (s + z * s * (F32(1.0) - s))
    elif activation == "sigmoid":
        dz = dh * h * (F32(1.0) - h)
    else:
        dz = dh
    dz = dz.astype(F32)
    dx = np.matmul(dz, _t(w1), dtype=F32)
    dw1 = np.matmul(_t(x), dz, dtype=F32)
    return dx, dw1, dw2


def make_inputs(H: int, B: int, D: int, E: int, dtype: str, seed: int = 0):
    """Seeded inputs with the measurement distributions: X ~ N(0,1), W1 ~ N(0,1/D),
    W2 ~ N(0,1/E), dO ~ N(0,1); values rounded to `dtype`, returned as float32."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((H, B, D), dtype=F32)
    w1 = rng.standard_normal((H, D, E), dtype=F32) / F32(np.sqrt(D))
    w2 = rng.standard_normal((H, E, D), dtype=F32) / F32(np.sqrt(E))
    do = rng.standard_normal((H, B, D), dtype=F32)
    return tuple(round_to(a.astype(F32), dtype) for a in (x, w1, w2, do))
