"""Shared helpers of the GPU parity tests: input generation, a plain-PyTorch fp32 reference
with the kernels' rounding points (run on the GPU for large shapes), and the tolerance.

Tolerance for an output a against a reference r of a contraction sum_k p_k q_k:

    |a - r| <= atol + rtol * |r| + kappa * sum_k |p_k| |q_k|  (+ leaky-relu term)

atol/rtol are the reference's README tolerances (fwd 1e-2, bwd 3e-2 for bf16; tighter
for fp16). The kappa term is the standard floating-point bound for a long dot product:
it covers fp32 accumulation order over K = B = 65536 rows and one-step flips of the
16-bit rounded intermediates H and dZ. leaky_relu's derivative jumps at z = 0, so an
element whose |z| is within the fp32 accumulation error may legitimately take the other
branch; its possible contribution 0.99 |dh| |w| is added for those elements only.
"""
from __future__ import annotations

import numpy as np
import torch

KAPPA = 2.0 ** -10
Z_AMBIGUOUS = 1e-3


def tol_for(dtype: torch.dtype, kind: str):
    """bf16: the README's 1e-2 / 3e-2; fp16 and fp32 inputs (TF32 products, the same
    10-bit mantissa as fp16 for the operands): 5e-3 / 1e-2."""
    if dtype == torch.bfloat16:
        return (1e-2, 1e-2) if kind == "fwd" else (3e-2, 3e-2)
    return (5e-3, 5e-3) if kind == "fwd" else (1e-2, 1e-2)


def make_inputs(H, B, D, E, dtype, seed=0, device="cuda"):
    """X ~ N(0,1), W1 ~ N(0,1/D), W2 ~ N(0,1/E), dO ~ N(0,1), generated in fp32 from a
    seeded CPU generator, then rounded to `dtype`."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(H, B, D, generator=g)
    w1 = torch.randn(H, D, E, generator=g) / D ** 0.5
    w2 = torch.randn(H, E, D, generator=g) / E ** 0.5
    do = torch.randn(H, B, D, generator=g)
    return [t.to(dtype).to(device) for t in (x, w1, w2, do)]


def _act(z, a):
    if a == "leaky_relu":
        return torch.where(z >= 0, z, 0.01 * z)
    if a == "silu":
        return z * torch.sigmoid(z)
    if a == "sigmoid":
        return torch.sigmoid(z)
    return z


def ref_fwd(x, w1, w2, a):
    """Returns (o_ref fp32, o_bound) with the kernel's rounding of H."""
    dt = x.dtype
    z = torch.bmm(x.float(), w1.float())
    h = _act(z, a).to(dt).float()
    w2f = w2.float()
    return torch.bmm(h, w2f), torch.bmm(h.abs(), w2f.abs())


def ref_bwd(x, w1, w2, do, a):
    """Returns dict name -> (ref fp32, bound) for dx, dw1, dw2."""
    dt = x.dtype
    xf, w1f, w2f, dof = x.float(), w1.float(), w2.float(), do.float()
    z = torch.bmm(xf, w1f)
    h = _act(z, a).to(dt).float()
    dh = torch.bmm(dof, w2f.transpose(1, 2))
    if a == "leaky_relu":
        dz = dh * torch.where(z >= 0, 1.0, 0.01)
    elif a == "silu":
        s = torch.sigmoid(z)
        dz = dh * (s + h * (1 - s))
    elif a == "sigmoid":
        dz = (dh * h) * (1 - h).to(dt).float()
    else:
        dz = dh
    dz = dz.to(dt).float()
    out = {
        "dx": [torch.bmm(dz, w1f.transpose(1, 2)), torch.bmm(dz.abs(), w1f.abs().transpose(1, 2))],
        "dw1": [torch.bmm(xf.transpose(1, 2), dz), torch.bmm(xf.abs().transpose(1, 2), dz.abs())],
        "dw2": [torch.bmm(h.transpose(1, 2), dof), torch.bmm(h.abs().transpose(1, 2), dof.abs())],
    }
    if a == "leaky_relu":
        # |z| within its own error of 0 may take either branch: fp32 accumulation error for
        # 16-bit operands; for fp32 inputs the products use TF32 operands, so z's error is
        # up to the dot-product bound KAPPA * sum |x| |w1|
        win = Z_AMBIGUOUS
        if dt == torch.float32:
            win = win + KAPPA * torch.bmm(xf.abs(), w1f.abs())
        amb = (z.abs() < win).float() * dh.abs() * 0.99
        out["dx"][1] = out["dx"][1] + torch.bmm(amb, w1f.abs().transpose(1, 2)) / KAPPA
        out["dw1"][1] = out["dw1"][1] + torch.bmm(xf.abs().transpose(1, 2), amb) / KAPPA
    return {k: tuple(v) for k, v in out.items()}


def assert_close(a: torch.Tensor, ref: torch.Tensor, bound: torch.Tensor, dtype, kind, name=""):
    atol, rtol = tol_for(dtype, kind)
    a = a.float()
    assert torch.isfinite(a).all(), f"{name}: non-finite values"
    err = (a - ref).abs()
    tol = atol + rtol * ref.abs() + KAPPA * bound
    bad = err > tol
    if bad.any():
        i = torch.argmax(err - tol)
        raise AssertionError(
            f"{name}: {int(bad.sum())} of {err.numel()} elements out of tolerance; worst "
            f"got {a.flatten()[i].item():.6g} want {ref.flatten()[i].item():.6g} "
            f"(err {err.flatten()[i].item():.3g}, tol {tol.flatten()[i].item():.3g})")


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()
