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

The elementwise bound is loose where K is large: at K = B = 65536 its kappa term is about
a quarter of a typical |dW| element, so a uniform few-percent error, or one dropped
128-row B tile, could pass it. Every check therefore also applies a norm-wise bound per
head slice (dim 0 of a 3-D tensor, the whole tensor otherwise):

    ||a - r||_F <= c * ||r||_F  (+ ||slack||_F for leaky_relu with fp32 inputs)

with c = 5e-3 (bf16), 2e-3 (fp16), 3e-3 (fp32 inputs, TF32 products). The floor any
16-bit result with fp32 accumulation has is its final rounding: about 1.5e-3 (bf16) and
2e-4 (fp16) of ||r||_F for these value distributions (cuBLAS bf16 batched GEMMs on the
same inputs measure that floor, tests/test_triton_reference_gpu.py). The constants are
3x and 10x it. A uniform 2 % error, or one dropped 128-row B tile of a dW sum over
65536 rows (about 4.4 %), fails it (tests/test_refcheck_cpu.py). Slices with fewer than
NORM_MIN_ELEMS elements are checked elementwise only: a norm over a handful of elements
says nothing more than the elements do.
"""
from __future__ import annotations

import numpy as np
import torch

KAPPA = 2.0 ** -10
Z_AMBIGUOUS = 1e-3
NORM_C = {torch.bfloat16: 5e-3, torch.float16: 2e-3, torch.float32: 3e-3}
NORM_MIN_ELEMS = 4096
# largest norm-wise relative error seen per (dtype, kind) in this process; reported at the
# end of a pytest session (tests/conftest.py)
NORM_SEEN: dict = {}
# free-form measurements the tests record for the same end-of-session report
INFO: list = []


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
        amb_dx = torch.bmm(amb, w1f.abs().transpose(1, 2))
        amb_dw1 = torch.bmm(xf.abs().transpose(1, 2), amb)
        out["dx"][1] = out["dx"][1] + amb_dx / KAPPA
        out["dw1"][1] = out["dw1"][1] + amb_dw1 / KAPPA
        if dt == torch.float32:
            # TF32 products put about 2e-4 of the z values on the other side of 0, enough
            # to move the norm of dX and dW1 by ~1e-2: the norm-wise check allows exactly
            # those elements' possible contribution (16-bit inputs: fp32 accumulation
            # error flips a negligible fraction, so no allowance)
            out["dx"][1].fmlp_slack = amb_dx
            out["dw1"][1].fmlp_slack = amb_dw1
    return {k: tuple(v) for k, v in out.items()}


def norm_rel_errors(a: torch.Tensor, ref: torch.Tensor, slack=None):
    """Per head slice (dim 0 of a 3-D tensor, else the whole tensor): (||a - r||_F -
    ||slack||_F) / ||r||_F, for slices with at least NORM_MIN_ELEMS elements."""
    a, ref = a.float(), ref.float()
    if a.dim() != 3:
        a, ref = a.reshape(1, -1), ref.reshape(1, -1)
        slack = None if slack is None else slack.reshape(1, -1)
    else:
        a, ref = a.reshape(a.shape[0], -1), ref.reshape(ref.shape[0], -1)
        slack = None if slack is None else slack.reshape(slack.shape[0], -1)
    if a.shape[1] < NORM_MIN_ELEMS:
        return []
    num = torch.linalg.vector_norm(a - ref, dim=1)
    if slack is not None:
        num = (num - torch.linalg.vector_norm(slack, dim=1)).clamp_min(0)
    den = torch.linalg.vector_norm(ref, dim=1)
    return [float(n / d) if d > 0 else (0.0 if n == 0 else float("inf")) for n, d in zip(num, den)]


def check_norm(a: torch.Tensor, ref: torch.Tensor, dtype, kind="bwd", name="", slack=None):
    c = NORM_C[dtype]
    rel = norm_rel_errors(a, ref, slack)
    if not rel:
        return None
    worst = max(rel)
    if worst <= c:
        key = (str(dtype).replace("torch.", ""), kind)
        NORM_SEEN[key] = max(NORM_SEEN.get(key, 0.0), worst)
    else:
        raise AssertionError(
            f"{name}: norm-wise relative error {worst:.3g} exceeds {c:g} in head slice "
            f"{rel.index(worst)} (||a - r||_F / ||r||_F per slice: "
            f"{', '.join(f'{v:.2e}' for v in rel[:8])}{' ...' if len(rel) > 8 else ''})")
    return worst


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
    check_norm(a, ref, dtype, kind, name, getattr(bound, "fmlp_slack", None))


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()
