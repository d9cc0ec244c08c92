"""Parity with the reference's own Triton kernels, run unmodified on the B200.

The reference module (dtadpole/flashMLP flashmlp.py, installed unmodified into the
git-ignored baseline/_ref/) is loaded by file path and its public wrappers flashmlp_fwd /
flashmlp_bwd (flashmlp.py:428-538, over flashmlp_fwd_kernel :63-158 and
flashmlp_bwd_kernel :341-421, autotuned on first use) run on the same seeded inputs as
this library's kernels. Cases: BASELINE configs C1 (fp16 silu) and C2 (bf16 leaky_relu)
in full, a 4-head slice of C4 (bf16 silu) and a 2-head slice of C5 (fp16 sigmoid). Only
shapes the reference handles correctly are used: D a power of two, B a multiple of 128,
E a multiple of 64. For other shapes (e.g. C3) its forward reads and writes past its
block-pointer extents, so it is never run on them.

Checked, per output, at the README tolerance (atol = rtol = 1e-2 forward / 3e-2 backward
for bf16, 5e-3 / 1e-2 for fp16) plus the dot-product bound and the norm-wise bound of
tests/_refcheck.py:
  * this library against the fp32 PyTorch reference with the kernels' rounding points;
  * this library against the reference's Triton outputs directly.
The Triton outputs' own norm-wise errors against the fp32 reference, and those of a plain
cuBLAS 16-bit chain (torch.bmm in the input dtype), are recorded for the session report.
"""
import pytest
import torch

from _refcheck import INFO, _act, assert_close, check_norm, make_inputs, norm_rel_errors, ref_bwd, ref_fwd

pytestmark = pytest.mark.gpu

CASES = [
    ("C1", (12, 1024, 64, 768), torch.float16, "silu"),
    ("C2", (16, 16384, 128, 512), torch.bfloat16, "leaky_relu"),
    ("C4/4 heads", (4, 65536, 128, 2048), torch.bfloat16, "silu"),
    ("C5/2 heads", (2, 131072, 256, 1024), torch.float16, "sigmoid"),
]


@pytest.fixture(scope="module")
def reference():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from oracle.reference_loader import REF_PATH, load_reference

    mod = load_reference()
    if mod is None:
        pytest.skip(f"the reference is not installed at {REF_PATH}")
    return mod


def _cublas_chain(x, w1, w2, do, act):
    """The same math as plain 16-bit torch.bmm calls (cuBLAS, fp32 accumulation, output
    rounded per GEMM), with the reference's formulas (flashmlp.py:671-723)."""
    z = torch.bmm(x, w1)
    h = _act(z.float(), act).to(x.dtype)
    o = torch.bmm(h, w2)
    dh = torch.bmm(do, w2.transpose(1, 2)).float()
    zf = z.float()
    if act == "leaky_relu":
        dz = dh * torch.where(zf >= 0, 1.0, 0.01)
    elif act == "silu":
        s = torch.sigmoid(zf)
        dz = dh * (s + zf * s * (1 - s))
    elif act == "sigmoid":
        s = h.float()
        dz = dh * s * (1 - s)
    else:
        dz = dh
    dz = dz.to(x.dtype)
    return o, torch.bmm(dz, w1.transpose(1, 2)), torch.bmm(x.transpose(1, 2), dz), torch.bmm(h.transpose(1, 2), do)


@pytest.mark.parametrize("name,shape,dt,act", CASES, ids=[c[0] for c in CASES])
def test_matches_reference_triton_kernels(reference, name, shape, dt, act):
    import flashmlp_b200 as F

    H, B, D, E = shape
    x, w1, w2, do = make_inputs(H, B, D, E, dt, seed=11)
    o_t = reference.flashmlp_fwd(x, w1, w2, act)
    dx_t, dw1_t, dw2_t = reference.flashmlp_bwd(x, w1, w2, do, act)
    o = F.flashmlp_fwd(x, w1, w2, act)
    dx, dw1, dw2 = F.flashmlp_bwd(x, w1, w2, do, act)
    cub = _cublas_chain(x, w1, w2, do, act)
    torch.cuda.synchronize()
    for t in (o_t, dx_t, dw1_t, dw2_t):
        assert t.dtype == dt and torch.isfinite(t.float()).all()

    r_o, b_o = ref_fwd(x, w1, w2, act)
    refs = ref_bwd(x, w1, w2, do, act)
    assert_close(o, r_o, b_o, dt, "fwd", f"{name}/o vs fp32")
    assert_close(o, o_t.float(), b_o, dt, "fwd", f"{name}/o vs triton")
    rows = [("o", o, o_t, r_o, cub[0])]
    for k, got, tri, cb in (("dx", dx, dx_t, cub[1]), ("dw1", dw1, dw1_t, cub[2]), ("dw2", dw2, dw2_t, cub[3])):
        ref, bound = refs[k]
        assert_close(got, ref, bound, dt, "bwd", f"{name}/{k} vs fp32")
        assert_close(got, tri.float(), bound, dt, "bwd", f"{name}/{k} vs triton")
        rows.append((k, got, tri, ref, cb))
    for k, got, tri, ref, cb in rows:
        ours, theirs, blas = (max(norm_rel_errors(t, ref)) for t in (got, tri, cb))
        INFO.append(f"triton parity {name} {str(dt)[6:]} {act} {k}: ||.-r||/||r|| ours {ours:.2e}, "
                    f"reference triton {theirs:.2e}, cuBLAS 16-bit chain {blas:.2e}, "
                    f"ours vs triton {max(norm_rel_errors(got, tri.float())):.2e}")
    # the Triton result meets the same norm-wise bar (it is the reference; a miss here
    # would be a finding about the bar, so it is checked, not only reported)
    check_norm(o_t, r_o, dt, "fwd", f"{name}/triton o")
    for k, tri in (("dx", dx_t), ("dw1", dw1_t), ("dw2", dw2_t)):
        check_norm(tri, refs[k][0], dt, "bwd", f"{name}/triton {k}")
