"""The parity check itself (tests/_refcheck.py) must catch the bugs it is there for.

At the statistics of BASELINE config 4 (bf16 silu, B = 65536 rows, D = 128; a 256-column
slice of E keeps it quick on the CPU), a result that is the fp32 reference rounded once to
bf16 (what an exact kernel returns) must pass; a uniform 2 % error, and a dW sum that
dropped one 128-row B tile, must fail. The elementwise bound alone lets both through
at this K (its kappa term grows with the 65536-term sums); the norm-wise bound does not.
"""
import pytest
import torch

from _refcheck import KAPPA, assert_close, norm_rel_errors, ref_bwd, tol_for


@pytest.fixture(scope="module")
def c4_slice():
    H, B, D, E = 1, 65536, 128, 256
    g = torch.Generator().manual_seed(5)
    dt = torch.bfloat16
    x = torch.randn(H, B, D, generator=g).to(dt)
    w1 = (torch.randn(H, D, E, generator=g) / D ** 0.5).to(dt)
    w2 = (torch.randn(H, E, D, generator=g) / 2048 ** 0.5).to(dt)  # C4's E = 2048 scale
    do = torch.randn(H, B, D, generator=g).to(dt)
    refs = ref_bwd(x, w1, w2, do, "silu")
    return x, w1, w2, do, refs


def _elementwise_ok(a, ref, bound, dtype):
    atol, rtol = tol_for(dtype, "bwd")
    return bool(((a.float() - ref).abs() <= atol + rtol * ref.abs() + KAPPA * bound).all())


def test_exact_result_rounded_to_bf16_passes(c4_slice):
    *_, refs = c4_slice
    for k in ("dx", "dw1", "dw2"):
        ref, bound = refs[k]
        assert_close(ref.to(torch.bfloat16), ref, bound, torch.bfloat16, "bwd", k)
        rel = norm_rel_errors(ref.to(torch.bfloat16), ref)
        assert max(rel) < 2.5e-3, f"{k}: bf16 rounding alone gives {rel}"


@pytest.mark.parametrize("k", ["dx", "dw1", "dw2"])
def test_uniform_two_percent_error_fails(c4_slice, k):
    *_, refs = c4_slice
    ref, bound = refs[k]
    bad = (ref * 1.02).to(torch.bfloat16)
    if k == "dw1":
        assert _elementwise_ok(bad, ref, bound, torch.bfloat16), "the elementwise bound alone passes it"
    with pytest.raises(AssertionError, match="norm-wise"):
        assert_close(bad, ref, bound, torch.bfloat16, "bwd", k)


@pytest.mark.parametrize("k", ["dw1", "dw2"])
def test_dropped_b_tile_fails(c4_slice, k):
    x, w1, w2, do, refs = c4_slice
    ref, bound = refs[k]
    # the contribution of rows 0..127 to the sum over B, from the same rounded operands
    part = ref_bwd(x[:, :128], w1, w2, do[:, :128], "silu")[k][0]
    bad = (ref - part).to(torch.bfloat16)
    with pytest.raises(AssertionError):
        assert_close(bad, ref, bound, torch.bfloat16, "bwd", k)
    assert max(norm_rel_errors(bad, ref)) > 2e-2
