"""Pins the CPU oracle against fixtures produced by the reference itself (CPU only).

* oracle.fwd_fp32 / bwd_fp32 vs the reference's PyTorch path (flashmlp_torch_fwd/bwd in
  fp32, flashmlp.py:671-723): same math, only BLAS summation order differs.
* oracle.fwd_kernel / bwd_kernel vs the reference's Triton kernels run under the Triton
  CPU interpreter in fp16 (flashmlp.py:63-158, :341-421): same rounding points; the
  kernels sum in E/B chunks, so a rounded output may differ by one fp16 step.
"""
import numpy as np
import pytest

from conftest import load_golden, GOLDEN_CASES
from oracle import flashmlp_oracle as orc


def _close_fp32(a, ref):
    scale = np.abs(ref).max() + 1e-30
    return np.abs(a - ref).max() / scale


def _ulp16(ref):
    return np.spacing(np.abs(ref).astype(np.float16)).astype(np.float32)


def _assert_kernel_match(a, ref, name):
    """Rounded-output agreement: within one fp16 step of the element plus a 2e-4 slack
    relative to the tensor's largest value (fp32 summation order), >= 99% bit-exact."""
    err = np.abs(a - ref)
    tol = _ulp16(ref) + 2e-4 * np.abs(ref).max()
    assert (err <= tol).all(), f"{name}: max err {err.max()} (tol at worst {tol[np.argmax(err - tol)]})"
    assert (err == 0).mean() >= 0.99, f"{name}: only {(err == 0).mean():.4f} bit-exact"


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_oracle_matches_reference_torch_fp32(golden, case):
    g = golden[case]
    for act in g["acts"]:
        tag = act or "linear"
        o = orc.fwd_fp32(g["x"], g["w1"], g["w2"], act)
        dx, dw1, dw2 = orc.bwd_fp32(g["x"], g["w1"], g["w2"], g["do"], act)
        assert _close_fp32(o, g[f"torch_o_{tag}"]) < 1e-5, (case, tag, "o")
        assert _close_fp32(dx, g[f"torch_dx_{tag}"]) < 1e-5, (case, tag, "dx")
        assert _close_fp32(dw1, g[f"torch_dw1_{tag}"]) < 1e-5, (case, tag, "dw1")
        assert _close_fp32(dw2, g[f"torch_dw2_{tag}"]) < 1e-5, (case, tag, "dw2")


@pytest.mark.parametrize("case", [c for c in GOLDEN_CASES if c.startswith("f16")])
def test_oracle_matches_reference_triton_kernels(golden, case):
    g = golden[case]
    checked = 0
    for act in g["acts"]:
        tag = act or "linear"
        if f"triton_o_{tag}" in g:
            o = orc.fwd_kernel(g["x"], g["w1"], g["w2"], act, "f16")
            _assert_kernel_match(o, g[f"triton_o_{tag}"], f"{case}/{tag}/o")
            checked += 1
        if f"triton_dx_{tag}" in g:
            dx, dw1, dw2 = orc.bwd_kernel(g["x"], g["w1"], g["w2"], g["do"], act, "f16")
            _assert_kernel_match(dx, g[f"triton_dx_{tag}"], f"{case}/{tag}/dx")
            _assert_kernel_match(dw1, g[f"triton_dw1_{tag}"], f"{case}/{tag}/dw1")
            _assert_kernel_match(dw2, g[f"triton_dw2_{tag}"], f"{case}/{tag}/dw2")
            checked += 1
    assert checked > 0


def test_oracle_matches_reference_triton_kernels_fp32():
    # float32 case: the reference's Triton kernels under the interpreter evaluate tl.dot in
    # full fp32 and round nothing between the products; so does the oracle's "f32" path
    g = load_golden("f32_main")
    for act in g["acts"]:
        tag = act or "linear"
        o = orc.fwd_kernel(g["x"], g["w1"], g["w2"], act, "f32")
        np.testing.assert_allclose(o, g[f"triton_o_{tag}"], rtol=1e-5, atol=1e-5, err_msg=f"{tag}/o")
        got = orc.bwd_kernel(g["x"], g["w1"], g["w2"], g["do"], act, "f32")
        for name, a in zip(("dx", "dw1", "dw2"), got):
            np.testing.assert_allclose(a, g[f"triton_{name}_{tag}"], rtol=1e-5, atol=1e-5, err_msg=f"{tag}/{name}")


def test_bf16_rounding_is_round_to_nearest_even():
    # 1 + 2^-8 is a tie between 1 and 1 + 2^-7: even mantissa (1.0) wins.
    x = np.array([1.0 + 2.0 ** -8, 1.0 + 3 * 2.0 ** -8, -2.5, 3.0e38, 1e-40], dtype=np.float32)
    r = orc.round_bf16(x)
    assert r[0] == 1.0
    assert r[1] == np.float32(1.0 + 2 * 2.0 ** -7)
    assert r[2] == -2.5
    assert np.isfinite(r[3]) or np.isinf(r[3])
    assert np.array_equal(orc.bf16_from_bits(orc.bf16_bits(x)), r)


def test_fp16_rounding_matches_numpy():
    x = np.linspace(-3, 3, 1001, dtype=np.float32)
    assert np.array_equal(orc.round_f16(x), x.astype(np.float16).astype(np.float32))


def test_unknown_activation_is_linear():
    x, w1, w2, do = orc.make_inputs(1, 8, 16, 16, "f16", seed=3)
    assert np.array_equal(orc.fwd_kernel(x, w1, w2, "gelu", "f16"), orc.fwd_kernel(x, w1, w2, "", "f16"))


def test_make_inputs_distribution():
    x, w1, w2, do = orc.make_inputs(2, 4096, 64, 256, "bf16", seed=0)
    assert abs(x.std() - 1.0) < 0.02
    assert abs(w1.std() - 1.0 / 8.0) < 0.005
    assert abs(w2.std() - 1.0 / 16.0) < 0.003
