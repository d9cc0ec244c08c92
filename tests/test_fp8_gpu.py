"""FP8 (e4m3) forward (fmlp_fwd_fp8) against an fp32 PyTorch reference of the same
quantized computation: Z from the dequantized e4m3 operands (their products are exact in
fp32), act(Z) / h_scale rounded to e4m3 by torch's cast (saturated at 448 first), O from
that and W2. The kernel's sigmoid/silu use the SFU tanh (relative error about 5e-4) on
seven of every eight column pairs and a polynomial exp2 with a Newton reciprocal on the
FMA pipe (relative error about 1e-4) on the eighth; either moves a small fraction of the
e4m3 roundings of H by one step. The bounds below cover that and the bf16/fp16 output
rounding. The reference has no FP8 path, so there is no golden.
"""
import pytest
import torch

import flashmlp_b200 as F
from flashmlp_b200 import _lib

pytestmark = pytest.mark.gpu

ACTS = {"silu": torch.nn.functional.silu, "sigmoid": torch.sigmoid,
        "leaky_relu": lambda z: torch.nn.functional.leaky_relu(z, 0.01), "": lambda z: z}


def fp8_reference(x8, W, act, x_scale, h_scale):
    z = torch.bmm(x8.float(), W.w1t.float().transpose(1, 2)) * (x_scale * W.w1_scale)
    h8 = (ACTS[act](z) / h_scale).clamp(-448.0, 448.0).to(torch.float8_e4m3fn).float()
    o = torch.bmm(h8, W.w2t.float().transpose(1, 2)) * (h_scale * W.w2_scale)
    return o, z


def make_case(H, B, D, E, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(H, B, D, device="cuda", generator=g)
    w1 = torch.randn(H, D, E, device="cuda", generator=g) / D ** 0.5
    w2 = torch.randn(H, E, D, device="cuda", generator=g) / E ** 0.5
    x8, sx = F.quantize_e4m3(x)
    return x8, sx, F.prepare_fp8_weights(w1, w2)


def h_scale_for(z, act):
    return max(float(ACTS[act](z).abs().max()) / 448.0, 1e-6)


@pytest.mark.parametrize("H,B,D,E,act,out", [
    (4, 8192, 128, 2048, "silu", torch.bfloat16),   # a 4-head slice of the C4 shape
    (2, 1000, 64, 272, "sigmoid", torch.float16),   # ragged B, E not a multiple of 128
    (3, 384, 48, 512, "leaky_relu", torch.bfloat16),  # D < 128 (zero-filled K), odd B tiles
    (1, 257, 128, 128, "", torch.float16),          # one E chunk, linear
    (2, 4096, 112, 1040, "silu", torch.bfloat16),
])
def test_fp8_forward_matches_quantized_reference(H, B, D, E, act, out):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    x8, sx, W = make_case(H, B, D, E, seed=H * 7 + D)
    _, z = fp8_reference(x8, W, act, sx, 1.0)
    sh = h_scale_for(z, act)
    ref, _ = fp8_reference(x8, W, act, sx, sh)
    o = F.flashmlp_fwd_fp8(x8, W, act, x_scale=sx, h_scale=sh, out_dtype=out)
    torch.cuda.synchronize()
    assert o.shape == (H, B, D) and o.dtype == out
    assert torch.isfinite(o.float()).all()
    err = (o.float() - ref)
    rel = float(err.norm() / ref.norm())
    print(f"fp8 fwd ({H},{B},{D},{E}) {act or 'linear'}: ||o-r||/||r|| {rel:.2e}, max abs {float(err.abs().max()):.3e}")
    assert rel <= 1e-2, rel
    assert float(err.abs().max()) <= 0.05 * float(ref.abs().max()) + 1e-6
    assert _lib.lib().fmlp_device_status(1) == 0


def test_fp8_forward_close_to_16bit_forward():
    """End to end, quantization included: the FP8 forward of bf16 data stays within a few
    percent (norm-wise) of the bf16 kernel on the same values."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    H, B, D, E = 2, 4096, 128, 1024
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(H, B, D, device="cuda", generator=g).bfloat16()
    w1 = (torch.randn(H, D, E, device="cuda", generator=g) / D ** 0.5).bfloat16()
    w2 = (torch.randn(H, E, D, device="cuda", generator=g) / E ** 0.5).bfloat16()
    o16 = F.flashmlp_fwd(x, w1, w2, "silu").float()
    x8, sx = F.quantize_e4m3(x)
    W = F.prepare_fp8_weights(w1, w2)
    _, z = fp8_reference(x8, W, "silu", sx, 1.0)
    o8 = F.flashmlp_fwd_fp8(x8, W, "silu", x_scale=sx, h_scale=h_scale_for(z, "silu")).float()
    rel = float((o8 - o16).norm() / o16.norm())
    print(f"fp8 vs bf16 forward: {rel:.3e}")
    assert rel < 0.08, rel


def test_fp8_forward_rejects_bad_arguments():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    x8, sx, W = make_case(1, 256, 64, 256, seed=3)
    with pytest.raises(F.FlashMLPError):
        F.flashmlp_fwd_fp8(x8, W, "silu", x_scale=0.0)
    x8b, _, Wb = make_case(1, 256, 144, 256, seed=4)
    with pytest.raises(F.FlashMLPError):
        F.flashmlp_fwd_fp8(x8b, Wb, "silu")
    with pytest.raises(TypeError):
        F.flashmlp_fwd_fp8(x8, W, "silu", out_dtype=torch.float32)
