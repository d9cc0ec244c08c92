"""Host-side FP8 helpers (flashmlp_b200.fp8), no GPU: per-tensor e4m3 quantization and
the transposed weight layout fmlp_fwd_fp8 takes."""
import pytest
import torch

import flashmlp_b200 as F


def test_quantize_e4m3_scale_and_saturation():
    g = torch.Generator().manual_seed(0)
    t = torch.randn(4, 64, 96, generator=g) * 3.0
    t8, s = F.quantize_e4m3(t)
    assert t8.dtype == torch.float8_e4m3fn
    assert s == pytest.approx(float(t.abs().max()) / 448.0)
    back = t8.float() * s
    # e4m3 keeps 3 mantissa bits: relative error at most 2^-4 above the subnormal range
    big = t.abs() > s * 2.0 ** -6
    assert ((back - t).abs()[big] <= t.abs()[big] * 2.0 ** -4 + 1e-12).all()
    assert float(t8.float().abs().max()) == 448.0  # the amax element maps to the top value
    # a fixed scale saturates instead of overflowing to NaN
    t8s, s2 = F.quantize_e4m3(t, scale=1e-3)
    assert s2 == 1e-3 and torch.isfinite(t8s.float()).all() and float(t8s.float().abs().max()) == 448.0
    z8, sz = F.quantize_e4m3(torch.zeros(3, 3))
    assert sz == 1.0 and (z8.float() == 0).all()


def test_prepare_fp8_weights_transposes():
    g = torch.Generator().manual_seed(1)
    w1 = torch.randn(3, 64, 160, generator=g) / 8
    w2 = torch.randn(3, 160, 64, generator=g) / 12
    W = F.prepare_fp8_weights(w1, w2)
    assert W.w1t.shape == (3, 160, 64) and W.w2t.shape == (3, 64, 160)
    assert W.w1t.is_contiguous() and W.w2t.is_contiguous()
    q1, s1 = F.quantize_e4m3(w1)
    q2, s2 = F.quantize_e4m3(w2)
    assert W.w1_scale == s1 and W.w2_scale == s2
    assert torch.equal(W.w1t.float(), q1.float().transpose(1, 2))
    assert torch.equal(W.w2t.float(), q2.float().transpose(1, 2))
    with pytest.raises(AssertionError):
        F.prepare_fp8_weights(w1, w2[:, :100])


def test_fp8_forward_needs_cuda_tensors():
    x8 = torch.zeros(1, 128, 64).to(torch.float8_e4m3fn)
    W = F.prepare_fp8_weights(torch.zeros(1, 64, 128), torch.zeros(1, 128, 64))
    with pytest.raises(RuntimeError, match="CUDA"):
        F.flashmlp_fwd_fp8(x8, W)
    with pytest.raises(TypeError):
        F.flashmlp_fwd_fp8(torch.zeros(1, 128, 64), W)
