"""Host-side API behaviour that needs no GPU: the reference's assertion messages, the
activation mapping, loud failure for non-CUDA tensors, and the plain-PyTorch exports."""
import numpy as np
import pytest
import torch

import flashmlp_b200 as F
from oracle import flashmlp_oracle as orc


def t(*shape, dtype=torch.bfloat16):
    return torch.zeros(*shape, dtype=dtype)


@pytest.mark.parametrize(
    "shapes,msg",
    [
        (((2, 8, 16), (3, 16, 32), (2, 32, 16)), "Number of heads must match"),
        (((2, 8, 16), (2, 16, 32), (3, 32, 16)), "Number of heads must match"),
        (((2, 8, 16), (2, 8, 32), (2, 32, 16)), "Hidden dimension mismatch"),
        (((2, 8, 16), (2, 16, 32), (2, 24, 16)), "Intermediate dimension mismatch"),
        (((2, 8, 16), (2, 16, 32), (2, 32, 8)), "Output dimension mismatch"),
    ],
)
def test_fwd_shape_assertions_match_reference(shapes, msg):
    with pytest.raises(AssertionError, match=msg):
        F.flashmlp_fwd(*(t(*s) for s in shapes))


def test_bwd_shape_assertions_match_reference():
    x, w1, w2 = t(2, 8, 16), t(2, 16, 32), t(2, 32, 16)
    with pytest.raises(AssertionError, match="Gradient shape mismatch"):
        F.flashmlp_bwd(x, w1, w2, t(2, 9, 16))
    with pytest.raises(AssertionError, match="Hidden dimension mismatch"):
        F.flashmlp_bwd(x, t(2, 8, 32), w2, x)


def test_noncontiguous_after_reshape_is_rejected_like_reference():
    base = t(2, 8, 32)
    x = base[:, :, ::2]  # reshape(H*B, D) is a non-contiguous view
    with pytest.raises(AssertionError, match="Input X must be contiguous"):
        F.flashmlp_fwd(x, t(2, 16, 32), t(2, 32, 16))


def test_cpu_tensors_fail_loudly():
    with pytest.raises(RuntimeError, match="CUDA"):
        F.flashmlp_fwd(t(2, 8, 16), t(2, 16, 32), t(2, 32, 16), "silu")
    with pytest.raises(RuntimeError, match="CUDA"):
        F.flashmlp_bwd(t(2, 8, 16), t(2, 16, 32), t(2, 32, 16), t(2, 8, 16), "silu")


def test_activation_codes():
    assert F.activation_code("") == 0
    assert F.activation_code("leaky_relu") == 1
    assert F.activation_code("silu") == 2
    assert F.activation_code("sigmoid") == 3
    assert F.activation_code("gelu") == 0  # unknown names are linear, as in the reference


def test_module_parameters_match_reference_layout():
    m = F.FlashMLP(4, 32, 64, activation="sigmoid", dtype=torch.float32, device="cpu")
    assert m.w1.shape == (4, 32, 64) and m.w2.shape == (4, 64, 32)
    assert set(m.state_dict()) == {"w1", "w2"}
    assert m.num_heads == 4 and m.hidden_dim == 32 and m.intermediate_dim == 64
    # randn / sqrt(E) and randn / sqrt(D) (flashmlp.py:586-591)
    big = F.FlashMLP(2, 256, 1024, dtype=torch.float32, device="cpu")
    assert abs(big.w1.std().item() - 1 / 32) < 3e-3
    assert abs(big.w2.std().item() - 1 / 16) < 6e-3


@pytest.mark.parametrize("act", ["", "leaky_relu", "silu", "sigmoid"])
def test_torch_reference_exports_match_oracle(act):
    x, w1, w2, do = orc.make_inputs(2, 64, 32, 96, "f16", seed=1)
    tx, tw1, tw2, tdo = map(torch.from_numpy, (x, w1, w2, do))
    o = F.flashmlp_torch_fwd(tx, tw1, tw2, act).numpy()
    np.testing.assert_allclose(o, orc.fwd_fp32(x, w1, w2, act), rtol=1e-5, atol=1e-5)
    for a, r in zip(F.flashmlp_torch_bwd(tx, tw1, tw2, tdo, act), orc.bwd_fp32(x, w1, w2, do, act)):
        np.testing.assert_allclose(a.numpy(), r, rtol=1e-4, atol=1e-5)
    m = F.PyTorchMLP(2, 32, 96, activation=act, dtype=torch.float32, device="cpu")
    with torch.no_grad():
        m.w1.copy_(tw1)
        m.w2.copy_(tw2)
        np.testing.assert_allclose(m(tx).numpy(), orc.fwd_fp32(x, w1, w2, act), rtol=1e-5, atol=1e-5)
        o2 = m(tx[0]).numpy()  # 2-D input: broadcast to every head, mean over heads
        want = orc.fwd_fp32(np.broadcast_to(x[0], x.shape).copy(), w1, w2, act).mean(0)
        np.testing.assert_allclose(o2, want, rtol=1e-5, atol=1e-5)
