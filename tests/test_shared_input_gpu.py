"""Shared-input (2-D) path: one (B, D) input for every head, output the mean over heads.

The reference's FlashMLP expands a 2-D input to (H, B, D), runs the per-head kernels and
averages the outputs (flashmlp.py:603-614); its backward sums the per-head dX (the
expand) and feeds each head dO / H (the mean). fmlp_fwd_shared_x / fmlp_bwd_shared_x do
the same without the H copies. Checked against a plain-PyTorch fp32 evaluation with the
kernels' rounding points (the README tolerance plus the dot-product bound), against the
per-head kernels on the expanded input, and through the module's autograd."""
import pytest
import torch

from _refcheck import assert_close, make_inputs, ref_bwd, ref_fwd

pytestmark = pytest.mark.gpu

ACTS = ["", "leaky_relu", "silu", "sigmoid"]


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import flashmlp_b200  # noqa: F401
    yield
    from flashmlp_b200 import _lib
    assert _lib.lib().fmlp_device_status(1) == 0, "a kernel reported a pipeline timeout"


def F():
    import flashmlp_b200
    return flashmlp_b200


def _shared_inputs(H, B, D, E, dt, seed):
    x, w1, w2, do = make_inputs(H, B, D, E, dt, seed=seed)
    return x[0].contiguous(), w1, w2, do[0].contiguous()


def _check(H, B, D, E, dt, act, seed):
    x, w1, w2, do = _shared_inputs(H, B, D, E, dt, seed)
    xe = x.unsqueeze(0).expand(H, B, D)
    o = F().flashmlp_fwd_shared_x(x, w1, w2, act)
    r, bnd = ref_fwd(xe, w1, w2, act)
    assert_close(o, r.mean(0), bnd.mean(0), dt, "fwd", f"{(H, B, D, E)}/{act}/o")
    dx, dw1, dw2 = F().flashmlp_bwd_shared_x(x, w1, w2, do, act)
    refs = ref_bwd(xe, w1, w2, (do.float() / H).unsqueeze(0).expand(H, B, D), act)
    assert_close(dx, refs["dx"][0].sum(0), refs["dx"][1].sum(0), dt, "bwd", f"{(H, B, D, E)}/{act}/dx")
    assert_close(dw1, *refs["dw1"], dt, "bwd", f"{(H, B, D, E)}/{act}/dw1")
    assert_close(dw2, *refs["dw2"], dt, "bwd", f"{(H, B, D, E)}/{act}/dw2")
    return x, w1, w2, do, o, (dx, dw1, dw2)


@pytest.mark.parametrize("shape,dt", [((4, 2048, 128, 512), torch.bfloat16), ((12, 1000, 96, 3000), torch.bfloat16),
                                      ((3, 333, 64, 200), torch.float16), ((1, 1, 16, 8), torch.bfloat16),
                                      ((2, 4096, 128, 256), torch.float16)])
def test_shared_input_vs_torch_fp32(shape, dt):
    for act in ACTS:
        _check(*shape, dt, act, seed=sum(shape))


def test_shared_input_matches_expanded_per_head_kernels():
    # the same quantities through the per-head kernels on the materialised expansion
    H, B, D, E = 8, 4096, 128, 1024
    dt = torch.bfloat16
    x, w1, w2, do, o, (dx, dw1, dw2) = _check(H, B, D, E, dt, "silu", seed=3)
    xe = x.unsqueeze(0).expand(H, B, D).contiguous()
    oe = F().flashmlp_fwd(xe, w1, w2, "silu").float().mean(0)
    assert (o.float() - oe).abs().max().item() < 2e-2
    dxe, dw1e, dw2e = F().flashmlp_bwd(xe, w1, w2, (do.float() / H).to(dt).unsqueeze(0).expand(H, B, D).contiguous(),
                                       "silu")
    refs = ref_bwd(xe, w1, w2, (do.float() / H).unsqueeze(0).expand(H, B, D), "silu")
    assert_close(dx, dxe.float().sum(0), refs["dx"][1].sum(0), dt, "bwd", "dx vs expanded")
    assert_close(dw1, dw1e.float(), refs["dw1"][1], dt, "bwd", "dw1 vs expanded")
    assert_close(dw2, dw2e.float(), refs["dw2"][1], dt, "bwd", "dw2 vs expanded")


def test_shared_input_deterministic_and_split_dw():
    from flashmlp_b200 import _lib

    H, B, D, E = 2, 4096, 128, 256
    assert _lib.lib().fmlp_bwd_workspace_size_min(H, B, D, E, 1) > 0  # dW programs split over B
    x, w1, w2, do = _shared_inputs(H, B, D, E, torch.bfloat16, 9)
    a = F().flashmlp_bwd_shared_x(x, w1, w2, do, "sigmoid")
    b = F().flashmlp_bwd_shared_x(x, w1, w2, do, "sigmoid")
    for u, v in zip(a, b):
        assert torch.equal(u, v)
    assert torch.equal(F().flashmlp_fwd_shared_x(x, w1, w2, "sigmoid"), F().flashmlp_fwd_shared_x(x, w1, w2, "sigmoid"))


def test_module_two_dim_input_uses_shared_kernels_and_matches_pytorch_module():
    torch.manual_seed(1)
    H, B, D, E = 6, 1000, 128, 640
    fm = F().FlashMLP(H, D, E, activation="leaky_relu", dtype=torch.bfloat16, device="cuda")
    pm = F().PyTorchMLP(H, D, E, activation="leaky_relu", dtype=torch.bfloat16, device="cuda")
    pm.load_state_dict(fm.state_dict())
    x = torch.randn(B, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    of = fm(x)
    assert of.shape == (B, D) and of.grad_fn.__class__.__name__.startswith("FlashMLPSharedInputFunction")
    of.float().sum().backward()
    gx, g1, g2 = x.grad.clone(), fm.w1.grad.clone(), fm.w2.grad.clone()
    x.grad = None
    op = pm(x)
    op.float().sum().backward()
    assert torch.allclose(of.float(), op.float(), atol=1e-2, rtol=1e-2)
    for a, b in ((gx, x.grad), (g1, pm.w1.grad), (g2, pm.w2.grad)):
        assert torch.allclose(a.float(), b.float(), atol=3e-2, rtol=3e-2)


def test_shared_input_rejects_large_d_and_zero_heads():
    x, w1, w2, do = _shared_inputs(1, 64, 256, 64, torch.bfloat16, 0)
    with pytest.raises(F().FlashMLPError, match="hidden dim"):
        F().flashmlp_fwd_shared_x(x, w1, w2, "")
    with pytest.raises(F().FlashMLPError, match="hidden dim"):
        F().flashmlp_bwd_shared_x(x, w1, w2, do, "")
    x, w1, w2, do = _shared_inputs(1, 64, 64, 64, torch.bfloat16, 0)
    with pytest.raises(F().FlashMLPError, match="invalid shape"):
        F().flashmlp_fwd_shared_x(x, w1[:0], w2[:0], "")
