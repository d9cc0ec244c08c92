"""Autograd and module glue, re-expressing the reference's own checks as asserts:
test_autograd (flashmlp.py:799-855), test_module (flashmlp.py:858-887) and
example.py:compare_correctness (example.py:11-61)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def test_autograd_function_matches_torch_autograd():
    import flashmlp_b200 as F

    torch.manual_seed(42)
    dtype = torch.bfloat16
    H, B, D, E = 8, 512, 64, 512
    x = (torch.randn((H, B, D), device="cuda", dtype=dtype) / np.sqrt(D)).requires_grad_(True)
    w1 = (torch.randn((H, D, E), device="cuda", dtype=dtype) / np.sqrt(E)).requires_grad_(True)
    w2 = (torch.randn((H, E, D), device="cuda", dtype=dtype) / np.sqrt(D)).requires_grad_(True)
    o = F.FlashMLPFunction.apply(x, w1, w2, "silu")
    o.sum().backward()
    grads = [t.grad.clone() for t in (x, w1, w2)]
    for t in (x, w1, w2):
        t.grad = None
    o_ref = F.flashmlp_torch_fwd(x, w1, w2, "silu")
    o_ref.sum().backward()
    assert torch.allclose(o, o_ref, atol=1e-2, rtol=1e-2)
    for g, t in zip(grads, (x, w1, w2)):
        assert torch.allclose(g, t.grad, atol=3e-2, rtol=3e-2)


def test_autograd_saves_only_inputs():
    import flashmlp_b200 as F

    x, w1, w2 = (torch.randn(s, device="cuda", dtype=torch.float16, requires_grad=True)
                 for s in ((2, 64, 64), (2, 64, 128), (2, 128, 64)))
    o = F.FlashMLPFunction.apply(x, w1, w2, "sigmoid")
    saved = o.grad_fn.saved_tensors
    assert len(saved) == 3
    assert all(s.data_ptr() == t.data_ptr() for s, t in zip(saved, (x, w1, w2)))


@pytest.mark.parametrize("activation", ["", "silu", "leaky_relu", "sigmoid"])
def test_module_matches_pytorch_module(activation):
    """example.py:compare_correctness, with asserts. Both modules run in bf16; the
    PyTorch module rounds every intermediate to bf16, so the comparison is made against
    an fp32 evaluation of the same weights: FlashMLP must be at least as close to it as
    the reference's bf16 PyTorch module, and agree with that module within the
    reference's tolerance (fwd 1e-2 everywhere, grads 3e-2 on >= 99.9% of elements)."""
    import flashmlp_b200 as F

    torch.manual_seed(42)
    dtype = torch.bfloat16
    H, B, D, E = 12, 1024, 64, 768
    fm = F.FlashMLP(H, D, E, activation=activation, dtype=dtype, device="cuda")
    pm = F.PyTorchMLP(H, D, E, activation=activation, dtype=dtype, device="cuda")
    pm.load_state_dict(fm.state_dict())  # same parameter names and shapes
    x = (torch.randn(H, B, D, device="cuda", dtype=dtype) / np.sqrt(D)).requires_grad_(True)
    of = fm(x)
    of.sum().backward()
    gx = x.grad.clone()
    x.grad = None
    op = pm(x)
    op.sum().backward()
    # fp32 evaluation of the same function
    xf = x.detach().float().requires_grad_(True)
    w1f = fm.w1.detach().float().requires_grad_(True)
    w2f = fm.w2.detach().float().requires_grad_(True)
    F.flashmlp_torch_fwd(xf, w1f, w2f, activation).sum().backward()
    assert torch.allclose(of, op, atol=1e-2, rtol=1e-2)
    for ours, theirs, truth in ((gx, x.grad, xf.grad), (fm.w1.grad, pm.w1.grad, w1f.grad),
                                (fm.w2.grad, pm.w2.grad, w2f.grad)):
        e_ours = (ours.float() - truth).abs().max().item()
        e_ref = (theirs.float() - truth).abs().max().item()
        assert e_ours <= 1.1 * e_ref + 1e-3, (e_ours, e_ref)
        ok = torch.isclose(ours, theirs, atol=3e-2, rtol=3e-2).float().mean().item()
        assert ok >= 0.999, ok


def test_module_two_dim_input_broadcasts_and_averages():
    import flashmlp_b200 as F

    torch.manual_seed(0)
    H, B, D, E = 4, 256, 64, 256
    fm = F.FlashMLP(H, D, E, activation="silu", dtype=torch.float16, device="cuda")
    pm = F.PyTorchMLP(H, D, E, activation="silu", dtype=torch.float16, device="cuda")
    pm.load_state_dict(fm.state_dict())
    x = torch.randn(B, D, device="cuda", dtype=torch.float16, requires_grad=True)
    of = fm(x)
    assert of.shape == (B, D)
    of.float().pow(2).sum().backward()
    gx = x.grad.clone()
    x.grad = None
    op = pm(x)
    op.float().pow(2).sum().backward()
    assert torch.allclose(of, op, atol=1e-2, rtol=1e-2)
    assert torch.allclose(gx, x.grad, atol=3e-2, rtol=3e-2)


def test_module_smoke_shapes_and_grads():
    import flashmlp_b200 as F

    torch.manual_seed(42)
    H, B, D, E = 8, 512, 64, 512
    model = F.FlashMLP(num_heads=H, hidden_dim=D, intermediate_dim=E, activation="silu",
                       dtype=torch.bfloat16, device="cuda")
    x = torch.randn((H, B, D), device="cuda", dtype=torch.bfloat16, requires_grad=True)
    o = model(x)
    assert o.shape == (H, B, D) and o.dtype == torch.bfloat16
    o.sum().backward()
    assert x.grad is not None and model.w1.grad is not None and model.w2.grad is not None
    assert torch.isfinite(model.w1.grad.float()).all()


def test_drop_in_module_name():
    import flashmlp

    assert flashmlp.FlashMLP is not None and flashmlp.PyTorchMLP is not None
    assert callable(flashmlp.flashmlp_fwd) and callable(flashmlp.flashmlp_bwd)


@pytest.mark.parametrize("H,hg", [(7, 3), (13, 4)])  # (13, 4): groups ramp 1, 2, 4, 3, 2, 1
def test_host_pipeline_matches_device_calls(H, hg):
    # host-resident inputs, head groups pipelined over three streams: the same bits as the
    # device calls on each head group; H not a multiple of the group
    import flashmlp_b200 as F
    from flashmlp_b200.host import HostPipeline

    B, D, E = 1000, 64, 264
    g = torch.Generator().manual_seed(3)
    x = torch.randn(H, B, D, generator=g).to(torch.bfloat16).pin_memory()
    w1 = (torch.randn(H, D, E, generator=g) / D ** 0.5).to(torch.bfloat16).pin_memory()
    w2 = (torch.randn(H, E, D, generator=g) / E ** 0.5).to(torch.bfloat16).pin_memory()
    do = torch.randn(H, B, D, generator=g).to(torch.bfloat16).pin_memory()
    pipe = HostPipeline("cuda", heads_per_group=hg)
    xd, w1d, w2d, dod = x.cuda(), w1.cuda(), w2.cuda(), do.cuda()
    whole = [F.flashmlp_fwd(xd, w1d, w2d, "silu"), *F.flashmlp_bwd(xd, w1d, w2d, dod, "silu")]
    # per head group, as the pipeline launches them: dW too is bit-identical (a launch's
    # dW split over B ranges depends on its head count, so against the whole-tensor call
    # only O and dX are)
    grouped = [[], [], [], []]
    for a, b in pipe._groups(H, hg):
        for k, t in enumerate([F.flashmlp_fwd(xd[a:b], w1d[a:b], w2d[a:b], "silu"),
                               *F.flashmlp_bwd(xd[a:b], w1d[a:b], w2d[a:b], dod[a:b], "silu")]):
            grouped[k].append(t)
    grouped = [torch.cat(ts) for ts in grouped]
    for _ in range(2):  # buffers reused on the second call
        outs = pipe.run(x, w1, w2, do, "silu")
        torch.cuda.synchronize()
        for a, r in zip(outs, grouped):
            assert a.device.type == "cpu" and torch.equal(a, r.cpu())
        for a, r in zip(outs[:2], whole[:2]):
            assert torch.equal(a, r.cpu())
