"""float32 inputs: the TF32 kernels (fmlp_tf32.cu) against the reference's fp32 semantics.

The reference's Triton kernels accept fp32 tensors; tl.dot then multiplies at TF32
precision and H / dZ stay fp32 (flashmlp.py:140-147, :227-235). The kernels here do the
same with tcgen05.mma kind::tf32. Checked against a plain-PyTorch fp32 evaluation on the
GPU (tolerance 5e-3 / 1e-2 plus the dot-product bound 2^-10 * sum |p||q|, the TF32 operand
rounding), against the reference's own goldens (tests/test_kernels_gpu.py, case f32_main)
and through the module."""
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


@pytest.mark.parametrize("shape", [(2, 200, 64, 136), (1, 333, 128, 520), (3, 1000, 96, 264), (1, 7, 16, 8),
                                   (4, 4096, 128, 1024), (2, 130, 48, 64)])
def test_tf32_vs_torch_fp32(shape):
    H, B, D, E = shape
    dt = torch.float32
    x, w1, w2, do = make_inputs(H, B, D, E, dt, seed=sum(shape))
    for act in ACTS:
        o = F().flashmlp_fwd(x, w1, w2, act)
        assert o.dtype == torch.float32
        r, bnd = ref_fwd(x, w1, w2, act)
        assert_close(o, r, bnd, dt, "fwd", f"{shape}/{act}/o")
        dx, dw1, dw2 = F().flashmlp_bwd(x, w1, w2, do, act)
        refs = ref_bwd(x, w1, w2, do, act)
        for k, v in (("dx", dx), ("dw1", dw1), ("dw2", dw2)):
            assert v.dtype == torch.float32
            assert_close(v, *refs[k], dt, "bwd", f"{shape}/{act}/{k}")


def test_tf32_deterministic_and_dw_f32_entry():
    x, w1, w2, do = make_inputs(2, 2048, 128, 512, torch.float32, seed=4)
    a = F().flashmlp_bwd(x, w1, w2, do, "silu")
    b = F().flashmlp_bwd(x, w1, w2, do, "silu")
    for u, v in zip(a, b):
        assert torch.equal(u, v)
    dx, dwf = F().flashmlp_bwd_dw_f32(x, w1, w2, do, "silu")
    n1 = w1.numel()
    assert torch.equal(dx, a[0]) and torch.equal(dwf[:n1].view(w1.shape), a[1]) and torch.equal(dwf[n1:].view(w2.shape), a[2])


def test_tf32_module_matches_pytorch_module():
    torch.manual_seed(2)
    H, B, D, E = 4, 512, 64, 256
    fm = F().FlashMLP(H, D, E, activation="sigmoid", dtype=torch.float32, device="cuda")
    pm = F().PyTorchMLP(H, D, E, activation="sigmoid", dtype=torch.float32, device="cuda")
    pm.load_state_dict(fm.state_dict())
    for shape in ((H, B, D), (B, D)):  # per-head input and the 2-D (expanded) input
        x = torch.randn(*shape, device="cuda", requires_grad=True)
        of = fm(x)
        of.sum().backward()
        gx, g1 = x.grad.clone(), fm.w1.grad.clone()
        x.grad = None
        fm.w1.grad = None
        op = pm(x)
        op.sum().backward()
        assert torch.allclose(of, op, atol=5e-3, rtol=5e-3)
        assert torch.allclose(gx, x.grad, atol=1e-2, rtol=1e-2)
        assert torch.allclose(g1, pm.w1.grad, atol=2e-2, rtol=2e-2)
        pm.w1.grad = None
        x.grad = None


def test_tf32_split_dw_programs():
    # 4 heads of C4 in fp32 (the per-GPU launch of 8-way head sharding): 64 (head, E chunk)
    # dW programs for 148 SMs, so they are split over B ranges, their fp32 partials added
    # in split order by fmlp_dw_reduce_f32_kernel.
    from flashmlp_b200 import _lib

    H, B, D, E = 4, 65536, 128, 2048
    dt = torch.float32
    L = _lib.lib()
    need = int(L.fmlp_bwd_workspace_size_min(H, B, D, E, _lib.FMLP_DTYPE_F32))
    mode, splits, launches = _lib.bwd_plan(H, B, D, E, _lib.FMLP_DTYPE_F32, need)
    assert need > 0 and mode == 0 and splits > 1 and launches == 2
    x, w1, w2, do = make_inputs(H, B, D, E, dt, seed=44)
    with F().low_memory_backward():  # the recompute mode (the default is the dZ-store mode)
        got = F().flashmlp_bwd(x, w1, w2, do, "silu")
        dxf, dwf = F().flashmlp_bwd_dw_f32(x, w1, w2, do, "silu")
        again = F().flashmlp_bwd(x, w1, w2, do, "silu")
    refs = ref_bwd(x, w1, w2, do, "silu")
    for i, k in enumerate(("dx", "dw1", "dw2")):
        assert_close(got[i], *refs[k], dt, "bwd", k)
    n1 = H * D * E
    assert torch.equal(dxf, got[0])
    assert torch.equal(dwf[:n1].view(H, D, E), got[1]) and torch.equal(dwf[n1:].view(H, E, D), got[2])
    for u, v in zip(got, again):  # a second call repeats every bit
        assert torch.equal(u, v)
