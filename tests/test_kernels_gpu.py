"""Parity of the sm_100a forward and unified backward kernels (through the C ABI).

* against the golden fixtures produced by the reference itself (its PyTorch path in fp32
  and its Triton kernels in fp16);
* against the CPU oracle (kernel rounding points) on seeded inputs with ragged shapes;
* at BASELINE sizes against a plain-PyTorch fp32 reference on the GPU, plus
  size-independent properties (determinism, head/row permutation equivariance);
* edge cases: empty dimensions, unsupported shapes, guard regions around outputs.
"""
import numpy as np
import pytest
import torch

from conftest import GOLDEN_CASES, load_golden
from _refcheck import assert_close, make_inputs, ref_bwd, ref_fwd, tol_for, to_np

pytestmark = pytest.mark.gpu

ACTS = ["", "leaky_relu", "silu", "sigmoid"]


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import flashmlp_b200  # noqa: F401  (fails loudly if the library is missing)
    yield
    from flashmlp_b200 import _lib
    assert _lib.lib().fmlp_device_status(1) == 0, "a kernel reported a pipeline timeout"


def F():
    import flashmlp_b200
    return flashmlp_b200


def _torch_dtype(d):
    return {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[d]


def _golden_tensors(g):
    dt = _torch_dtype(g["dtype"])
    return [torch.from_numpy(g[k]).to(dt).cuda() for k in ("x", "w1", "w2", "do")]


# ----------------------------------------------------------------------------- goldens
@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_fwd_matches_reference_goldens(case):
    g = load_golden(case)
    x, w1, w2, _ = _golden_tensors(g)
    dt = x.dtype
    atol, rtol = tol_for(dt, "fwd")
    for act in g["acts"]:
        tag = act or "linear"
        o = to_np(F().flashmlp_fwd(x, w1, w2, act))
        np.testing.assert_allclose(o, g[f"torch_o_{tag}"], atol=atol, rtol=rtol, err_msg=f"{case}/{tag}")
        if f"triton_o_{tag}" in g and dt == torch.float32:
            # the reference's Triton kernel on fp32 (exact fp32 dots under the interpreter;
            # TF32 products here): the README tolerance
            np.testing.assert_allclose(o, g[f"triton_o_{tag}"], atol=atol, rtol=rtol, err_msg=f"{case}/{tag} vs triton")
        elif f"triton_o_{tag}" in g:
            # the reference's own Triton kernel (fp16, same rounding points): within 2 steps
            t = g[f"triton_o_{tag}"]
            ulp = np.spacing(np.abs(t).astype(np.float16)).astype(np.float32)
            assert (np.abs(o - t) <= 2 * ulp + 1e-3 * np.abs(t).max()).all(), f"{case}/{tag} vs triton"


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_bwd_matches_reference_goldens(case):
    g = load_golden(case)
    x, w1, w2, do = _golden_tensors(g)
    dt = x.dtype
    for act in g["acts"]:
        tag = act or "linear"
        got = dict(zip(("dx", "dw1", "dw2"), F().flashmlp_bwd(x, w1, w2, do, act)))
        bounds = ref_bwd(x, w1, w2, do, act)
        for k in ("dx", "dw1", "dw2"):
            # vs the reference's PyTorch path in fp32: README tolerance plus the dot-product
            # bound (the kernels round dZ/H to 16 bits as the reference's kernels do)
            want = torch.from_numpy(g[f"torch_{k}_{tag}"]).cuda()
            assert_close(got[k], want, bounds[k][1], dt, "bwd", f"{case}/{tag}/{k}")
            if f"triton_{k}_{tag}" in g and dt == torch.float32:
                assert_close(got[k], torch.from_numpy(g[f"triton_{k}_{tag}"]).cuda(), bounds[k][1], dt, "bwd",
                             f"{case}/{tag}/{k} vs triton")
            elif f"triton_{k}_{tag}" in g:
                # vs the reference's own Triton kernel (fp16, same rounding points)
                t = g[f"triton_{k}_{tag}"]
                a = to_np(got[k])
                ulp = np.spacing(np.abs(t).astype(np.float16)).astype(np.float32)
                assert (np.abs(a - t) <= 2 * ulp + 2e-3 * np.abs(t).max()).all(), f"{case}/{tag}/{k} vs triton"


# ----------------------------------------------------------------------------- oracle, ragged
RAGGED = [
    (1, 1, 16, 8), (1, 7, 32, 40), (2, 129, 64, 136), (3, 200, 96, 200), (1, 256, 128, 8),
    (2, 333, 80, 264), (1, 130, 112, 520),
]


@pytest.mark.parametrize("shape", RAGGED)
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_fwd_bwd_vs_oracle_ragged(shape, dtype):
    from oracle import flashmlp_oracle as orc

    H, B, D, E = shape
    xs = orc.make_inputs(H, B, D, E, dtype, seed=sum(shape))
    dt = _torch_dtype(dtype)
    x, w1, w2, do = (torch.from_numpy(a).to(dt).cuda() for a in xs)
    for act in ACTS:
        o = to_np(F().flashmlp_fwd(x, w1, w2, act))
        ro = orc.fwd_kernel(*xs[:3], act, dtype)
        atol, rtol = tol_for(dt, "fwd")
        np.testing.assert_allclose(o, ro, atol=atol, rtol=rtol, err_msg=f"{shape} {act} o")
        got = [to_np(t) for t in F().flashmlp_bwd(x, w1, w2, do, act)]
        want = orc.bwd_kernel(*xs, act, dtype)
        atol, rtol = tol_for(dt, "bwd")
        for name, a, r in zip(("dx", "dw1", "dw2"), got, want):
            np.testing.assert_allclose(a, r, atol=atol, rtol=rtol, err_msg=f"{shape} {act} {name}")


def test_d256_vs_oracle():
    # 128 < D <= 256 runs on the DP = 256 kernels (fwd: single-tile forward; bwd: D-half dW
    # programs and 64-wide-chunk dX programs); ragged B, D and E
    from oracle import flashmlp_oracle as orc

    for shape, dtype in [((2, 300, 256, 136), "f16"), ((1, 128, 192, 64), "bf16"), ((1, 64, 240, 48), "bf16"),
                         ((1, 257, 144, 200), "bf16")]:
        xs = orc.make_inputs(*shape, dtype, seed=7)
        dt = _torch_dtype(dtype)
        x, w1, w2, do = (torch.from_numpy(a).to(dt).cuda() for a in xs)
        for act in ACTS:
            o = to_np(F().flashmlp_fwd(x, w1, w2, act))
            atol, rtol = tol_for(dt, "fwd")
            np.testing.assert_allclose(o, orc.fwd_kernel(*xs[:3], act, dtype), atol=atol, rtol=rtol,
                                       err_msg=f"{shape} {act} o")
            got = [to_np(t) for t in F().flashmlp_bwd(x, w1, w2, do, act)]
            want = orc.bwd_kernel(*xs, act, dtype)
            atol, rtol = tol_for(dt, "bwd")
            for name, a, r in zip(("dx", "dw1", "dw2"), got, want):
                np.testing.assert_allclose(a, r, atol=atol, rtol=rtol, err_msg=f"{shape} {act} {name}")


# ----------------------------------------------------------------------------- split dW programs
# (recompute mode, selected by the least workspace; the dZ-store mode has its own file)
def _ws_bytes(H, B, D, E, dt):
    from flashmlp_b200 import _lib
    code = _lib.FMLP_DTYPE_BF16 if dt == torch.bfloat16 else _lib.FMLP_DTYPE_F16
    return int(_lib.lib().fmlp_bwd_workspace_size_min(H, B, D, E, code))


@pytest.mark.parametrize("shape,dtype", [((2, 1000, 96, 200), "bf16"), ((1, 2048, 128, 256), "f16"),
                                         ((3, 1100, 64, 520), "bf16"), ((2, 4096, 16, 136), "f16")])
def test_split_dw_vs_oracle(shape, dtype):
    # Few (head, E chunk) pairs: the dW programs are split over B ranges and their fp32
    # partials reduced by a second kernel; ragged B (1000, 1100) ends inside the last split.
    from oracle import flashmlp_oracle as orc

    H, B, D, E = shape
    dt = _torch_dtype(dtype)
    assert _ws_bytes(H, B, D, E, dt) > 0, "shape chosen to exercise split dW programs"
    xs = orc.make_inputs(H, B, D, E, dtype, seed=B + E)
    x, w1, w2, do = (torch.from_numpy(a).to(dt).cuda() for a in xs)
    atol, rtol = tol_for(dt, "bwd")
    for act in ACTS:
        with F().low_memory_backward():
            got = [to_np(t) for t in F().flashmlp_bwd(x, w1, w2, do, act)]
        want = orc.bwd_kernel(*xs, act, dtype)
        for name, a, r in zip(("dx", "dw1", "dw2"), got, want):
            np.testing.assert_allclose(a, r, atol=atol, rtol=rtol, err_msg=f"{shape} {act} {name}")


def test_split_dw_matches_unsplit_launch():
    # The same two heads computed alone (dW split 8 ways) and inside a 16-head launch (no
    # split): dX is bit-identical (the dX programs do not depend on the split); dW differs
    # only by the order of fp32 additions over B.
    H, B, D, E = 16, 8192, 128, 1024
    dt = torch.bfloat16
    assert _ws_bytes(2, B, D, E, dt) > 0 and _ws_bytes(H, B, D, E, dt) == 0
    x, w1, w2, do = make_inputs(H, B, D, E, dt, seed=21)
    with F().low_memory_backward():
        big = F().flashmlp_bwd(x, w1, w2, do, "silu")
        small = F().flashmlp_bwd(x[:2].contiguous(), w1[:2].contiguous(), w2[:2].contiguous(),
                                 do[:2].contiguous(), "silu")
    assert torch.equal(big[0][:2], small[0])
    refs = ref_bwd(x[:2], w1[:2], w2[:2], do[:2], "silu")
    for k, i in (("dw1", 1), ("dw2", 2)):
        assert_close(small[i], big[i][:2].float(), refs[k][1], dt, "bwd", k)
        assert_close(small[i], *refs[k], dt, "bwd", k)


@pytest.mark.parametrize("shape,dtype", [((4, 4096, 128, 1024), torch.bfloat16), ((16, 8192, 128, 1024), torch.bfloat16),
                                         ((2, 1000, 256, 520), torch.float16), ((3, 700, 64, 200), torch.float16)])
def test_bwd_dw_f32_rounds_to_bwd(shape, dtype):
    # The fp32-dW backward is the same computation: rounding its dW gives fmlp_bwd's dW bit
    # for bit, and dX is identical (split and unsplit dW programs, D <= 128 and D = 256).
    H, B, D, E = shape
    x, w1, w2, do = make_inputs(H, B, D, E, dtype, seed=13)
    for act in ("silu", "leaky_relu"):
        dx, dw1, dw2 = F().flashmlp_bwd(x, w1, w2, do, act)
        dxf, dwf = F().flashmlp_bwd_dw_f32(x, w1, w2, do, act)
        n1 = H * D * E
        assert torch.equal(dx, dxf)
        assert torch.equal(dwf[:n1].view(H, D, E).to(dtype), dw1)
        assert torch.equal(dwf[n1:].view(H, E, D).to(dtype), dw2)
    x, w1, w2, do = make_inputs(H, 0, D, E, dtype)
    _, dwf = F().flashmlp_bwd_dw_f32(x, w1, w2, do, "silu", dw_out=torch.full((2 * H * D * E,), 7.0, device="cuda"))
    assert torch.count_nonzero(dwf) == 0


def test_workspace_too_small_is_rejected():
    from flashmlp_b200 import _lib
    import ctypes

    H, B, D, E = 2, 2048, 128, 512
    dt = torch.bfloat16
    need = _ws_bytes(H, B, D, E, dt)
    assert need > 0
    x, w1, w2, do = make_inputs(H, B, D, E, dt, seed=5)
    outs = [torch.empty_like(t) for t in (x, w1, w2)]
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    L = _lib.lib()
    args = [p(x), p(w1), p(w2), p(do), *map(p, outs)]
    assert L.fmlp_bwd(*args, p(ws), need - 16, H, B, D, E, 1, 2, None) == 9  # FMLP_ERR_WORKSPACE
    assert L.fmlp_bwd(*args, None, need, H, B, D, E, 1, 2, None) == 9
    assert L.fmlp_bwd(*args, p(ws), need, H, B, D, E, 1, 2, None) == 0
    torch.cuda.synchronize()
    with F().low_memory_backward():
        assert torch.equal(outs[1], F().flashmlp_bwd(x, w1, w2, do, "silu")[1])


# ----------------------------------------------------------------------------- BASELINE configs
CONFIGS = {
    # name: (H, B, D, E, dtype, activations)
    "C1": (12, 1024, 64, 768, torch.float16, ["silu"]),
    "C2": (16, 16384, 128, 512, torch.bfloat16, ["leaky_relu"]),
    "C3": (12, 1000, 96, 3000, torch.bfloat16, ["", "sigmoid"]),
    "C4": (32, 65536, 128, 2048, torch.bfloat16, ["silu"]),
    # C4 head-sharded over 8 GPUs: the per-GPU launch (4 heads) splits its dW programs
    "C4_per_gpu_at_8": (4, 65536, 128, 2048, torch.bfloat16, ["silu"]),
    "C5": (8, 131072, 256, 1024, torch.float16, ["sigmoid"]),
}


@pytest.mark.parametrize("name", list(CONFIGS))
def test_baseline_config_vs_torch_fp32(name):
    H, B, D, E, dt, acts = CONFIGS[name]
    x, w1, w2, do = make_inputs(H, B, D, E, dt, seed=0)
    heads = list(range(H)) if H * B <= 16 * 16384 else [0, H // 2, H - 1]
    for act in acts:
        o = F().flashmlp_fwd(x, w1, w2, act)
        dx, dw1, dw2 = F().flashmlp_bwd(x, w1, w2, do, act)
        for h in heads:  # heads are independent: check a slice against the reference
            sl = slice(h, h + 1)
            r, bnd = ref_fwd(x[sl], w1[sl], w2[sl], act)
            assert_close(o[sl], r, bnd, dt, "fwd", f"{name}/{act}/o/h{h}")
            refs = ref_bwd(x[sl], w1[sl], w2[sl], do[sl], act)
            for k, v in (("dx", dx), ("dw1", dw1), ("dw2", dw2)):
                assert_close(v[sl], *refs[k], dt, "bwd", f"{name}/{act}/{k}/h{h}")
        del o, dx, dw1, dw2
    torch.cuda.empty_cache()


# ----------------------------------------------------------------------------- properties
def test_determinism_bitwise():
    x, w1, w2, do = make_inputs(4, 4096, 128, 1024, torch.bfloat16, seed=11)
    a = F().flashmlp_bwd(x, w1, w2, do, "silu")
    b = F().flashmlp_bwd(x, w1, w2, do, "silu")
    for u, v in zip(a, b):
        assert torch.equal(u, v)
    assert torch.equal(F().flashmlp_fwd(x, w1, w2, "silu"), F().flashmlp_fwd(x, w1, w2, "silu"))


def test_head_permutation_equivariance_c4_size():
    H, B, D, E = 32, 65536, 128, 2048
    x, w1, w2, do = make_inputs(H, B, D, E, torch.bfloat16, seed=3)
    perm = torch.randperm(H, generator=torch.Generator().manual_seed(0)).cuda()
    o = F().flashmlp_fwd(x, w1, w2, "silu")
    op = F().flashmlp_fwd(x[perm].contiguous(), w1[perm].contiguous(), w2[perm].contiguous(), "silu")
    assert torch.equal(o[perm], op)
    g = F().flashmlp_bwd(x, w1, w2, do, "silu")
    gp = F().flashmlp_bwd(x[perm].contiguous(), w1[perm].contiguous(), w2[perm].contiguous(),
                          do[perm].contiguous(), "silu")
    for u, v in zip(g, gp):
        assert torch.equal(u[perm], v)


def test_row_permutation_equivariance():
    # Each output row of O and dX depends only on its own input row.
    H, B, D, E = 2, 8192, 128, 1024
    x, w1, w2, do = make_inputs(H, B, D, E, torch.bfloat16, seed=4)
    perm = torch.randperm(B, generator=torch.Generator().manual_seed(1)).cuda()
    o = F().flashmlp_fwd(x, w1, w2, "sigmoid")
    op = F().flashmlp_fwd(x[:, perm].contiguous(), w1, w2, "sigmoid")
    assert torch.equal(o[:, perm], op)
    dx = F().flashmlp_bwd(x, w1, w2, do, "sigmoid")[0]
    dxp = F().flashmlp_bwd(x[:, perm].contiguous(), w1, w2, do[:, perm].contiguous(), "sigmoid")[0]
    assert torch.equal(dx[:, perm], dxp)


def test_dw_is_additive_over_batch_halves():
    H, B, D, E = 2, 8192, 64, 512
    x, w1, w2, do = make_inputs(H, B, D, E, torch.float16, seed=9)
    _, dw1, dw2 = F().flashmlp_bwd(x, w1, w2, do, "leaky_relu")
    h = B // 2
    _, a1, a2 = F().flashmlp_bwd(x[:, :h].contiguous(), w1, w2, do[:, :h].contiguous(), "leaky_relu")
    _, b1, b2 = F().flashmlp_bwd(x[:, h:].contiguous(), w1, w2, do[:, h:].contiguous(), "leaky_relu")
    bounds = ref_bwd(x, w1, w2, do, "leaky_relu")
    for name, full, p, q in (("dw1", dw1, a1, b1), ("dw2", dw2, a2, b2)):
        assert_close(full, p.float() + q.float(), bounds[name][1], torch.float16, "bwd", name)


# ----------------------------------------------------------------------------- edge cases
def test_empty_dimensions():
    dt = torch.bfloat16
    x, w1, w2, do = make_inputs(2, 0, 64, 64, dt)
    assert F().flashmlp_fwd(x, w1, w2, "silu").shape == (2, 0, 64)
    dx, dw1, dw2 = F().flashmlp_bwd(x, w1, w2, do, "silu")
    assert dx.shape == (2, 0, 64) and torch.count_nonzero(dw1) == 0 and torch.count_nonzero(dw2) == 0
    x, w1, w2, do = make_inputs(2, 100, 64, 0, dt)
    assert torch.count_nonzero(F().flashmlp_fwd(x, w1, w2, "sigmoid")) == 0
    dx, dw1, dw2 = F().flashmlp_bwd(x, w1, w2, do, "sigmoid")
    assert torch.count_nonzero(dx) == 0 and dw1.numel() == 0
    x, w1, w2, do = make_inputs(0, 100, 64, 64, dt)
    assert F().flashmlp_fwd(x, w1, w2, "").shape == (0, 100, 64)


def test_unsupported_shapes_raise():
    dt = torch.bfloat16
    x, w1, w2, do = make_inputs(1, 64, 72, 64, dt)  # D % 16 != 0
    with pytest.raises(F().FlashMLPError, match="hidden dim"):
        F().flashmlp_fwd(x, w1, w2, "")
    x, w1, w2, do = make_inputs(1, 64, 64, 100, dt)  # E % 8 != 0
    with pytest.raises(F().FlashMLPError, match="intermediate dim"):
        F().flashmlp_fwd(x, w1, w2, "")
    x, w1, w2, do = make_inputs(1, 64, 272, 64, dt)  # D > 256
    with pytest.raises(F().FlashMLPError, match="hidden dim"):
        F().flashmlp_fwd(x, w1, w2, "")
    with pytest.raises(F().FlashMLPError, match="hidden dim"):
        F().flashmlp_bwd(x, w1, w2, do, "")
    x, w1, w2, do = make_inputs(1, 64, 64, 64, torch.float64)
    with pytest.raises(TypeError):
        F().flashmlp_fwd(x, w1, w2, "")
    x, w1, w2, do = make_inputs(1, 64, 192, 64, torch.float32)  # fp32 needs D <= 128
    with pytest.raises(F().FlashMLPError, match="hidden dim"):
        F().flashmlp_fwd(x, w1, w2, "")
    with pytest.raises(F().FlashMLPError, match="hidden dim"):
        F().flashmlp_bwd(x, w1, w2, do, "")


def test_misaligned_pointer_rejected():
    from flashmlp_b200 import _lib
    import ctypes

    x, w1, w2, _ = make_inputs(1, 64, 64, 64, torch.bfloat16)
    o = torch.empty(1 * 64 * 64 + 8, dtype=torch.bfloat16, device="cuda")
    rc = _lib.lib().fmlp_fwd(ctypes.c_void_p(x.data_ptr() + 2), ctypes.c_void_p(w1.data_ptr()),
                             ctypes.c_void_p(w2.data_ptr()), ctypes.c_void_p(o.data_ptr()),
                             1, 64, 64, 64, 1, 0, None)
    assert rc == 5  # FMLP_ERR_MISALIGNED


def test_outputs_stay_inside_their_allocation():
    # NaN guard regions before and after every output: a store outside the tensor's
    # extent (the reference's B/E tail bug class) would overwrite a sentinel.
    from flashmlp_b200 import _lib
    import ctypes

    H, B, D, E = 3, 200, 96, 200
    dt = torch.bfloat16
    x, w1, w2, do = make_inputs(H, B, D, E, dt, seed=2)
    G = 4096

    def guarded(n):
        buf = torch.full((n + 2 * G,), float("nan"), dtype=dt, device="cuda")
        return buf, buf[G:G + n]

    L = _lib.lib()
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    ob, o = guarded(H * B * D)
    assert L.fmlp_fwd(p(x), p(w1), p(w2), p(o), H, B, D, E, 1, 2, None) == 0
    bx, dx = guarded(H * B * D)
    b1, dw1 = guarded(H * D * E)
    b2, dw2 = guarded(H * E * D)
    assert L.fmlp_bwd(p(x), p(w1), p(w2), p(do), p(dx), p(dw1), p(dw2), None, 0, H, B, D, E, 1, 3, None) == 0
    torch.cuda.synchronize()
    for buf, inner in ((ob, o), (bx, dx), (b1, dw1), (b2, dw2)):
        assert torch.isnan(buf[:G]).all() and torch.isnan(buf[-G:]).all()
        assert torch.isfinite(inner).all()
