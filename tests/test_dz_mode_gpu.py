"""The dZ-store mode of the unified backward (16-bit inputs with D <= 256, fp32 inputs with
D <= 128).

With the workspace fmlp_bwd_workspace_size asks for, the dW programs also store their
rounded dZ^T tiles and dX is a GEMM over E of those tiles (fmlp_dx_gemm_kernel) instead of
dX programs that recompute Z and dH. The dZ values are the ones the reference's dX
programs form and round (flashmlp.py:212-235), so the results must meet the same parity
bar as the recompute mode:

* against the CPU oracle on seeded ragged shapes (B and E not multiples of the 128-wide
  tiles, D below the padded 64/128), every activation, bf16 and fp16, and against a
  plain PyTorch fp32 reference with magnitude bounds on longer batches;
* against the recompute mode (the low-memory path) on the same inputs: dX within the
  parity tolerance, dW bit-identical when both modes split the dW programs alike (for
  128 < D <= 256 that covers the D-half-1 GEMM over the stored dZ^T and H^T tiles, which
  must give the bits of the recompute mode's D-half-1 programs);
* with split dW programs (few heads, many B tiles) and with a shared (2-D) input;
* at the C4 per-GPU size of 8-way head sharding against a plain PyTorch fp32 reference;
* the workspace region past the dZ^T tiles and the outputs' neighbours are not written;
* heads that do not fit one launch's dZ^T cap (8 GiB), or a caller's workspace limit, run
  in head groups that reuse the workspace, with the one-launch results.
"""
import numpy as np
import pytest
import torch

from _refcheck import assert_close, make_inputs, ref_bwd, tol_for, to_np

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


def _code(dt):
    from flashmlp_b200 import _lib
    return {torch.bfloat16: _lib.FMLP_DTYPE_BF16, torch.float16: _lib.FMLP_DTYPE_F16,
            torch.float32: _lib.FMLP_DTYPE_F32}[dt]


def _plan(H, B, D, E, dt, low_memory=False):
    from flashmlp_b200 import _lib
    L = _lib.lib()
    ws = (L.fmlp_bwd_workspace_size_min if low_memory else L.fmlp_bwd_workspace_size)(H, B, D, E, _code(dt))
    return _lib.bwd_plan(H, B, D, E, _code(dt), int(ws))


@pytest.mark.parametrize("shape,dtype", [((2, 200, 64, 136), "bf16"), ((3, 300, 128, 264), "f16"),
                                         ((1, 257, 96, 200), "bf16"), ((5, 130, 112, 1032), "bf16"),
                                         ((2, 130, 256, 136), "f16"), ((1, 200, 192, 264), "bf16")])
def test_dz_mode_vs_oracle(shape, dtype):
    from oracle import flashmlp_oracle as orc

    H, B, D, E = shape
    dt = {"bf16": torch.bfloat16, "f16": torch.float16}[dtype]
    assert _plan(H, B, D, E, dt)[0] == 1, "the default workspace selects the dZ-store mode"
    xs = orc.make_inputs(H, B, D, E, dtype, seed=3 * B + E)
    x, w1, w2, do = (torch.from_numpy(a).to(dt).cuda() for a in xs)
    atol, rtol = tol_for(dt, "bwd")
    for act in ACTS:
        got = [to_np(t) for t in F().flashmlp_bwd(x, w1, w2, do, act)]
        want = orc.bwd_kernel(*xs, act, dtype)
        for name, a, r in zip(("dx", "dw1", "dw2"), got, want):
            np.testing.assert_allclose(a, r, atol=atol, rtol=rtol, err_msg=f"{shape} {act} {name}")


@pytest.mark.parametrize("shape,dtype", [((2, 1000, 96, 200), torch.bfloat16), ((1, 2048, 128, 256), torch.float16),
                                         ((2, 4096, 16, 136), torch.bfloat16), ((2, 1000, 256, 520), torch.float16)])
def test_dz_mode_vs_torch_fp32_longer_batches(shape, dtype):
    # Over long batches dW sums many H / dZ values whose 16-bit rounding may flip against
    # an exact-activation oracle; the bound of the fp32 reference scales with that sum.
    H, B, D, E = shape
    assert _plan(H, B, D, E, dtype)[0] == 1
    x, w1, w2, do = make_inputs(H, B, D, E, dtype, seed=3 * B + E)
    for act in ACTS:
        got = F().flashmlp_bwd(x, w1, w2, do, act)
        refs = ref_bwd(x, w1, w2, do, act)
        for i, k in enumerate(("dx", "dw1", "dw2")):
            assert_close(got[i], *refs[k], dtype, "bwd", f"{shape} {act} {k}")


@pytest.mark.parametrize("shape,dtype", [((8, 8192, 128, 1024), torch.bfloat16), ((6, 3000, 64, 520), torch.float16),
                                         ((3, 4096, 256, 512), torch.float16), ((6, 256, 256, 1024), torch.bfloat16),
                                         ((2, 200, 192, 264), torch.float16)])
def test_dz_mode_matches_recompute_mode(shape, dtype):
    H, B, D, E = shape
    fast, slow = _plan(H, B, D, E, dtype), _plan(H, B, D, E, dtype, low_memory=True)
    assert fast[0] == 1 and slow[0] == 0
    x, w1, w2, do = make_inputs(H, B, D, E, dtype, seed=H + B)
    for act in ACTS:
        a = F().flashmlp_bwd(x, w1, w2, do, act)
        with F().low_memory_backward():
            b = F().flashmlp_bwd(x, w1, w2, do, act)
        refs = ref_bwd(x, w1, w2, do, act)
        for i, k in enumerate(("dx", "dw1", "dw2")):
            assert_close(a[i], b[i].float(), refs[k][1], dtype, "bwd", f"{act} {k} dz vs recompute")
            assert_close(a[i], *refs[k], dtype, "bwd", f"{act} {k}")
        if fast[1] == slow[1]:  # same dW split: the dW programs did the same arithmetic
            assert torch.equal(a[1], b[1]) and torch.equal(a[2], b[2])
        # deterministic: a second call repeats every bit
        c = F().flashmlp_bwd(x, w1, w2, do, act)
        for u, v in zip(a, c):
            assert torch.equal(u, v)


def test_dz_mode_split_dw_c4_per_gpu_at_8():
    # 4 heads of C4 (the per-GPU launch of 8-way head sharding): 64 (head, E chunk) pairs
    # on 148 SMs, so the dZ-store launch splits its dW programs and reduces the partials.
    H, B, D, E = 4, 65536, 128, 2048
    dt = torch.bfloat16
    mode, splits, launches = _plan(H, B, D, E, dt)
    assert mode == 1 and splits > 1 and launches == 3
    x, w1, w2, do = make_inputs(H, B, D, E, dt, seed=8)
    got = F().flashmlp_bwd(x, w1, w2, do, "silu")
    refs = ref_bwd(x, w1, w2, do, "silu")
    for i, k in enumerate(("dx", "dw1", "dw2")):
        assert_close(got[i], *refs[k], dt, "bwd", k)
    dxf, dwf = F().flashmlp_bwd_dw_f32(x, w1, w2, do, "silu")
    n1 = H * D * E
    assert torch.equal(dxf, got[0])
    assert torch.equal(dwf[:n1].view(H, D, E).to(dt), got[1])
    assert torch.equal(dwf[n1:].view(H, E, D).to(dt), got[2])


def test_dz_mode_split_dw_d256():
    # 128 < D <= 256: the dW programs of D half 0 store dZ^T and H^T, a GEMM over B forms D
    # half 1 from them; with few heads both split over B ranges (fp32 partials, ordered
    # reduce): dW programs, D-half-1 GEMM, dX GEMM, reduce.
    H, B, D, E = 2, 16384, 256, 1024
    dt = torch.float16
    mode, splits, launches = _plan(H, B, D, E, dt)
    assert mode == 1 and splits > 1 and launches == 4
    x, w1, w2, do = make_inputs(H, B, D, E, dt, seed=21)
    got = F().flashmlp_bwd(x, w1, w2, do, "sigmoid")
    refs = ref_bwd(x, w1, w2, do, "sigmoid")
    for i, k in enumerate(("dx", "dw1", "dw2")):
        assert_close(got[i], *refs[k], dt, "bwd", f"d256 split {k}")
    with F().low_memory_backward():  # recompute mode: one dW program per (head, chunk, half)
        slow = F().flashmlp_bwd(x, w1, w2, do, "sigmoid")
    assert torch.equal(got[0], slow[0])  # dX: the same dZ, the same GEMM order
    dxf, dwf = F().flashmlp_bwd_dw_f32(x, w1, w2, do, "sigmoid")
    n1 = H * D * E
    assert torch.equal(dxf, got[0])
    assert torch.equal(dwf[:n1].view(H, D, E).to(dt), got[1])
    assert torch.equal(dwf[n1:].view(H, E, D).to(dt), got[2])


def test_dz_mode_shared_input():
    # 2-D input: dZ^T of every head already carries the head mean's 1/H; the dX GEMM sums
    # over (head, e). Checked against the backward of the explicitly expanded input.
    H, B, D, E = 3, 1500, 128, 392
    dt = torch.bfloat16
    g = torch.Generator().manual_seed(17)
    x = torch.randn(B, D, generator=g).to(dt).cuda()
    w1 = (torch.randn(H, D, E, generator=g) / D ** 0.5).to(dt).cuda()
    w2 = (torch.randn(H, E, D, generator=g) / E ** 0.5).to(dt).cuda()
    do = torch.randn(B, D, generator=g).to(dt).cuda()
    assert _plan(H, B, D, E, dt)[0] == 1
    for act in ("silu", "sigmoid"):
        dx, dw1, dw2 = F().flashmlp_bwd_shared_x(x, w1, w2, do, act)
        with F().low_memory_backward():
            dx0, dw10, dw20 = F().flashmlp_bwd_shared_x(x, w1, w2, do, act)
        xe = x.unsqueeze(0).expand(H, B, D)
        refs = ref_bwd(xe, w1, w2, (do.float() / H).unsqueeze(0).expand(H, B, D), act)
        assert_close(dx, refs["dx"][0].sum(0), refs["dx"][1].sum(0), dt, "bwd", f"{act} dx")
        assert_close(dx, dx0.float(), refs["dx"][1].sum(0), dt, "bwd", f"{act} dx vs recompute")
        assert_close(dw1, *refs["dw1"], dt, "bwd", f"{act} dw1")
        assert_close(dw2, *refs["dw2"], dt, "bwd", f"{act} dw2")


def test_dz_mode_writes_stay_inside_their_buffers():
    # Guard regions around every output and past the dZ^T / partial-sum workspace keep
    # their sentinel after a dZ-store call through the C ABI.
    import ctypes
    from flashmlp_b200 import _lib

    H, B, D, E = 2, 1000, 96, 200
    dt = torch.bfloat16
    L = _lib.lib()
    need = int(L.fmlp_bwd_workspace_size(H, B, D, E, 1))
    assert _lib.bwd_plan(H, B, D, E, 1, need)[0] == 1
    x, w1, w2, do = make_inputs(H, B, D, E, dt, seed=4)
    G = 4096  # guard elements on each side
    bufs = [torch.full((t.numel() + 2 * G,), 7.0, dtype=dt, device="cuda") for t in (x, w1, w2)]
    ws = torch.full((need + 2 * 4096,), 0x5A, dtype=torch.uint8, device="cuda")
    p = lambda t, off=0: ctypes.c_void_p(t.data_ptr() + off)
    rc = L.fmlp_bwd(p(x), p(w1), p(w2), p(do), *(p(b, 2 * G) for b in bufs), p(ws, 4096), need, H, B, D, E, 1,
                    2, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, _lib.error_string(rc)
    torch.cuda.synchronize()
    for b in bufs:
        assert bool((b[:G] == 7.0).all()) and bool((b[-G:] == 7.0).all())
    assert bool((ws[:4096] == 0x5A).all()) and bool((ws[-4096:] == 0x5A).all())
    want = F().flashmlp_bwd(x, w1, w2, do, "silu")
    for b, w in zip(bufs, want):
        assert torch.equal(b[G:-G].view_as(w), w)


def test_dz_mode_runs_in_head_groups_above_8_gib():
    # C4 on one GPU needs exactly 8 GiB of dZ^T (the cap of one launch: every element
    # offset fits in 32 bits). One more head no longer falls back to the recompute mode:
    # the heads run in two groups of 17 and 16 that reuse one workspace. Plan queries
    # only, nothing is allocated.
    from flashmlp_b200 import _lib

    L = _lib.lib()
    B, D, E = 65536, 128, 2048
    assert _plan(32, B, D, E, torch.bfloat16) == (1, 2, 3)
    assert int(L.fmlp_bwd_workspace_size(32, B, D, E, 1)) >= 8 << 30
    mode, splits, launches = _plan(33, B, D, E, torch.bfloat16)
    assert mode == 1 and launches == 2 * (2 + (splits > 1))
    ws33 = int(L.fmlp_bwd_workspace_size(33, B, D, E, 1))
    assert (17 << 28) <= ws33 < (8 << 30), "the workspace of the 17-head group"
    # a smaller workspace gives smaller groups; below 4 heads' tiles, the recompute mode
    per_head = 2 * E * B
    mode, _, launches = _lib.bwd_plan(32, B, D, E, 1, 8 * per_head + (64 << 20))
    assert mode == 1 and launches >= 4 * 2
    mode, _, _ = _lib.bwd_plan(32, B, D, E, 1, 3 * per_head + (64 << 20))
    assert mode == 0
    # below fmlp_bwd_workspace_size_min the plan (and fmlp_bwd) refuse the call
    need = int(L.fmlp_bwd_workspace_size_min(4, B, D, E, 1))
    assert need > 0
    with pytest.raises(_lib.FlashMLPError):
        _lib.bwd_plan(4, B, D, E, 1, need - 16)


@pytest.mark.parametrize("dt,D", [(torch.bfloat16, 128), (torch.float32, 128), (torch.float16, 256)])
def test_dz_mode_head_groups_match_one_launch(dt, D):
    # A workspace limit that holds 4 of 6 heads' dZ tiles: the dZ-store mode runs in head
    # groups (fmlp_bwd_plan counts their launches). dX comes from the same dZ tiles and
    # the same GEMM per head, so it is bit-identical to the one-launch result; dW too when
    # the groups split their dW programs as the one launch does; all of it within the
    # parity bar of the fp32 reference. At D = 256 the groups also reuse the H^T region
    # of the workspace for the D-half-1 GEMM.
    from flashmlp_b200 import _lib

    H, B, E = 6, 4096, 1024
    code = _code(dt)
    L = _lib.lib()
    full = int(L.fmlp_bwd_workspace_size(H, B, D, E, code))
    limit = int(L.fmlp_bwd_workspace_size(4, B, D, E, code))
    one = _lib.bwd_plan(H, B, D, E, code, full)
    grouped = _lib.bwd_plan(H, B, D, E, code, limit)
    assert one[0] == 1 and grouped[0] == 1 and grouped[2] >= 2 * one[2], (one, grouped)
    x, w1, w2, do = make_inputs(H, B, D, E, dt, seed=77)
    a = F().flashmlp_bwd(x, w1, w2, do, "silu")
    with F().backward_workspace_limit(limit):
        b = F().flashmlp_bwd(x, w1, w2, do, "silu")
    refs = ref_bwd(x, w1, w2, do, "silu")
    assert torch.equal(a[0], b[0]), "dX of the grouped launches differs from one launch"
    for i, k in enumerate(("dx", "dw1", "dw2")):
        assert_close(b[i], *refs[k], dt, "bwd", f"grouped {k}")
        assert_close(b[i], a[i].float(), refs[k][1], dt, "bwd", f"grouped vs one launch {k}")
    if grouped[1] == one[1]:
        assert torch.equal(a[1], b[1]) and torch.equal(a[2], b[2])


@pytest.mark.parametrize("shape", [(2, 300, 64, 136), (3, 1000, 128, 264), (4, 65536, 128, 2048)])
def test_dz_mode_fp32_tf32(shape):
    # fp32 inputs: the TF32 dW programs (split over B ranges when few) store dZ (fp32,
    # (H, B, E) with e contiguous) and a TF32 GEMM forms dX from it.
    H, B, D, E = shape
    dt = torch.float32
    fast, slow = _plan(H, B, D, E, dt), _plan(H, B, D, E, dt, low_memory=True)
    assert fast[0] == 1 and slow[0] == 0
    x, w1, w2, do = make_inputs(H, B, D, E, dt, seed=B + D)
    acts = ACTS if B < 10000 else ["silu"]
    for act in acts:
        a = F().flashmlp_bwd(x, w1, w2, do, act)
        with F().low_memory_backward():
            b = F().flashmlp_bwd(x, w1, w2, do, act)
        refs = ref_bwd(x, w1, w2, do, act)
        for i, k in enumerate(("dx", "dw1", "dw2")):
            assert_close(a[i], *refs[k], dt, "bwd", f"{shape} {act} {k}")
            assert_close(a[i], b[i], refs[k][1], dt, "bwd", f"{shape} {act} {k} dz vs recompute")
        if fast[1] == slow[1]:
            assert torch.equal(a[1], b[1]) and torch.equal(a[2], b[2])
        c = F().flashmlp_bwd(x, w1, w2, do, act)
        for u, v in zip(a, c):
            assert torch.equal(u, v)
