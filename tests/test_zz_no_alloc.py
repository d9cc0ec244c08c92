"""fmlp_bwd_noalloc: the backward entry point for callers that cannot allocate device memory.

Engines that plan all device memory themselves hand a custom operator only its inputs and
outputs, so the operator cannot cudaMalloc the fp32 workspace fmlp_bwd needs when it
splits its dW programs over batch ranges. fmlp_bwd_noalloc keeps that scratch in a static
device array inside the library instead. This test calls it through the C ABI on a shape
that uses the scratch (16-bit inputs and fp32 inputs, whose TF32 dW programs split too),
twice in a row with different inputs (the array keeps the first call's partial sums,
which the second call must not pick up), and checks each result against the fp32 PyTorch
reference with the kernels' rounding points (tests/_refcheck.py) and against fmlp_bwd's
result, both within the parity tolerance of the other GPU tests.

The file name sorts last so that a run stopping at the first failure has already run
every other test.
"""
import ctypes

import pytest
import torch

from _refcheck import assert_close, make_inputs, ref_bwd

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_bwd_noalloc_matches_bwd_on_two_calls_in_a_row(dtype):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import flashmlp_b200 as F
    from flashmlp_b200 import _lib

    L = _lib.lib()
    H, B, D, E = 4, 4096, 128, 1024
    dt = {"bf16": torch.bfloat16, "f32": torch.float32}[dtype]
    code = {"bf16": _lib.FMLP_DTYPE_BF16, "f32": _lib.FMLP_DTYPE_F32}[dtype]
    need = int(L.fmlp_bwd_workspace_size_min(H, B, D, E, code))
    assert 0 < need <= (32 << 20), "shape chosen so that the backward uses scratch memory"
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    for seed, act in ((31, "silu"), (32, "sigmoid")):
        x, w1, w2, do = make_inputs(H, B, D, E, dt, seed=seed)
        dx, dw1, dw2 = (torch.empty_like(t) for t in (x, w1, w2))
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        rc = L.fmlp_bwd_noalloc(p(x), p(w1), p(w2), p(do), p(dx), p(dw1), p(dw2), H, B, D, E,
                                code, F.activation_code(act), stream)
        assert rc == 0, _lib.error_string(rc)
        want = F.flashmlp_bwd(x, w1, w2, do, act)  # the entry point with a caller workspace
        torch.cuda.synchronize()
        bounds = ref_bwd(x, w1, w2, do, act)
        for name, got, other in zip(("dx", "dw1", "dw2"), (dx, dw1, dw2), want):
            assert_close(got, *bounds[name], dt, "bwd", f"noalloc/{act}/{name} vs fp32 reference")
            assert_close(got, other.float(), bounds[name][1], dt, "bwd", f"noalloc/{act}/{name} vs fmlp_bwd")
    assert L.fmlp_device_status(1) == 0
