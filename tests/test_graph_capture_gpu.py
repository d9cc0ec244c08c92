"""The forward and backward entry points inside a CUDA graph.

A training step is a fixed sequence of launches on fixed shapes; capturing it once in a
CUDA graph (torch.cuda.CUDAGraph) removes the per-call host work (Python checks, tensor-map
encoding, workspace allocation from the caching allocator) from every later step, which
matters for the small BASELINE configs whose kernels take tens of microseconds. The C ABI
only enqueues kernels and memsets on the caller's stream, so the captured step must give,
on new data copied into the captured input buffers, exactly the results of eager calls:
compared bit for bit here, in the dZ-store mode (split and unsplit dW programs), the
recompute mode, the D = 256 kernel and the fp32 (TF32) kernels.
"""
import pytest
import torch

from _refcheck import make_inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import flashmlp_b200  # noqa: F401
    yield
    from flashmlp_b200 import _lib
    assert _lib.lib().fmlp_device_status(1) == 0


@pytest.mark.parametrize("shape,dtype,act,low_memory", [
    ((12, 1024, 64, 768), torch.float16, "silu", False),      # BASELINE C1
    ((2, 4096, 128, 256), torch.bfloat16, "sigmoid", False),  # split dW programs + reduce
    ((3, 1000, 96, 200), torch.bfloat16, "leaky_relu", True),  # recompute mode
    ((2, 700, 256, 264), torch.float16, "silu", False),       # D = 256
    ((2, 4096, 128, 512), torch.float32, "silu", False),      # fp32: TF32 kernels, split dW + dZ-store
])
def test_captured_step_matches_eager(shape, dtype, act, low_memory):
    import contextlib

    import flashmlp_b200 as F

    H, B, D, E = shape
    ctx = F.low_memory_backward if low_memory else contextlib.nullcontext
    x, w1, w2, do = make_inputs(H, B, D, E, dtype, seed=1)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s), ctx():  # warm-up outside the capture (library and device setup)
        F.flashmlp_fwd(x, w1, w2, act)
        F.flashmlp_bwd(x, w1, w2, do, act)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g), ctx():
        o = F.flashmlp_fwd(x, w1, w2, act)
        dx, dw1, dw2 = F.flashmlp_bwd(x, w1, w2, do, act)
    for seed in (7, 8):
        nx, nw1, nw2, ndo = make_inputs(H, B, D, E, dtype, seed=seed)
        for dst, src in zip((x, w1, w2, do), (nx, nw1, nw2, ndo)):
            dst.copy_(src)
        g.replay()
        torch.cuda.synchronize()
        with ctx():
            want = [F.flashmlp_fwd(nx, nw1, nw2, act), *F.flashmlp_bwd(nx, nw1, nw2, ndo, act)]
        for name, got, ref in zip(("o", "dx", "dw1", "dw2"), (o, dx, dw1, dw2), want):
            assert torch.equal(got, ref), f"{shape} {act} {name} differs after replay (seed {seed})"
    del g
