"""Failure detection on the GPU without a fault: a bounded wait that runs out.

The fused all-reduce + SGD (fmlp_grad_allreduce_sgd) waits on flags that the other ranks
write into this rank's memory. Here one process plays rank 0 of a world of 2 on one GPU;
"rank 1's" buffers are ordinary local allocations and nothing ever sets rank 1's slot in
rank 0's flag array, as if rank 1 had died before the collective. The barrier must give
up after its wait limit (2 s), record FMLP_ERR_DEVICE_TIMEOUT in the status word that
fmlp_device_status returns, skip the reduction (the weights stay untouched), and leave the
context usable: a forward afterwards still matches the plain PyTorch reference.
Nothing here traps, faults or hangs the GPU; the wait is the kernel's own bounded spin.
"""
import ctypes
import time

import pytest
import torch

from _refcheck import assert_close, make_inputs, ref_fwd

pytestmark = pytest.mark.gpu


def test_allreduce_barrier_times_out_when_a_rank_never_arrives():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import flashmlp_b200 as F
    from flashmlp_b200 import _lib

    L = _lib.lib()
    assert L.fmlp_device_status(1) == 0, "status word not clean before the test"
    n = 4096
    dev = torch.device("cuda")
    w = [torch.full((n,), 0.5, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    g = [torch.ones(n, dtype=torch.float32, device=dev) for _ in range(2)]
    flags = [torch.zeros(8, dtype=torch.int32, device=dev) for _ in range(2)]
    arr = lambda ts: (ctypes.c_void_p * 2)(*[ctypes.c_void_p(t.data_ptr()) for t in ts])
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.fmlp_grad_allreduce_sgd(arr(w), arr(g), arr(flags), 2, 0, n, 0.1, _lib.FMLP_DTYPE_BF16, 1, stream)
    assert rc == 0, _lib.error_string(rc)
    t0 = time.time()
    st = L.fmlp_device_status(1)  # synchronises, reads and clears the status word
    waited = time.time() - t0
    assert st == _lib.FMLP_ERR_DEVICE_TIMEOUT
    assert 1.5 < waited < 60, f"barrier gave up after {waited:.2f} s"
    # rank 0 published its epochs into both flag arrays, rank 1's slot stayed 0
    assert flags[0][0].item() == 2 and flags[1][0].item() == 2 and flags[0][1].item() == 0
    # the timed-out barrier stopped the reduction: no replica was written
    for t in w:
        assert bool((t == 0.5).all())
    assert L.fmlp_device_status(1) == 0
    # the context is still usable
    x, w1, w2, _ = make_inputs(2, 300, 64, 136, torch.bfloat16, seed=3)
    o = F.flashmlp_fwd(x, w1, w2, "silu")
    assert_close(o, *ref_fwd(x, w1, w2, "silu"), torch.bfloat16, "fwd", "after timeout")
    assert L.fmlp_device_status(1) == 0
