"""Failure detection on the GPU without a fault: bounded waits that run out, and abort
marks written by the host.

The fused all-reduce + SGD (fmlp_grad_allreduce_sgd) waits on flags that the other ranks
write into this rank's memory. Here one process plays one rank of a world of 2 on one GPU;
the other rank's buffers are ordinary local allocations, and the host writes into them
what that rank would have written (or nothing, as if it had died before the collective).
Only the single rank's own kernels run, never two ranks that wait on each other. Checked:

  * a rank that never arrives: the barrier gives up after its wait limit (2 s), the call
    status (word FMLP_PEER_STATUS_WORD of the own flag array) and fmlp_device_status read
    FMLP_ERR_DEVICE_TIMEOUT, the reduction is skipped (weights untouched), the abort mark is
    published to both ranks and no second epoch is, and the context stays usable;
  * the late peer: a rank that arrives after the other gave up finds its abort mark,
    fails at once with FMLP_ERR_PEER_ABORT (no 2 s wait) and writes nothing;
  * a stale timeout bit in the device-wide status word (left by another kernel) does not
    skip a later, healthy reduction;
  * FusedBatchShardedTrainer.step raises when a call fails (single-rank gloo group with an
    abort mark set, as left by an earlier failed call).
Nothing here traps, faults or hangs the GPU; every wait is the kernel's own bounded spin.
"""
import ctypes
import time

import pytest
import torch

from _refcheck import assert_close, make_inputs, ref_fwd

pytestmark = pytest.mark.gpu


def _setup():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from flashmlp_b200 import _lib

    return _lib, _lib.lib()


def _buffers(n, _lib):
    dev = torch.device("cuda")
    w = [torch.full((n,), 0.5, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    g = [torch.ones(n, dtype=torch.float32, device=dev) for _ in range(2)]
    flags = [torch.zeros(_lib.FMLP_PEER_FLAG_WORDS, dtype=torch.int32, device=dev) for _ in range(2)]
    return w, g, flags


def _call(L, _lib, w, g, flags, rank, n, epoch):
    arr = lambda ts: (ctypes.c_void_p * 2)(*[ctypes.c_void_p(t.data_ptr()) for t in ts])
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.fmlp_grad_allreduce_sgd(arr(w), arr(g), arr(flags), 2, rank, n, 0.1, _lib.FMLP_DTYPE_BF16, epoch, stream)
    assert rc == 0, _lib.error_string(rc)


def test_allreduce_barrier_times_out_when_a_rank_never_arrives():
    import flashmlp_b200 as F

    _lib, L = _setup()
    assert L.fmlp_device_status(1) == 0, "status word not clean before the test"
    n = 4096
    w, g, flags = _buffers(n, _lib)
    _call(L, _lib, w, g, flags, 0, n, 1)
    t0 = time.time()
    torch.cuda.synchronize()
    waited = time.time() - t0
    assert 1.5 < waited < 60, f"barrier gave up after {waited:.2f} s"
    S, A = _lib.FMLP_PEER_STATUS_WORD, _lib.FMLP_MAX_PEERS
    assert flags[0][S].item() == _lib.FMLP_ERR_DEVICE_TIMEOUT  # the call's own status
    assert L.fmlp_device_status(1) == _lib.FMLP_ERR_DEVICE_TIMEOUT  # and the device-wide word
    # rank 0 published epoch 1 and then its abort mark into both flag arrays, never epoch 2;
    # rank 1's slots stayed 0
    for f in flags:
        assert f[0].item() == 1 and f[A + 0].item() != 0 and f[1].item() == 0 and f[A + 1].item() == 0
    # the failed barrier stopped the reduction: no replica was written
    for t in w:
        assert bool((t == 0.5).all())
    assert L.fmlp_device_status(1) == 0
    # the context is still usable
    x, w1, w2, _ = make_inputs(2, 300, 64, 136, torch.bfloat16, seed=3)
    o = F.flashmlp_fwd(x, w1, w2, "silu")
    assert_close(o, *ref_fwd(x, w1, w2, "silu"), torch.bfloat16, "fwd", "after timeout")
    assert L.fmlp_device_status(1) == 0


def test_late_peer_sees_the_abort_and_fails_at_once():
    _lib, L = _setup()
    assert L.fmlp_device_status(1) == 0
    n = 4096
    w, g, flags = _buffers(n, _lib)
    S, A = _lib.FMLP_PEER_STATUS_WORD, _lib.FMLP_MAX_PEERS
    # rank 0 arrived (epoch 1 in rank 1's array), then gave up: its abort mark is there too
    flags[1][0] = 1
    flags[1][A + 0] = 1
    torch.cuda.synchronize()
    t0 = time.time()
    _call(L, _lib, w, g, flags, 1, n, 1)  # this process is rank 1, arriving late
    torch.cuda.synchronize()
    assert time.time() - t0 < 1.0, "the late rank waited instead of failing at once"
    assert flags[1][S].item() == _lib.FMLP_ERR_PEER_ABORT
    assert flags[0][A + 1].item() != 0 and flags[1][A + 1].item() != 0  # its own mark, everywhere
    assert flags[0][1].item() == 0, "a rank that failed published an epoch"
    for t in w:
        assert bool((t == 0.5).all())
    assert L.fmlp_device_status(1) == 0  # an abort is not a timeout of this device


def test_stale_device_timeout_bit_does_not_skip_a_later_reduction():
    _lib, L = _setup()
    assert L.fmlp_device_status(1) == 0
    n = 4096
    # leave FMLP_ERR_DEVICE_TIMEOUT in the device-wide word (a barrier nobody answers)
    w, g, flags = _buffers(n, _lib)
    _call(L, _lib, w, g, flags, 0, n, 1)
    torch.cuda.synchronize()  # not fmlp_device_status: the bit stays set
    # a fresh, healthy group: rank 1 has already published both epochs of the call
    w, g, flags = _buffers(n, _lib)
    flags[0][1] = 4
    torch.cuda.synchronize()
    _call(L, _lib, w, g, flags, 0, n, 3)
    torch.cuda.synchronize()
    assert flags[0][_lib.FMLP_PEER_STATUS_WORD].item() == 0
    # rank 0 owns the first half of the 4-element groups: 0.5 - 0.1 * (1 + 1) there, in both replicas
    want = torch.tensor(0.5 - 0.1 * 2.0).to(torch.bfloat16)
    for t in w:
        assert bool((t[: n // 2] == want).all()) and bool((t[n // 2:] == 0.5).all())
    assert L.fmlp_device_status(1) == _lib.FMLP_ERR_DEVICE_TIMEOUT  # the stale bit, reported
    assert L.fmlp_device_status(1) == 0


def test_trainer_step_raises_after_a_failed_call():
    import torch.distributed as dist

    from flashmlp_b200 import FlashMLPError, sharding

    _lib, L = _setup()
    assert L.fmlp_device_status(1) == 0
    dist.init_process_group("gloo", store=dist.HashStore(), rank=0, world_size=1)
    try:
        x, w1, w2, do = make_inputs(2, 256, 64, 128, torch.bfloat16, seed=4)
        tr = sharding.FusedBatchShardedTrainer(w1, w2)
        tr.step(x, do, "silu", 0.01)  # a healthy step passes its check
        assert tr.status() == 0
        before = (tr.w1.clone(), tr.w2.clone())
        tr.flags[_lib.FMLP_MAX_PEERS + 0] = 1  # the abort mark an earlier failed call leaves
        with pytest.raises(FlashMLPError) as e:
            tr.step(x, do, "silu", 0.01)
        assert e.value.code == _lib.FMLP_ERR_PEER_ABORT
        assert torch.equal(tr.w1, before[0]) and torch.equal(tr.w2, before[1])
        tr.close()
    finally:
        dist.destroy_process_group()
    assert L.fmlp_device_status(1) == 0
