"""Host logic of the multi-GPU wrappers, run as world_size-2 gloo process groups on CPU.
Compute is the CPU oracle (injected), so these tests check sharding, the collective and
the update bookkeeping, not the kernels."""
import datetime
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flashmlp_b200 import sharding
from oracle import flashmlp_oracle as orc


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_compute(dtype="f16"):
    def fwd(x, w1, w2, a):
        return torch.from_numpy(orc.fwd_kernel(x.numpy(), w1.numpy(), w2.numpy(), a, dtype))

    def bwd(x, w1, w2, do, a):
        return tuple(torch.from_numpy(v) for v in orc.bwd_kernel(x.numpy(), w1.numpy(), w2.numpy(), do.numpy(), a, dtype))

    def update(w, g, lr):
        w.sub_(lr * g.view_as(w))

    return sharding.Compute(fwd=fwd, bwd=bwd, update=update)


def _worker(rank, world, port, fn, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=20))
        q.put((rank, "ok", fn(rank, world)))
    except Exception:  # report to the parent instead of hanging it
        q.put((rank, "err", traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def run_ranks(fn, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fn, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        rank, status, payload = q.get(timeout=timeout)
        out[rank] = (status, payload)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return out


def _inputs():
    return orc.make_inputs(5, 37, 16, 24, "f16", seed=21)


def _head_case(rank, world):
    x, w1, w2, do = (torch.from_numpy(a) for a in _inputs())
    parts = [sharding.shard_heads(t, world, rank) for t in (x, w1, w2, do)]
    o, dx, dw1, dw2 = sharding.head_sharded_fwd_bwd(*parts, activation="silu", compute=_oracle_compute())
    return [sharding.gather_heads(v).numpy() for v in (o, dx, dw1, dw2)]


def _batch_case(rank, world):
    x, w1, w2, do = (torch.from_numpy(a) for a in _inputs())
    xl, dol = sharding.shard_batch(x, world, rank), sharding.shard_batch(do, world, rank)
    w1c, w2c = w1.clone(), w2.clone()
    o, dx, g1, g2 = sharding.batch_sharded_train_step(xl, dol, w1c, w2c, activation="sigmoid", lr=0.5,
                                                      compute=_oracle_compute())
    return w1c.numpy(), w2c.numpy(), g1.numpy(), g2.numpy()


def _dead_rank_case(rank, world):
    if rank == 1:
        raise RuntimeError("rank 1 fails before the collective")
    return _batch_case(rank, world)


def test_shard_range_partitions():
    for n in (0, 1, 5, 32, 131072):
        for world in (1, 2, 3, 8):
            spans = [sharding.shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(b - a for a, b in spans) - min(b - a for a, b in spans) <= 1
    with pytest.raises(ValueError):
        sharding.shard_range(4, 2, 2)


def test_head_sharded_equals_single_process():
    res = run_ranks(_head_case)
    x, w1, w2, do = _inputs()
    want = [orc.fwd_kernel(x, w1, w2, "silu", "f16"), *orc.bwd_kernel(x, w1, w2, do, "silu", "f16")]
    for rank in (0, 1):
        status, got = res[rank]
        assert status == "ok", got
        for a, b in zip(got, want):
            assert np.array_equal(a, b)


def test_batch_sharded_step_equals_full_batch_step():
    res = run_ranks(_batch_case)
    x, w1, w2, do = _inputs()
    _, dw1, dw2 = orc.bwd_kernel(x, w1, w2, do, "sigmoid", "f16")
    assert res[0][0] == "ok" and res[1][0] == "ok", res
    (a1, a2, g1, g2), (b1, b2, _, _) = res[0][1], res[1][1]
    # replicas stay identical after the step
    assert np.array_equal(a1, b1) and np.array_equal(a2, b2)
    # the all-reduced gradient equals the full-batch gradient up to the per-shard rounding
    np.testing.assert_allclose(g1, dw1, atol=5e-3, rtol=5e-3)
    np.testing.assert_allclose(g2, dw2, atol=5e-3, rtol=5e-3)
    np.testing.assert_allclose(a1, w1 - 0.5 * g1, rtol=1e-6, atol=1e-6)


def test_dead_rank_surfaces_as_error_not_hang():
    res = run_ranks(_dead_rank_case, timeout=90)
    assert res[1][0] == "err" and "fails before the collective" in res[1][1]
    assert res[0][0] == "err"  # the survivor's all-reduce fails (peer gone / timeout)
