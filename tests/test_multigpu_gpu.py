"""Multi-GPU wrappers on real GPUs: two NCCL ranks, one per GPU (skipped with fewer).

Head sharding must reproduce the single-GPU result bit for bit (heads are independent and
the kernels are deterministic). The batch-sharded training step must give every rank the
same gradients, equal to the fp32 sum of the per-rank partial gradients, and
bit-identical updated weights. Against the full-batch gradient of one launch the sum
agrees within the 16-bit rounding of the partials (each rank rounds its dW to the input
dtype before the all-reduce), a bound that also covers near-cancelling sums."""
import datetime
import os
import socket
import traceback

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(H, B, D, E, dtype, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(H, B, D, generator=g).to(dtype)
    w1 = (torch.randn(H, D, E, generator=g) / D ** 0.5).to(dtype)
    w2 = (torch.randn(H, E, D, generator=g) / E ** 0.5).to(dtype)
    do = torch.randn(H, B, D, generator=g).to(dtype)
    return x, w1, w2, do


def _head_case(rank, world):
    import flashmlp_b200 as F
    from flashmlp_b200 import sharding

    dev = torch.device("cuda", rank)
    x, w1, w2, do = (t.to(dev) for t in _inputs(6, 1000, 128, 640, torch.bfloat16))
    loc = [sharding.shard_heads(t, world, rank) for t in (x, w1, w2, do)]
    outs = sharding.head_sharded_fwd_bwd(*loc, activation="silu")
    full = [sharding.gather_heads(t) for t in outs]
    ref = [F.flashmlp_fwd(x, w1, w2, "silu"), *F.flashmlp_bwd(x, w1, w2, do, "silu")]
    torch.cuda.synchronize()
    return [bool(torch.equal(a, b)) for a, b in zip(full, ref)]


def _batch_case(rank, world):
    import torch.distributed as dist

    import flashmlp_b200 as F
    from flashmlp_b200 import sharding

    dev = torch.device("cuda", rank)
    x, w1, w2, do = (t.to(dev) for t in _inputs(4, 2048, 128, 512, torch.bfloat16, seed=1))
    xl, dol = sharding.shard_batch(x, world, rank), sharding.shard_batch(do, world, rank)
    w1r, w2r = w1.clone(), w2.clone()
    _, _, g1, g2 = sharding.batch_sharded_train_step(xl, dol, w1r, w2r, "sigmoid", lr=0.05)
    _, ref1, ref2 = F.flashmlp_bwd(x, w1, w2, do, "sigmoid")
    # this rank's partial gradients (the kernels are deterministic: same as inside the step)
    _, p1, p2 = F.flashmlp_bwd(xl, w1, w2, dol, "sigmoid")

    def check(g, p, ref):
        parts = [torch.empty_like(p) for _ in range(world)]
        dist.all_gather(parts, p)
        exact = torch.equal(g, sum(t.float() for t in parts))  # two fp32 terms: order-free
        # each partial and the reference carry one bf16 rounding (<= 2^-9 relative)
        bound = 2.0 ** -8 * (sum(t.float().abs() for t in parts) + ref.float().abs()) + 1e-3
        return exact and bool(((g - ref.float()).abs() <= bound).all())

    e1 = 0 if check(g1, p1, ref1) else 1
    e2 = 0 if check(g2, p2, ref2) else 1
    # every rank must hold the same weights after the update
    ws = torch.cat([w1r.reshape(-1), w2r.reshape(-1)]).float()
    gathered = [torch.empty_like(ws) for _ in range(world)]
    dist.all_gather(gathered, ws)
    same = all(torch.equal(gathered[0], t) for t in gathered[1:])
    moved = not torch.equal(w1r, w1)
    torch.cuda.synchronize()
    return e1 <= 0, e2 <= 0, same, moved


def _fused_case(rank, world):
    """Two steps of the fused batch-sharded trainer against the same arithmetic done with
    NCCL: fp32 partial gradients summed in rank order, then w - lr * g rounded once."""
    import torch.distributed as dist

    import flashmlp_b200 as F
    from flashmlp_b200 import sharding

    dev = torch.device("cuda", rank)
    results = []
    for (H, B, D, E, dt, act) in ((4, 2048, 128, 512, torch.bfloat16, "silu"),
                                  (2, 1000, 256, 264, torch.float16, "sigmoid")):
        x, w1, w2, do = (t.to(dev) for t in _inputs(H, B, D, E, dt, seed=5))
        xl, dol = sharding.shard_batch(x, world, rank), sharding.shard_batch(do, world, rank)
        tr = sharding.FusedBatchShardedTrainer(w1, w2)
        rw1, rw2 = w1.clone(), w2.clone()
        ok = True
        for step, lr in enumerate((0.05, 0.02)):
            # reference arithmetic on this rank, with NCCL moving the partials
            ro = F.flashmlp_fwd(xl, rw1, rw2, act)
            rdx, part = F.flashmlp_bwd_dw_f32(xl, rw1, rw2, dol, act)
            parts = [torch.empty_like(part) for _ in range(world)]
            dist.all_gather(parts, part)
            g = parts[0].clone()
            for p_ in parts[1:]:
                g += p_
            n1 = rw1.numel()
            rw1 = (rw1.float() - lr * g[:n1].view(rw1.shape)).to(dt)
            rw2 = (rw2.float() - lr * g[n1:].view(rw2.shape)).to(dt)
            o, dx = tr.step(xl, dol, act, lr)
            torch.cuda.synchronize()
            ok &= torch.equal(o, ro) and torch.equal(dx, rdx)
            ok &= torch.equal(tr.w1, rw1) and torch.equal(tr.w2, rw2)
            ws = torch.cat([tr.w1.reshape(-1), tr.w2.reshape(-1)]).float()
            gathered = [torch.empty_like(ws) for _ in range(world)]
            dist.all_gather(gathered, ws)
            ok &= all(torch.equal(gathered[0], t) for t in gathered[1:])
        ok &= not torch.equal(tr.w1, w1)
        ok &= tr.status() == 0
        ok &= F._lib.lib().fmlp_device_status(1) == 0
        tr.close()
        results.append(bool(ok))
    return results


def _worker(rank, world, port, case, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch.distributed as dist

    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                                timeout=datetime.timedelta(seconds=60))
        q.put((rank, "ok", case(rank, world)))
    except Exception:
        q.put((rank, "err", traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _run(case, world=2, timeout=240):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            rank, status, val = q.get(timeout=timeout)
            assert status == "ok", f"rank {rank} failed:\n{val}"
            out[rank] = val
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return out


def _need_two():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")


def test_head_sharded_matches_single_gpu_bitwise():
    _need_two()
    out = _run(_head_case)
    for rank, flags in out.items():
        assert all(flags), f"rank {rank}: (o, dx, dw1, dw2) equal = {flags}"


def test_batch_sharded_step_gradients_and_replicas():
    _need_two()
    out = _run(_batch_case)
    for rank, (ok1, ok2, same, moved) in out.items():
        assert ok1 and ok2, f"rank {rank}: summed gradients outside tolerance (dw1 {ok1}, dw2 {ok2})"
        assert same, f"rank {rank}: replicas differ after the update"
        assert moved, f"rank {rank}: weights not updated"


def test_fused_allreduce_sgd_trainer_two_steps():
    # fmlp_grad_allreduce_sgd over NVLink peer memory: replicas bit-identical and equal to
    # the fixed-order fp32 sum of the ranks' partial gradients followed by the SGD step
    _need_two()
    out = _run(_fused_case)
    for rank, flags in out.items():
        assert all(flags), f"rank {rank}: (bf16 D=128, fp16 D=256) cases ok = {flags}"
