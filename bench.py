"""Benchmark of the fused multi-head MLP fwd+bwd (head-sharded).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

For N > 1 launch one process per GPU with torch.distributed.run; heads are split across
ranks (32/N per GPU, no communication) and the time is the max over ranks. One step is
one forward + one unified backward over the rank's heads with the batch B=65536, D=128,
E=2048, bf16, silu. Metric: algorithmic TFLOP/s of fwd+bwd (12*H*B*D*E per step) for
the whole job. Rank 0 prints one JSON line.

--impl reference times the reference's PyTorch path (flashmlp_torch_fwd/bwd, restated in
numpy fp32 by the test oracle, since the reference itself does not travel) on the host
cores with all threads, on a bounded sample of the same workload, on rank 0 only.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

WORKLOAD = dict(H=32, B=65536, D=128, E=2048, activation="silu", dtype="bf16")
WORKLOAD_NAME = "C4 head-sharded fwd+bwd H=32 B=65536 D=128 E=2048 bf16 silu"
METRIC = "fused MLP fwd+bwd TFLOP/s (algorithmic 12*H*B*D*E per step)"
FALLBACK_PEAKS = {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0}
SPEC_BF16_TFLOPS = 2250.0
CPU_SAMPLE_ROWS = 8192  # rows of one head per CPU step (about 26 GFLOP of fwd+bwd)


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return d, "measured"
        except Exception:
            pass
    return FALLBACK_PEAKS, "fallback"


def cpu_threads():
    try:
        from threadpoolctl import threadpool_info

        n = [i.get("num_threads", 0) for i in threadpool_info() if i.get("user_api") == "blas"]
        if n:
            return max(n)
    except Exception:
        pass
    return os.cpu_count() or 1


def cpu_reference_step(inputs):
    """One fwd+bwd of the reference's PyTorch path (flashmlp.py:671-723) on the CPU."""
    from oracle import flashmlp_oracle as orc

    x, w1, w2, do = inputs
    orc.fwd_fp32(x, w1, w2, WORKLOAD["activation"])
    orc.bwd_fp32(x, w1, w2, do, WORKLOAD["activation"])


def cpu_sample_inputs(rows):
    from oracle import flashmlp_oracle as orc

    return orc.make_inputs(1, rows, WORKLOAD["D"], WORKLOAD["E"], WORKLOAD["dtype"], seed=0)


def measure_cpu_baseline(min_seconds=10.0, max_seconds=30.0):
    inputs = cpu_sample_inputs(CPU_SAMPLE_ROWS)
    flops = 12.0 * CPU_SAMPLE_ROWS * WORKLOAD["D"] * WORKLOAD["E"]
    cpu_reference_step(inputs)  # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        cpu_reference_step(inputs)
        n += 1
        el = time.perf_counter() - t0
        if el >= min_seconds or (el >= max_seconds / 2 and n >= 1):
            break
    return {
        "value": round(flops * n / el / 1e12, 4),
        "unit": "TFLOP/s",
        "cores": cpu_threads(),
        "kind": "port",
        "sample": f"{n} x fwd+bwd of 1 head x {CPU_SAMPLE_ROWS} rows of {WORKLOAD_NAME} "
                  f"(numpy fp32 restatement of flashmlp_torch_fwd/bwd), {el:.1f} s",
    }


class ClockSampler:
    """nvidia-smi clock/throttle sampling while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = set(gpus)
        self.proc = None
        self.path = Path(tempfile.mkstemp(prefix="fmlp_clocks_", suffix=".csv")[1])

    def start(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            f = [s.strip() for s in line.split(",")]
            if len(f) < 9 or not f[0].isdigit() or int(f[0]) not in self.gpus:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        self.path.unlink(missing_ok=True)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        hi = [s for s in sm if s >= 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(hi), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def run_reference(args, rank):
    if rank != 0:
        return 0
    inputs = cpu_sample_inputs(CPU_SAMPLE_ROWS)
    flops = 12.0 * CPU_SAMPLE_ROWS * WORKLOAD["D"] * WORKLOAD["E"]
    for _ in range(args.warmup):
        cpu_reference_step(inputs)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_reference_step(inputs)
    el = time.perf_counter() - t0
    value = flops * args.steps / el / 1e12
    sample = (f"each step: fwd+bwd of 1 head x {CPU_SAMPLE_ROWS} rows of {WORKLOAD_NAME}, "
              f"numpy fp32 restatement of flashmlp_torch_fwd/bwd (the reference is Python and "
              f"does not travel to the GPU box)")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD_NAME, "sample_rows": CPU_SAMPLE_ROWS, "heads": 1,
                   "parallelism": "host cores"},
        "cpu_baseline": {"value": round(value, 4), "unit": "TFLOP/s", "cores": cpu_threads(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import flashmlp_b200 as F
    from flashmlp_b200 import sharding

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=120))
    H, B, D, E = (WORKLOAD[k] for k in "HBDE")
    act = WORKLOAD["activation"]
    h0, h1 = sharding.shard_range(H, world, rank)
    Hl = h1 - h0
    dt = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    x = torch.randn(Hl, B, D, device=dev, generator=g).to(dt)
    w1 = (torch.randn(Hl, D, E, device=dev, generator=g) / D ** 0.5).to(dt)
    w2 = (torch.randn(Hl, E, D, device=dev, generator=g) / E ** 0.5).to(dt)
    do = torch.randn(Hl, B, D, device=dev, generator=g).to(dt)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        F.flashmlp_fwd(x, w1, w2, act)
        F.flashmlp_bwd(x, w1, w2, do, act)
    barrier()

    n = args.steps
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3 * n)]
    sampler = ClockSampler(range(world)) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier()
    for i in range(n):
        ev[3 * i].record()
        F.flashmlp_fwd(x, w1, w2, act)
        ev[3 * i + 1].record()
        F.flashmlp_bwd(x, w1, w2, do, act)
        ev[3 * i + 2].record()
    barrier()
    clocks = sampler.stop() if sampler else None
    total_ms = ev[0].elapsed_time(ev[3 * n - 1])
    fwd_ms = [ev[3 * i].elapsed_time(ev[3 * i + 1]) for i in range(n)]
    bwd_ms = [ev[3 * i + 1].elapsed_time(ev[3 * i + 2]) for i in range(n)]
    t = torch.tensor([total_ms, statistics.mean(fwd_ms), statistics.mean(bwd_ms)], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, fwd_avg, bwd_avg = (float(v) for v in t.tolist())
    status = F._lib.lib().fmlp_device_status(1)
    # fmlp_fwd_pair_kernel + the backward's launches: fmlp_bwd_kernel, fmlp_dx_gemm_kernel in
    # the dZ-store mode, fmlp_dw_reduce_kernel when the dW programs are split
    bwd_ws = int(F._lib.lib().fmlp_bwd_workspace_size(Hl, B, D, E, 1))
    bwd_mode, bwd_splits, bwd_launches = F._lib.bwd_plan(Hl, B, D, E, 1, bwd_ws)
    launches_per_step = 1 + bwd_launches

    # ---- e2e through the public API with host buffers (pinned), copies inside the timed region
    n_e2e = max(1, min(n, 5))
    hx = x.cpu().pin_memory(); hw1 = w1.cpu().pin_memory(); hw2 = w2.cpu().pin_memory(); hdo = do.cpu().pin_memory()
    ho = torch.empty_like(hx).pin_memory(); hdx = torch.empty_like(hx).pin_memory()
    hdw1 = torch.empty_like(hw1).pin_memory(); hdw2 = torch.empty_like(hw2).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in (hx, hw1, hw2, hdo))
    d2h = sum(t.numel() * t.element_size() for t in (ho, hdx, hdw1, hdw2))

    from flashmlp_b200.host import HostPipeline

    hpg = max(1, Hl // 8)  # about 8 groups in flight: 4 heads at N=1, 1 head at N=8
    pipe = HostPipeline(dev, heads_per_group=hpg)

    def e2e_step():  # host in, host out; head groups pipelined over copy-in/compute/copy-out streams
        pipe.run(hx, hw1, hw2, hdo, act, out=(ho, hdx, hdw1, hdw2))

    e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n_e2e):
        e2e_step()
    e1.record()
    barrier()
    te = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_ms = float(te.item())

    cpu = measure_cpu_baseline() if (rank == 0 and world == 1 and not args.no_cpu_baseline) else None
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0

    fl_step_total = 12.0 * H * B * D * E
    value = fl_step_total * n / (total_ms / 1e3) / 1e12
    peaks, peak_src = load_peaks()
    peak_sus = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
    peak_burst = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    bwd_fl = 8.0 * Hl * B * D * E
    fwd_fl = 4.0 * Hl * B * D * E
    bwd_tf = bwd_fl / (bwd_avg / 1e3) / 1e12
    fwd_tf = fwd_fl / (fwd_avg / 1e3) / 1e12
    # DRAM bytes of the backward's launches (ncu, per head, scaled to this launch's heads)
    traffic = None
    tp = ROOT / "profiles" / "roofline_traffic.json"
    if tp.exists():
        try:
            key = "fmlp_bwd_dz_store" if bwd_mode == 1 else "fmlp_bwd_kernel"
            traffic = json.loads(tp.read_text())[key]["bytes_per_launch_per_head"] * Hl
        except Exception:
            traffic = None
    bwd_kernels = ("fmlp_bwd_kernel (dW programs, storing dZ^T) + fmlp_dx_gemm_kernel" if bwd_mode == 1
                   else "fmlp_bwd_kernel") + (" + fmlp_dw_reduce_kernel" if bwd_splits > 1 else "")
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": n,
        "warmup": args.warmup,
        "ms_per_step": round(total_ms / n, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": WORKLOAD_NAME, "H": H, "B": B, "D": D, "E": E, "activation": act,
                   "heads_per_gpu": Hl, "parallelism": f"head-sharded x{world} (no communication)",
                   "l2": "inputs larger than L2 every step (X and dO are 2x64-512 MiB per GPU); no flush"},
        "roofline": {
            "bound": "tensor", "kernel": "fmlp_bwd: " + bwd_kernels,
            "achieved": round(bwd_tf, 2), "peak": peak_sus, "unit": "TFLOP/s",
            "frac": round(bwd_tf / peak_sus, 4), "traffic": traffic,
            "peak_source": f"{peak_src} bf16_tflops_sustained (kernel timed inside a long step loop)",
            "algorithmic_flops_per_launch": bwd_fl,
            "bwd_mode": "dz-store" if bwd_mode == 1 else "recompute", "bwd_dw_splits": bwd_splits,
        },
        "fwd_ms": round(fwd_avg, 4), "bwd_ms": round(bwd_avg, 4),
        "fwd_tflops": round(fwd_tf, 2), "bwd_tflops": round(bwd_tf, 2),
        "frac_of_measured_burst": round(value / world / peak_burst, 4),
        "frac_of_spec_2250": round(value / world / SPEC_BF16_TFLOPS, 4),
        # tensor FLOPs the kernels execute: forward 4, backward 8 for the dW programs (Z^T,
        # dH^T, dW1, dW2) plus 2 (dX GEMM) in the dZ-store mode or 6 (dX programs) otherwise
        "executed_tensor_flops_per_step": (14.0 if bwd_mode == 1 else 18.0) * H * B * D * E,
        "cpu_baseline": cpu,
        "e2e": {"value": round(fl_step_total * n_e2e / (e2e_ms / 1e3) / 1e12, 3), "unit": "TFLOP/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": n_e2e,
                "path": "flashmlp_b200.host.HostPipeline.run: pinned host X, W1, W2, dO in; O, dX, dW1, dW2 "
                        f"back to pinned host memory; groups of {hpg} head(s) pipelined (copy-in / flashmlp_fwd "
                        "+ flashmlp_bwd / copy-out on three streams)"},
        "gpu_launches": launches_per_step * n,
        "clocks": clocks,
        "device_status": status,
    }
    print(json.dumps(line), flush=True)
    return 0


C5 = dict(H=8, B=131072, D=256, E=1024, activation="sigmoid", dtype="f16")
C5_NAME = "C5 batch-sharded training step H=8 B=131072 D=256 E=1024 fp16 sigmoid"


def run_c5(args, rank, world, local_rank):
    """data-parallel training step (fwd + bwd on B/N rows per GPU, dW
    all-reduce over NVLink, SGD). --allreduce fused: FusedBatchShardedTrainer (fp32 partials,
    fmlp_grad_allreduce_sgd); nccl: batch_sharded_train_step (NCCL all-reduce + update)."""
    import torch
    import torch.distributed as dist

    import flashmlp_b200 as F
    from flashmlp_b200 import sharding

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29517")
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    H, B, D, E = (C5[k] for k in "HBDE")
    act, dt, lr = C5["activation"], torch.float16, 1e-4
    b0, b1 = sharding.shard_range(B, world, rank)
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    x = torch.randn(H, b1 - b0, D, device=dev, generator=g).to(dt)
    do = torch.randn(H, b1 - b0, D, device=dev, generator=g).to(dt)
    gw = torch.Generator(device=dev).manual_seed(7)  # replicas start equal
    w1 = (torch.randn(H, D, E, device=dev, generator=gw) / D ** 0.5).to(dt)
    w2 = (torch.randn(H, E, D, device=dev, generator=gw) / E ** 0.5).to(dt)
    fused = args.allreduce == "fused"
    tr = sharding.FusedBatchShardedTrainer(w1, w2) if fused else None

    def step():
        if fused:
            tr.step(x, do, act, lr)
        else:
            sharding.batch_sharded_train_step(x, do, w1, w2, act, lr)

    for _ in range(args.warmup):
        step()
    dist.barrier()
    torch.cuda.synchronize()
    n = args.steps
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(range(world)) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    dist.barrier()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(n):
        step()
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop() if sampler else None
    t = torch.tensor([e0.elapsed_time(e1)], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    status = F._lib.lib().fmlp_device_status(1)
    if tr is not None:
        tr.close()
    dist.barrier()
    dist.destroy_process_group()
    if rank != 0:
        return 0
    fl = 12.0 * H * B * D * E
    line = {
        "metric": METRIC, "value": round(fl * n / (total_ms / 1e3) / 1e12, 2), "unit": "TFLOP/s",
        "n_gpus": world, "steps": n, "warmup": args.warmup, "ms_per_step": round(total_ms / n, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": C5_NAME, "H": H, "B": B, "D": D, "E": E, "activation": act,
                   "rows_per_gpu": b1 - b0, "parallelism": f"batch-sharded x{world}",
                   "allreduce": "fused fmlp_grad_allreduce_sgd (NVLink peer memory)" if fused
                   else "NCCL all-reduce + fmlp_sgd_update",
                   "l2": "inputs larger than L2 every step; no flush"},
        "clocks": clocks, "device_status": status,
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["c4", "c5"], default="c4",
                    help="c4 (default, the headline): head-sharded fwd+bwd; c5: batch-sharded training step")
    ap.add_argument("--allreduce", choices=["fused", "nccl"], default="fused", help="c5 only")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", str(rank)))
    if world != args.gpus:
        print(f"warning: WORLD_SIZE={world} but --gpus {args.gpus}", file=sys.stderr)
    if args.impl == "reference":
        return run_reference(args, rank)
    if args.workload == "c5":
        return run_c5(args, rank, world, local_rank)
    return run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    sys.exit(main())
