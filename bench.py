"""Benchmark of the fused multi-head MLP fwd+bwd (head-sharded).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

For N > 1 launch one process per GPU with torch.distributed.run; heads are split across
ranks (32/N per GPU, no communication) and the time is the max over ranks. One step is
one forward + one unified backward over the rank's heads with the batch B=65536, D=128,
E=2048, bf16, silu. Metric: algorithmic TFLOP/s of fwd+bwd (12*H*B*D*E per step) for
the whole job. Rank 0 prints one JSON line. Around the timed C4 region, and outside it:
  * parity: before timing, every rank checks head 0 of its shard (forward and backward
    of the full-shard launch) against an fp32 PyTorch reference on its own GPU;
  * the recompute-mode backward (low_memory_backward) timed alone, and the peak device
    memory of a fwd+bwd in both backward modes (measured as the reference's example.py
    does: max_memory_allocated above the resident inputs);
  * e2e: the same step from pinned host memory through flashmlp_b200.host.HostPipeline,
    plus the bare host-link copy rate of the same bytes on the same streams;
  * c5: BASELINE config 5 (batch-sharded training step, H=8, B=131072 split over the N
    ranks, D=256, E=1024, fp16 sigmoid) at the same N, with the fused NVLink all-reduce
    + SGD and with NCCL all-reduce + fmlp_sgd_update, each checked (replicas bit-identical,
    update equal to the fixed-order sum of the ranks' partial gradients).

--impl reference times the reference's own PyTorch path (flashmlp_torch_fwd/bwd,
flashmlp.py:671-723) on the host cores with all threads, on a bounded sample of the same
workload, on rank 0 only; the unmodified reference is loaded from baseline/_ref (the
oracle's numpy restatement stands in when it is absent). At N = 1 it also times the
reference's Triton kernels (flashmlp_fwd / flashmlp_bwd, flashmlp.py:428-538) on the GPU
at the full C4 shape (key triton_b200).
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
FALLBACK_PEAKS = {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0, "sm_max_mhz": 1965.0}
SPEC_BF16_TFLOPS = 2250.0
CPU_SAMPLE_ROWS = 8192  # rows of one head per CPU step (about 26 GFLOP of fwd+bwd)
C5 = dict(H=8, B=131072, D=256, E=1024, activation="sigmoid", dtype="f16")
C5_NAME = "C5 batch-sharded training step H=8 B=131072 D=256 E=1024 fp16 sigmoid"


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return d, "measured"
        except Exception:
            pass
    return FALLBACK_PEAKS, "fallback"


def select_peak(clocks, peaks, src):
    """The bf16 peak that applies to a run whose SM clocks were sampled: the burst figure
    (cuBLAS timed alone, at max clock) when the median SM clock under load sat at the
    maximum, otherwise the burst figure scaled by median / max clock."""
    burst = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    mx = (clocks or {}).get("sm_max_mhz") or peaks.get("sm_max_mhz") or FALLBACK_PEAKS["sm_max_mhz"]
    med = (clocks or {}).get("sm_mhz")
    if not med:
        return burst, f"{src} bf16_tflops (burst; no clock samples)"
    if med >= 0.98 * mx:
        return burst, f"{src} bf16_tflops (burst): median SM clock under load {med:.0f} MHz = max {mx:.0f} MHz"
    return burst * med / mx, (f"{src} bf16_tflops (burst) x median/max SM clock ({med:.0f}/{mx:.0f} MHz): the run "
                              "sat below max clock")


def set_host_threads():
    """All host cores for the CPU legs, whatever OMP_NUM_THREADS torchrun exported."""
    n = os.cpu_count() or 1
    try:
        import torch

        torch.set_num_threads(n)
    except Exception:
        pass
    try:
        from threadpoolctl import threadpool_limits

        threadpool_limits(n)
    except Exception:
        pass
    return n


def cpu_threads():
    try:
        import torch

        return torch.get_num_threads()
    except Exception:
        return os.cpu_count() or 1


def cpu_sample_inputs(rows):
    from oracle import flashmlp_oracle as orc

    return orc.make_inputs(1, rows, WORKLOAD["D"], WORKLOAD["E"], WORKLOAD["dtype"], seed=0)


def cpu_reference_stepper(rows):
    """(step function, kind, description) for one fwd+bwd of the reference's PyTorch path
    (flashmlp.py:671-723) on the host: the unmodified reference from baseline/_ref when it
    is installed, else the oracle's numpy restatement of the same functions."""
    from oracle.reference_loader import load_reference

    act = WORKLOAD["activation"]
    inputs = cpu_sample_inputs(rows)
    ref = None
    try:
        ref = load_reference()
    except Exception:
        ref = None
    if ref is not None:
        import torch

        x, w1, w2, do = (torch.from_numpy(a) for a in inputs)

        def step():
            ref.flashmlp_torch_fwd(x, w1, w2, act)
            ref.flashmlp_torch_bwd(x, w1, w2, do, act)

        return step, "reference", "the reference's flashmlp_torch_fwd + flashmlp_torch_bwd in fp32 (torch CPU)"
    from oracle import flashmlp_oracle as orc

    def step():
        orc.fwd_fp32(*inputs[:3], act)
        orc.bwd_fp32(*inputs, act)

    return step, "port", "numpy fp32 restatement of flashmlp_torch_fwd/bwd (reference not installed)"


def measure_cpu_baseline(min_seconds=10.0, max_seconds=30.0):
    set_host_threads()
    step, kind, what = cpu_reference_stepper(CPU_SAMPLE_ROWS)
    flops = 12.0 * CPU_SAMPLE_ROWS * WORKLOAD["D"] * WORKLOAD["E"]
    step()  # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        step()
        n += 1
        el = time.perf_counter() - t0
        if el >= min_seconds or (el >= max_seconds / 2 and n >= 1):
            break
    return {
        "value": round(flops * n / el / 1e12, 4),
        "unit": "TFLOP/s",
        "cores": cpu_threads(),
        "kind": kind,
        "sample": f"{n} x fwd+bwd of 1 head x {CPU_SAMPLE_ROWS} rows of {WORKLOAD_NAME} ({what}), {el:.1f} s",
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


# ----------------------------------------------------------------------------- reference arm
# The four configurations the reference publishes timings for (performance.md; bf16, silu,
# FlashMLP module on a 3-D input), timed the way its example.py does: wall clock over 100
# calls after 10 warm-ups, module and autograd overhead included.
PUBLISHED_CONFIGS = [(8, 512, 64, 512), (12, 1024, 64, 768), (16, 2048, 64, 1024), (32, 4096, 64, 512)]


def time_published_configs(module_cls, warmup=10, iters=100):
    """fwd and fwd+bwd (o.sum().backward()) wall-clock ms of `module_cls(H, D, E, ...)` at
    the reference's published configurations on cuda:0."""
    import numpy as np
    import torch

    out = []
    for H, B, D, E in PUBLISHED_CONFIGS:
        torch.manual_seed(0)
        model = module_cls(H, D, E, activation="silu", dtype=torch.bfloat16, device="cuda")
        x = torch.randn(H, B, D, device="cuda", dtype=torch.bfloat16) / np.sqrt(D)

        def fwd():
            return model(x)

        def fwd_bwd():
            x_in = x.detach().requires_grad_(True)
            model(x_in).sum().backward()

        res = {"config": [H, B, D, E]}
        for name, fn in (("fwd_ms", fwd), ("fwd_bwd_ms", fwd_bwd)):
            for _ in range(warmup):
                fn()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for _ in range(iters):
                fn()
            torch.cuda.synchronize()
            res[name] = round((time.perf_counter() - t0) / iters * 1e3, 4)
        out.append(res)
        del model, x
    return out


def time_reference_triton(steps, warmup):
    """The reference's Triton wrappers (flashmlp.py:428-538, autotuned on first call) on
    cuda:0 at the full C4 shape, CUDA events on torch's current stream (the stream Triton
    launches on), plus their peak memory as the reference's example.py measures it."""
    import torch

    from oracle.reference_loader import load_reference

    ref = load_reference()
    if ref is None or not torch.cuda.is_available():
        return {"unavailable": "reference not installed in baseline/_ref" if ref is None else "no CUDA device"}
    H, B, D, E = (WORKLOAD[k] for k in "HBDE")
    act = WORKLOAD["activation"]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(1000)
    x = torch.randn(H, B, D, device=dev, generator=g).to(torch.bfloat16)
    w1 = (torch.randn(H, D, E, device=dev, generator=g) / D ** 0.5).to(torch.bfloat16)
    w2 = (torch.randn(H, E, D, device=dev, generator=g) / E ** 0.5).to(torch.bfloat16)
    do = torch.randn(H, B, D, device=dev, generator=g).to(torch.bfloat16)
    t0 = time.perf_counter()
    ref.flashmlp_fwd(x, w1, w2, act)
    ref.flashmlp_bwd(x, w1, w2, do, act)
    torch.cuda.synchronize()
    tune_s = time.perf_counter() - t0
    for _ in range(max(0, warmup - 1)):
        ref.flashmlp_fwd(x, w1, w2, act)
        ref.flashmlp_bwd(x, w1, w2, do, act)
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3 * steps)]
    for i in range(steps):
        ev[3 * i].record()
        ref.flashmlp_fwd(x, w1, w2, act)
        ev[3 * i + 1].record()
        ref.flashmlp_bwd(x, w1, w2, do, act)
        ev[3 * i + 2].record()
    torch.cuda.synchronize()
    fwd = statistics.mean(ev[3 * i].elapsed_time(ev[3 * i + 1]) for i in range(steps))
    bwd = statistics.mean(ev[3 * i + 1].elapsed_time(ev[3 * i + 2]) for i in range(steps))
    hbde = float(H) * B * D * E
    torch.cuda.reset_peak_memory_stats(dev)
    before = torch.cuda.memory_allocated(dev)
    o = ref.flashmlp_fwd(x, w1, w2, act)  # O stays alive through the backward, as in training
    grads = ref.flashmlp_bwd(x, w1, w2, do, act)
    torch.cuda.synchronize()
    peak = torch.cuda.max_memory_allocated(dev) - before
    del o, grads
    return {
        "config": WORKLOAD_NAME, "steps": steps, "autotune_and_compile_s": round(tune_s, 1),
        "fwd_ms": round(fwd, 4), "bwd_ms": round(bwd, 4), "step_ms": round(fwd + bwd, 4),
        "fwd_tflops": round(4 * hbde / fwd / 1e9, 2), "bwd_tflops": round(8 * hbde / bwd / 1e9, 2),
        "tflops": round(12 * hbde / (fwd + bwd) / 1e9, 2),
        "peak_mem_above_inputs_bytes": int(peak),
        "timing": "CUDA events on torch's current stream, mean over steps, after autotune and warm-up",
    }


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    cores = set_host_threads()
    step, kind, what = cpu_reference_stepper(CPU_SAMPLE_ROWS)
    flops = 12.0 * CPU_SAMPLE_ROWS * WORKLOAD["D"] * WORKLOAD["E"]
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    value = flops * args.steps / el / 1e12
    sample = f"each step: fwd+bwd of 1 head x {CPU_SAMPLE_ROWS} rows of {WORKLOAD_NAME}, {what}"
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD_NAME, "sample_rows": CPU_SAMPLE_ROWS, "heads": 1,
                   "parallelism": "host cores"},
        "cpu_baseline": {"value": round(value, 4), "unit": "TFLOP/s", "cores": cores,
                         "kind": kind, "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    if world == 1 and not args.no_triton:
        try:
            line["triton_b200"] = time_reference_triton(args.steps, args.warmup)
            from oracle.reference_loader import load_reference
            ref = load_reference()
            if ref is not None:
                line["triton_b200"]["published_configs"] = time_published_configs(ref.FlashMLP)
        except Exception as e:  # reported, not fatal: the line's value is the CPU path
            line["triton_b200"] = {"unavailable": f"{type(e).__name__}: {str(e)[:300]}"}
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- our arm
def _tests_helpers():
    sys.path.insert(0, str(ROOT / "tests"))
    import _refcheck

    return _refcheck


def check_head0(F, x, w1, w2, do, act, o, dx, dw1, dw2):
    """Head 0 of this rank's full-shard results against the fp32 PyTorch reference with the
    kernels' rounding points: elementwise README tolerance + dot-product bound and the
    norm-wise bound. Returns (ok, worst norm-wise relative error, message)."""
    import torch

    rc = _tests_helpers()
    sl = slice(0, 1)
    worst, msg = 0.0, ""
    try:
        r, bnd = rc.ref_fwd(x[sl], w1[sl], w2[sl], act)
        rc.assert_close(o[sl], r, bnd, x.dtype, "fwd", "o")
        worst = max(worst, max(rc.norm_rel_errors(o[sl], r)))
        del r, bnd
        refs = rc.ref_bwd(x[sl], w1[sl], w2[sl], do[sl], act)
        for k, v in (("dx", dx), ("dw1", dw1), ("dw2", dw2)):
            rc.assert_close(v[sl], *refs[k], x.dtype, "bwd", k)
            worst = max(worst, max(rc.norm_rel_errors(v[sl], refs[k][0])))
        del refs
        ok = True
    except AssertionError as e:
        ok, msg = False, str(e)[:300]
    torch.cuda.empty_cache()
    return ok, worst, msg


def numa_bind(dev):
    """Binds this process to the CPUs of its GPU's NUMA node when the host has more than
    one node (pinned buffers allocated afterwards are then node-local). Returns a record."""
    import torch

    nodes = sorted(p.name for p in Path("/sys/devices/system/node").glob("node[0-9]*"))
    rec = {"nodes": len(nodes), "gpu_node": None, "bound": False}
    try:
        p = torch.cuda.get_device_properties(dev)
        bus = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        node = int(Path(f"/sys/bus/pci/devices/{bus}/numa_node").read_text().strip())
        rec["gpu_node"] = node
        if len(nodes) > 1 and node >= 0:
            cpus = Path(f"/sys/devices/system/node/node{node}/cpulist").read_text().strip()
            sel = set()
            for part in cpus.split(","):
                a, _, b = part.partition("-")
                sel.update(range(int(a), int(b or a) + 1))
            os.sched_setaffinity(0, sel)
            rec["bound"] = True
    except Exception as e:
        rec["error"] = f"{type(e).__name__}: {e}"[:120]
    return rec


def copy_only_rates(dev, host_in, dev_in, dev_out, host_out, reps=3):
    """Host-link rate of the step's bytes alone: the same pinned buffers, H2D and D2H
    copies running at once on two streams (one cudaMemcpyAsync per tensor), no kernels.
    Returns (h2d GB/s, d2h GB/s)."""
    import torch

    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    bi = sum(t.numel() * t.element_size() for t in host_in)
    bo = sum(t.numel() * t.element_size() for t in host_out)
    best_in, best_out = 0.0, 0.0
    for _ in range(reps):
        torch.cuda.synchronize(dev)
        ei = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        eo = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        with torch.cuda.stream(s_in):
            ei[0].record(s_in)
            for d, h in zip(dev_in, host_in):
                d.copy_(h, non_blocking=True)
            ei[1].record(s_in)
        with torch.cuda.stream(s_out):
            eo[0].record(s_out)
            for h, d in zip(host_out, dev_out):
                h.copy_(d, non_blocking=True)
            eo[1].record(s_out)
        torch.cuda.synchronize(dev)
        best_in = max(best_in, bi / (ei[0].elapsed_time(ei[1]) / 1e3) / 1e9)
        best_out = max(best_out, bo / (eo[0].elapsed_time(eo[1]) / 1e3) / 1e9)
    return best_in, best_out


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import flashmlp_b200 as F
    from flashmlp_b200 import sharding

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    numa = numa_bind(dev)
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

    def max_over_ranks(vals):
        t = torch.tensor(vals, device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return [float(v) for v in t.tolist()]

    def gather(vals):
        t = torch.tensor(vals, device=dev, dtype=torch.float64)
        if world == 1:
            return [t.tolist()]
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t)
        return [p.tolist() for p in parts]

    # ---- parity of this rank's shard (head 0 of the full-shard launch), before the
    # warm-up so that the check's allocations are gone before timing
    o = F.flashmlp_fwd(x, w1, w2, act)
    dx, dw1, dw2 = F.flashmlp_bwd(x, w1, w2, do, act)
    ok, worst, msg = check_head0(F, x, w1, w2, do, act, o, dx, dw1, dw2)
    del o, dx, dw1, dw2
    for _ in range(args.warmup):
        F.flashmlp_fwd(x, w1, w2, act)
        F.flashmlp_bwd(x, w1, w2, do, act)
    par = gather([1.0 if ok else 0.0, worst])
    parity = {"ranks_ok": int(sum(p[0] for p in par)), "ranks": world,
              "max_norm_rel_err": float(f"{max(p[1] for p in par):.3e}"),
              "checked": "head 0 of every rank's shard: O, dX, dW1, dW2 of the timed launch vs fp32 PyTorch with "
                         "the kernels' rounding points (README atol/rtol + dot bound per element, and "
                         "||a-r||_F <= 5e-3 ||r||_F)"}
    if not ok:
        parity["rank_error"] = msg
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
    total_ms, fwd_avg, bwd_avg = max_over_ranks([total_ms, statistics.mean(fwd_ms), statistics.mean(bwd_ms)])
    status = F._lib.lib().fmlp_device_status(1)
    # fmlp_fwd_pair_kernel + the backward's launches: fmlp_bwd_kernel, fmlp_dx_gemm_kernel in
    # the dZ-store mode, fmlp_dw_reduce_kernel when the dW programs are split
    bwd_ws = int(F._lib.lib().fmlp_bwd_workspace_size(Hl, B, D, E, 1))
    bwd_mode, bwd_splits, bwd_launches = F._lib.bwd_plan(Hl, B, D, E, 1, bwd_ws)
    launches_per_step = 1 + bwd_launches

    # ---- the recompute-mode backward (the PID-split kernel, low_memory_backward), timed alone
    with F.low_memory_backward():
        rmode, rsplits, rlaunch = F._lib.bwd_plan(Hl, B, D, E, 1, int(F._lib.lib().fmlp_bwd_workspace_size_min(
            Hl, B, D, E, 1)))
        for _ in range(2):
            F.flashmlp_bwd(x, w1, w2, do, act)
        barrier()
        r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        r0.record()
        for _ in range(n):
            F.flashmlp_bwd(x, w1, w2, do, act)
        r1.record()
        barrier()
    (rec_ms,) = max_over_ranks([r0.elapsed_time(r1) / n])

    # ---- peak device memory of one fwd+bwd, as the reference's example.py measures it
    # (max_memory_allocated above what is allocated before the step: the inputs)
    def peak_of(ctx):
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        torch.cuda.reset_peak_memory_stats(dev)
        before = torch.cuda.memory_allocated(dev)
        with ctx:
            o_ = F.flashmlp_fwd(x, w1, w2, act)
            r_ = F.flashmlp_bwd(x, w1, w2, do, act)
        torch.cuda.synchronize()
        pk = torch.cuda.max_memory_allocated(dev) - before
        del o_, r_
        return pk

    import contextlib

    peak_dz = peak_of(contextlib.nullcontext())
    peak_rec = peak_of(F.low_memory_backward())
    inputs_bytes = sum(t.numel() * t.element_size() for t in (x, w1, w2, do))
    peaks_mem = max_over_ranks([peak_dz, peak_rec])

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
    (e2e_ms,) = max_over_ranks([e0.elapsed_time(e1)])
    # the host link alone, all ranks at once (the step's bytes, same pinned buffers)
    dev_out = [torch.empty_like(t, device=dev) for t in (hx, hx, hw1, hw2)]
    barrier()
    cin, cout = copy_only_rates(dev, (hx, hw1, hw2, hdo), (x, w1, w2, do), dev_out, (ho, hdx, hdw1, hdw2))
    rates = gather([cin, cout])
    del dev_out, pipe

    # ---- FP8 (e4m3) forward of the same shard (not in the reference)
    fp8 = None
    if not args.no_fp8:
        fp8 = run_fp8_leg(F, x, w1, w2, act, n, barrier, max_over_ranks, gather)

    # ---- C5 at the same N (batch-sharded training step)
    del x, w1, w2, do
    torch.cuda.empty_cache()
    c5 = None
    if not args.no_c5:
        c5 = run_c5_leg(args, rank, world, dev, barrier, max_over_ranks, gather)

    # the reference's published configurations, timed as its example.py does (N = 1 only)
    pub = time_published_configs(F.FlashMLP) if (rank == 0 and world == 1) else None
    cpu = measure_cpu_baseline() if (rank == 0 and world == 1 and not args.no_cpu_baseline) else None
    if world > 1:
        dist.barrier()
    if dist.is_initialized():
        dist.destroy_process_group()
    if rank != 0:
        return 0

    fl_step_total = 12.0 * H * B * D * E
    value = fl_step_total * n / (total_ms / 1e3) / 1e12
    peaks, peak_src = load_peaks()
    peak, peak_why = select_peak(clocks, peaks, peak_src)
    bwd_fl = 8.0 * Hl * B * D * E
    fwd_fl = 4.0 * Hl * B * D * E
    bwd_tf = bwd_fl / (bwd_avg / 1e3) / 1e12
    fwd_tf = fwd_fl / (fwd_avg / 1e3) / 1e12
    step_tf_gpu = value / world
    exec_fl = (14.0 if bwd_mode == 1 else 18.0) * H * B * D * E
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
        "parity": parity,
        "roofline": {
            "bound": "tensor", "kernel": "fmlp_bwd: " + bwd_kernels,
            "achieved": round(bwd_tf, 2), "peak": round(peak, 1), "unit": "TFLOP/s",
            "frac": round(bwd_tf / peak, 4), "traffic": traffic,
            "peak_source": peak_why,
            "algorithmic_flops_per_launch": bwd_fl,
            "frac_fwd": round(fwd_tf / peak, 4), "frac_step_per_gpu": round(step_tf_gpu / peak, 4),
            "frac_executed_step_per_gpu": round(exec_fl * n / world / (total_ms / 1e3) / 1e12 / peak, 4),
            "bwd_mode": "dz-store" if bwd_mode == 1 else "recompute", "bwd_dw_splits": bwd_splits,
        },
        "fwd_ms": round(fwd_avg, 4), "bwd_ms": round(bwd_avg, 4),
        "fwd_tflops": round(fwd_tf, 2), "bwd_tflops": round(bwd_tf, 2),
        "frac_of_spec_2250": round(step_tf_gpu / SPEC_BF16_TFLOPS, 4),
        # tensor FLOPs the kernels execute: forward 4, backward 8 for the dW programs (Z^T,
        # dH^T, dW1, dW2) plus 2 (dX GEMM) in the dZ-store mode or 6 (dX programs) otherwise
        "executed_tensor_flops_per_step": exec_fl,
        "bwd_recompute": {"ms": round(rec_ms, 4), "tflops": round(bwd_fl / (rec_ms / 1e3) / 1e12, 2),
                          "dw_splits": rsplits, "launches": rlaunch,
                          "what": "the unified backward with the reference's dW/dX program-ID split "
                                  "(low_memory_backward: dX programs recompute Z and dH), timed alone"},
        "peak_mem_bytes": {"dz_store": int(peaks_mem[0]), "recompute": int(peaks_mem[1]),
                           "inputs": int(inputs_bytes),
                           "how": "torch.cuda.max_memory_allocated above the resident inputs over one fwd+bwd "
                                  "(outputs and workspace included), max over ranks, as example.py measures it"},
        "cpu_baseline": cpu,
        "e2e": {"value": round(fl_step_total * n_e2e / (e2e_ms / 1e3) / 1e12, 3), "unit": "TFLOP/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": n_e2e,
                "path": "flashmlp_b200.host.HostPipeline.run: pinned host X, W1, W2, dO in; O, dX, dW1, dW2 "
                        f"back to pinned host memory; groups of {hpg} head(s) pipelined (copy-in / flashmlp_fwd "
                        "+ flashmlp_bwd / copy-out on three streams)",
                "copy_only_gbs": {"h2d": [round(r[0], 1) for r in rates], "d2h": [round(r[1], 1) for r in rates],
                                  "what": "per rank, all ranks at once: the step's bytes between the same pinned "
                                          "buffers and the device, H2D and D2H concurrently on two streams, no kernels"},
                "copy_bound_ms": round(max(h2d / (min(r[0] for r in rates) * 1e9),
                                           d2h / (min(r[1] for r in rates) * 1e9)) * 1e3, 3),
                "numa": numa},
        "c5": c5,
        "published_configs": pub,
        "fp8_forward": None if fp8 is None else dict(
            fp8, tflops=round(fwd_fl / (fp8["ms"] / 1e3) / 1e12, 2),
            speedup_vs_bf16_forward=round(fwd_avg / fp8["ms"], 3)),
        "gpu_launches": launches_per_step * n,
        "clocks": clocks,
        "device_status": status,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_fp8_leg(F, x, w1, w2, act, n, barrier, max_over_ranks, gather):
    """The shard's forward in FP8 (flashmlp_fwd_fp8): X, W1, W2 quantized to e4m3 with
    per-tensor scales, h_scale from the amax of head 0's activations, head 0 of the output
    checked against the quantized fp32 reference (norm-wise), then `n` forwards timed on
    the device (max over ranks)."""
    import torch

    acts = {"silu": torch.nn.functional.silu, "sigmoid": torch.sigmoid,
            "leaky_relu": lambda z: torch.nn.functional.leaky_relu(z, 0.01)}
    actf = acts.get(act, lambda z: z)
    x8, sx = F.quantize_e4m3(x)
    W = F.prepare_fp8_weights(w1, w2)
    z0 = torch.mm(x8[0].float(), W.w1t[0].float().t()) * (sx * W.w1_scale)
    h0 = actf(z0)
    sh = max(float(h0.abs().max()) / 448.0, 1e-6)
    h8 = (h0 / sh).clamp(-448.0, 448.0).to(torch.float8_e4m3fn).float()
    r0 = torch.mm(h8, W.w2t[0].float().t()) * (sh * W.w2_scale)
    del z0, h0, h8
    o = F.flashmlp_fwd_fp8(x8, W, act, x_scale=sx, h_scale=sh)
    rel = float((o[0].float() - r0).norm() / r0.norm())
    del o, r0
    for _ in range(3):
        F.flashmlp_fwd_fp8(x8, W, act, x_scale=sx, h_scale=sh)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n):
        F.flashmlp_fwd_fp8(x8, W, act, x_scale=sx, h_scale=sh)
    e1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks([e0.elapsed_time(e1) / n])[0]
    rels = gather([rel])
    del x8, W
    torch.cuda.empty_cache()
    return {"ms": round(ms, 4), "max_norm_rel_err_head0": float(f"{max(r[0] for r in rels):.3e}"),
            "kernel": "fmlp_fwd_fp8_kernel (tcgen05.mma kind::f8f6f4, e4m3 x e4m3, fp32 accumulation)",
            "what": "flashmlp_fwd_fp8 of the same shard: per-tensor e4m3 scales, H8 = e4m3(act(Z) / h_scale), "
                    "bf16 output; head 0 checked against the quantized fp32 reference"}


def run_c5_leg(args, rank, world, dev, barrier, max_over_ranks, gather):
    """BASELINE config 5 at this N: each rank owns B/N rows, runs fwd + bwd, and the dW are
    summed over ranks before an SGD step. Two variants: the fused NVLink all-reduce + SGD
    (FusedBatchShardedTrainer, fp32 partials) and NCCL all-reduce + fmlp_sgd_update
    (batch_sharded_train_step). Before timing, one step of each is checked."""
    import torch
    import torch.distributed as dist

    import flashmlp_b200 as F
    from flashmlp_b200 import sharding

    if not dist.is_initialized():  # N = 1: a one-rank group (the trainer's plumbing needs one)
        dist.init_process_group("nccl", store=dist.HashStore(), rank=0, world_size=1, device_id=dev)
    H, B, D, E = (C5[k] for k in "HBDE")
    act, dt, lr = C5["activation"], torch.float16, 1e-4
    b0, b1 = sharding.shard_range(B, world, rank)
    g = torch.Generator(device=dev).manual_seed(2000 + rank)
    x = torch.randn(H, b1 - b0, D, device=dev, generator=g).to(dt)
    do = torch.randn(H, b1 - b0, D, device=dev, generator=g).to(dt)
    gw = torch.Generator(device=dev).manual_seed(7)  # replicas start equal
    w1_0 = (torch.randn(H, D, E, device=dev, generator=gw) / D ** 0.5).to(dt)
    w2_0 = (torch.randn(H, E, D, device=dev, generator=gw) / E ** 0.5).to(dt)
    fl = 12.0 * H * B * D * E
    out = {"config": C5_NAME, "rows_per_gpu": b1 - b0}
    n = args.steps

    def replicas_equal(w1, w2):
        ws = torch.cat([w1.reshape(-1), w2.reshape(-1)])
        if world == 1:
            return True
        parts = [torch.empty_like(ws) for _ in range(world)]
        dist.all_gather(parts, ws)
        return all(torch.equal(parts[0], p) for p in parts[1:])

    for variant in ("fused", "nccl"):
        w1, w2 = w1_0.clone(), w2_0.clone()
        tr = sharding.FusedBatchShardedTrainer(w1, w2) if variant == "fused" else None
        # ---- check one step: the update equals the fixed-order fp32 sum of every rank's
        # partial gradient (fused: bit for bit; NCCL: within fp32 summation-order error)
        if variant == "fused":
            _, part = F.flashmlp_bwd_dw_f32(x, tr.w1, tr.w2, do, act)
        else:
            _, pd1, pd2 = F.flashmlp_bwd(x, w1, w2, do, act)
            part = torch.cat([pd1.reshape(-1).float(), pd2.reshape(-1).float()])
        if world > 1:
            parts = [torch.empty_like(part) for _ in range(world)]
            dist.all_gather(parts, part)
        else:
            parts = [part]
        gsum = parts[0].clone()
        for p_ in parts[1:]:
            gsum += p_
        n1 = w1.numel()
        rw1 = (w1_0.float() - lr * gsum[:n1].view(w1.shape)).to(dt)
        rw2 = (w2_0.float() - lr * gsum[n1:].view(w2.shape)).to(dt)
        if variant == "fused":
            tr.step(x, do, act, lr)  # raises if the all-reduce failed on any rank
            upd_ok = torch.equal(tr.w1, rw1) and torch.equal(tr.w2, rw2)
            same = replicas_equal(tr.w1, tr.w2)
        else:
            _, _, g1, g2 = sharding.batch_sharded_train_step(x, do, w1, w2, act, lr)
            gflat = torch.cat([g1.reshape(-1), g2.reshape(-1)])
            tol = 1e-5 * gsum.abs().max().item() * world
            upd_ok = bool(((gflat - gsum).abs() <= tol).all())
            same = replicas_equal(w1, w2)
        del parts, gsum, part, rw1, rw2
        checks = gather([1.0 if upd_ok else 0.0, 1.0 if same else 0.0])

        def step():
            if tr is not None:
                tr.step(x, do, act, lr, check=False)
            else:
                sharding.batch_sharded_train_step(x, do, w1, w2, act, lr)

        for _ in range(args.warmup):
            step()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            step()
        e1.record()
        barrier()
        (ms,) = max_over_ranks([e0.elapsed_time(e1) / n])
        ok_after = True
        if tr is not None:
            ok_after = tr.status() == 0
            same_after = replicas_equal(tr.w1, tr.w2)
            tr.close()
        else:
            same_after = replicas_equal(w1, w2)
        after = gather([1.0 if ok_after else 0.0, 1.0 if same_after else 0.0])
        out[variant] = {
            "ms_per_step": round(ms, 4), "tflops": round(fl / (ms / 1e3) / 1e12, 2),
            "update_matches_sum_of_partials": all(c[0] == 1.0 for c in checks),
            "replicas_bit_identical": all(c[1] == 1.0 for c in checks) and all(a[1] == 1.0 for a in after),
            "allreduce_status_ok": all(a[0] == 1.0 for a in after),
            "allreduce": ("fmlp_grad_allreduce_sgd: fixed-order fp32 sum over NVLink peer memory + SGD, "
                          "replicas written by the owning rank") if variant == "fused"
            else "NCCL all-reduce (fp32) + fmlp_sgd_update",
        }
        del w1, w2, tr
        torch.cuda.empty_cache()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-c5", action="store_true", help="skip the C5 batch-sharded leg")
    ap.add_argument("--no-fp8", action="store_true", help="skip the FP8 forward leg")
    ap.add_argument("--no-triton", action="store_true", help="reference arm: skip the Triton-on-GPU timing")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", str(rank)))
    if world != args.gpus:
        print(f"warning: WORLD_SIZE={world} but --gpus {args.gpus}", file=sys.stderr)
    if args.impl == "reference":
        return run_reference(args, rank, world)
    return run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    sys.exit(main())
