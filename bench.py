#!/usr/bin/env python3
"""Planner benchmark: plan steps/s, candidate-steps/s and p50/p95 plan latency.

Default workload: SkyJEPA learned MPPI, one vehicle, 512 candidates x 15
steps, latent/GRU 256, state TCN [128,128,128], action TCN [4,4,4], prober
32 x 2, f32, seeded random weights and synthetic context (figure-eight
reference).  A "step" is one plan call.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload skyjepa|nominal]
    python bench.py --impl reference ...   # the CPU restatement on the host cores
    python bench.py --workload fleet [--shard auto|vehicles|candidates] [--vehicles V --samples S --horizon T]
    python bench.py --workload lewm-vector|lewm-image    # LeWM CEM (vector obs) / MPPI (NV12 frames + ViT)
    python bench.py --workload media [--precision f32|bf16] [--media-format nv12|rgb|rgba]
                                           # frame preprocessing -> NCHW vs the HBM roofline
    python bench.py --workload closed-loop [--dynamics learned|nominal] [--random-domains N]
                                          # closed-loop session scenarios; --steps = control steps per scenario

`value` is timed with CUDA events around each plan on the device with the
context resident (L2 flushed between steps); `e2e` times the public C-ABI
calls with host buffers (context upload + plan + result download).  With
--gpus N every rank plans its own vehicle ("replicas only": one vehicle's
512-candidate plan does not shard) and `value` is the job-wide plans/s.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "le-wm-nv_b200"))

# Algorithmic work per candidate-step (op count of the model; see the
# workload notes in the design document): GRU 4x768 + 256x768 MAC, action TCN
# 2,880 MAC, prober 9,696 MAC, integrator + cost ~200 FLOP.
FLOP_PER_CANDIDATE_STEP = {
    "skyjepa": 2 * (4 * 768 + 256 * 768 + 2880 + 256 * 32 + 32 * 32 + 32 * 15) + 200,
    "nominal": 10 * 262 + 60,
}
FLOP_PER_CANDIDATE_STEP["fleet"] = FLOP_PER_CANDIDATE_STEP["skyjepa"]
# The rollout kernel's share: everything above but the action TCN, which the
# input kernel ahead of it evaluates.
ROLLOUT_FLOP_PER_CANDIDATE_STEP = 2 * (4 * 768 + 256 * 768 + 256 * 32 + 32 * 32 + 32 * 15) + 200
# DRAM bytes (read + write) of one rollout launch of the default workload
# (512 x 15, latent 256, split-fp16 tensor-core kernel), from an ncu capture
# of that launch: the packed weights and the x tiles (the per-step h exchange
# through its global buffer stays in L2).
ROLLOUT_DRAM_BYTES = {"skyjepa": 1847040}


NCCL_LOG = None  # where this process's NCCL communicator log goes (multi-GPU runs)


def nccl_log_setup():
    """Turn on NCCL's communicator log (INIT lines: ranks, devices, NVLS) on
    stderr, so stdout keeps the one JSON line (NCCL's own default is
    stdout); returns where it goes.  Called before torch (and NCCL) are
    loaded, so NCCL reads the settings.  A caller's own NCCL_DEBUG wins."""
    if "NCCL_DEBUG" in os.environ:
        return os.environ.get("NCCL_DEBUG_FILE", "stdout") + f" (NCCL_DEBUG={os.environ['NCCL_DEBUG']}, caller's)"
    os.environ["NCCL_DEBUG"] = "INFO"
    os.environ["NCCL_DEBUG_SUBSYS"] = "INIT"
    os.environ["NCCL_DEBUG_FILE"] = "/dev/stderr"
    return "stderr (NCCL_DEBUG=INFO, NCCL_DEBUG_SUBSYS=INIT)"


if int(os.environ.get("WORLD_SIZE", "1")) > 1:
    NCCL_LOG = nccl_log_setup()


def default_workload_config(kind: str, world: int) -> dict:
    """The `config` both arms print for the default and nominal workloads
    (the same seeded inputs, planner and model widths in both)."""
    model = (", latent 256, TCN [128,128,128]/[4,4,4], prober 32x2" if kind == "skyjepa" else ", 10 rotor substeps")
    return {"workload": f"{kind} MPPI, 1 vehicle per plan, 512 candidates x 15 steps, 1 iteration, seed 17" + model,
            "parallelism": f"one vehicle per rank, replicas x{world}"}


def percentile(values, q):
    """values[round((n-1) q)] of the sorted list (lewm-bench-skyjepa.rs:547-553)."""
    v = sorted(values)
    return v[int(round((len(v) - 1) * q))] if v else 0.0


class ClockSampler:
    """nvidia-smi clocks and throttle reasons while the timed region runs."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[3:7]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(mx), "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except OSError:
        return {}


def sgemm_peak_tflops(torch):
    """FP32 CUDA-core GEMM throughput (cuBLAS SGEMM, TF32 off), measured here:
    the denominator for FP32 FFMA kernels (MEASURED_PEAKS has HBM and bf16 only)."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    n = 8192
    a = torch.randn(n, n, device="cuda")
    b = torch.randn(n, n, device="cuda")
    for _ in range(2):
        torch.matmul(a, b)
    torch.cuda.synchronize()
    best = 1e9
    for _ in range(5):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch.matmul(a, b)
        e.record()
        torch.cuda.synchronize()
        best = min(best, s.elapsed_time(e))
    torch.backends.cuda.matmul.allow_tf32 = prev
    del a, b
    return 2 * n ** 3 / (best * 1e-3) / 1e12


# ----------------------------------------------------------------- our arm

def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import lewm_b200 as L
    from lewm_b200 import workloads as W

    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", init_method="env://", timeout=__import__("datetime").timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    ctx = L.Context(local_rank)
    stream = ctx.torch_stream()
    kind = args.workload
    seed = 17 + rank
    if kind == "skyjepa":
        w = W.skyjepa(seed=seed)
        sc = L.SkyJepaScorer(ctx, w.model, w.weights, w.state_mean, w.state_std, w.action_mean, w.action_std, w.cost,
                             w.dt)
        set_ctx = lambda: sc.set_context(w.state_history, w.action_history, w.reference_states, w.reference_actions)
        h2d = (w.state_history.nbytes + w.action_history.nbytes + w.reference_states.nbytes +
               w.reference_actions.nbytes)
    else:
        w = W.nominal(seed=seed)
        sc = L.NominalScorer(ctx, w.dt, w.trim, w.cost, w.substeps)
        set_ctx = lambda: sc.set_context(w.initial, w.motors, w.reference_states, w.reference_actions)
        h2d = w.initial.nbytes + w.motors.nbytes + w.reference_states.nbytes + w.reference_actions.nbytes
    set_ctx()
    planner = L.MppiPlanner(ctx, w.mppi)
    planner.set_warm_start_sequence(w.warm_start)
    S, T = w.samples, w.horizon
    cand_steps = w.batch * S * T * w.mppi.iterations
    flush = torch.empty(256 * 1024 * 1024 // 4, device="cuda")  # > 126 MB L2

    def flush_l2():
        with torch.cuda.stream(stream):
            flush.add_(1.0)

    # ---- device-resident timing (value)
    for _ in range(args.warmup):
        planner.plan_device(sc)
    ctx.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    n0 = ctx.launch_count()
    times = []
    clocks = ClockSampler(local_rank)
    with clocks:
        for _ in range(args.steps):
            flush_l2()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            planner.plan_device(sc)
            e.record(stream)
            e.synchronize()
            times.append(s.elapsed_time(e))
    launches = (ctx.launch_count() - n0) // args.steps
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    # ---- the dominant kernel alone (for the roofline): CUDA events the
    # library records on its stream around the rollout launch, same loop
    kernel_ms = []
    if kind == "skyjepa":
        ctx.set_kernel_timing(True)
        for _ in range(args.steps):
            flush_l2()
            planner.plan_device(sc)
            kernel_ms.append(ctx.kernel_time_ms())
        ctx.set_kernel_timing(False)

    # ---- end to end through the public ABI (host context in, host result out)
    e2e_times = []
    for _ in range(args.warmup):
        set_ctx()
        planner.plan(sc)
    for _ in range(args.steps):
        flush_l2()
        ctx.synchronize()
        t0 = time.perf_counter()
        set_ctx()
        r = planner.plan(sc)
        e2e_times.append((time.perf_counter() - t0) * 1e3)
    d2h = 4 * (w.batch * 4 + w.batch * T * 4 + w.batch * S + w.batch)

    total_ms = sum(times)
    stats = torch.tensor([total_ms, float(np.mean(e2e_times))], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    total_ms, e2e_mean = stats.tolist()
    result = None
    if rank == 0:
        ms = total_ms / args.steps
        plans_per_s = world * args.steps / (total_ms * 1e-3)
        e2e_plans_per_s = world * 1e3 / e2e_mean
        peaks = measured_peaks()
        if kind == "skyjepa":
            # the split-fp16 tensor-core rollout: FLOP of the model (not the
            # three fp16 products each f32 MAC takes) over its mean device time
            kmean = float(np.mean(kernel_ms))
            flop = ROLLOUT_FLOP_PER_CANDIDATE_STEP * cand_steps
            achieved = flop / (kmean * 1e-3) / 1e12
            peak = float(peaks.get("bf16_tflops") or 1590.0)
            roofline = {"bound": "tensor", "achieved": round(achieved, 3), "peak": round(peak, 1),
                        "unit": "TFLOP/s", "frac": round(achieved / peak, 5),
                        "traffic": ROLLOUT_DRAM_BYTES.get(kind),
                        "kernel": "skyjepa_mma_kernel (split-fp16 tcgen05 GRU rollout, 4 clusters x 16 CTAs)",
                        "kernel_ms": {"mean": round(kmean, 5), "p50": round(percentile(kernel_ms, 0.5), 5)},
                        "kernel_share_of_plan": round(kmean / float(np.mean(times)), 3),
                        "peak_source": ("MEASURED_PEAKS bf16_tflops burst (of measured)" if peaks.get("bf16_tflops")
                                        else "1.59 PFLOP/s bf16 (of fallback)"),
                        "note": "achieved = model FLOP of the rollout (GRU, prober, integrator, cost) per launch / "
                                "mean CUDA-event launch time; the f32-class split executes 3 fp16 products per MAC "
                                "and the 15-step recurrence on 128-row tiles is latency-bound, not throughput-bound"}
        else:
            sgemm = sgemm_peak_tflops(torch)
            flop = FLOP_PER_CANDIDATE_STEP[kind] * cand_steps
            achieved = flop / (percentile(times, 0.5) * 1e-3) / 1e12
            roofline = {"bound": "fp32", "achieved": round(achieved, 3), "peak": round(sgemm, 2),
                        "unit": "TFLOP/s", "frac": round(achieved / sgemm, 4), "traffic": None,
                        "peak_source": "cuBLAS SGEMM 8192^3 (TF32 off) measured in this run",
                        "note": "achieved = algorithmic FLOP per plan / p50 plan time (one fused kernel)"}
        result = {
            "metric": "plan steps/s (one plan of 512 candidates x 15 steps per step); candidate-steps/s and "
                      "p50/p95 plan latency alongside",
            "value": round(plans_per_s, 2),
            "unit": "plans/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 5),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic (seeded random-init weights, generated figure-eight references)",
            "config": default_workload_config(kind, world),
            "timing": "CUDA events around each plan on the planner's stream; L2 flushed between steps "
                      "(256 MiB write outside the timed region)",
            "candidate_steps_per_s": round(plans_per_s * cand_steps, 1),
            "latency_ms": {"p50": round(percentile(times, 0.5), 5), "p95": round(percentile(times, 0.95), 5),
                           "p99": round(percentile(times, 0.99), 5), "max": round(max(times), 5)},
            "e2e": {"value": round(e2e_plans_per_s, 2), "unit": "plans/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h),
                    "latency_ms": {"p50": round(percentile(e2e_times, 0.5), 5),
                                   "p95": round(percentile(e2e_times, 0.95), 5)}},
            "gpu_launches": int(launches * args.steps),
            "roofline": roofline,
            "clocks": clocks.summary(),
        }
        if args.cpu_baseline and world == 1:
            result["cpu_baseline"] = cpu_baseline(kind, args.cpu_seconds)
            result["cpu_baseline_1thread"] = cpu_baseline(kind, min(args.cpu_seconds, 10.0), threads=1)
    planner.close()
    sc.close()
    if args.fleet_record and kind == "skyjepa":
        fleet = fleet_collective_record(args, rank, world, local_rank, ctx)
        if rank == 0:
            result["fleet"] = fleet
    ctx.close()
    if world > 1:
        dist.destroy_process_group()
    return result


def fleet_collective_record(args, rank, world, local_rank, ctx):
    """The fleet across every rank by candidate shards: 256 vehicles x 4096
    candidates x 30 steps, bf16 rollout on the tensor cores, each rank scoring
    4096 / N candidates of every vehicle and reducing them to per-vehicle
    MPPI tuples, one NCCL all-gather of the tuples per plan, then the combine
    kernel.  Times are device times (CUDA events), max over ranks; `t1_ms` is
    the whole fleet planned by one GPU in the same run (rank 0), the
    reference for the per-N overhead; `exchange_ms` is the all-gather alone."""
    import dataclasses
    import torch
    import torch.distributed as dist
    import lewm_b200 as L
    from lewm_b200 import fleet as F
    from lewm_b200 import workloads as W

    V, S, T = 256, 4096, 30
    steps, warmup = max(5, min(args.steps, 20)), 3
    parts = F.partition(V, S, world, "candidates")
    group = F.new_groups(parts) if world > 1 else None
    part = parts[rank]
    full = W.fleet(seed=23, vehicles=V, samples=S, horizon=T)
    stream = ctx.torch_stream()
    sc = L.SkyJepaScorer(ctx, full.model, full.weights, full.state_mean, full.state_std, full.action_mean,
                         full.action_std, full.cost, full.dt)
    sc.set_precision("bf16")
    sc.set_context(full.state_history, full.action_history, full.reference_states, full.reference_actions,
                   vehicle_mass=full.masses)
    fp = F.FleetPlanner(ctx, part, sc, full.mppi, group, time_exchange=True)
    fp.planner.set_warm_start_sequence(full.warm_start)
    flush = torch.empty(256 * 1024 * 1024 // 4, device="cuda")

    def timed(fn, n):
        out = []
        for _ in range(n):
            with torch.cuda.stream(stream):
                flush.add_(1.0)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            fn()
            e.record(stream)
            e.synchronize()
            out.append(s.elapsed_time(e))
        return out

    for _ in range(warmup):
        fp.plan_device()
    ctx.synchronize()
    fp.exchange_ms()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    with clocks:
        times = timed(fp.plan_device, steps)
    exch = fp.exchange_ms()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    # the whole fleet on one GPU (rank 0 only; the others wait at the barrier)
    t1 = None
    if rank == 0:
        if world == 1:
            t1 = times
        else:
            one = L.MppiPlanner(ctx, dataclasses.replace(full.mppi))
            one.set_warm_start_sequence(full.warm_start)
            for _ in range(warmup):
                one.plan_device(sc)
            ctx.synchronize()
            t1 = timed(lambda: one.plan_device(sc), steps)
            one.close()
    if world > 1:
        dist.barrier()
    stats = torch.tensor([float(np.mean(times)), percentile(times, 0.5), percentile(times, 0.95),
                          float(np.mean(exch)) if exch else 0.0], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    mean_ms, p50, p95, exch_ms = stats.tolist()
    fp.close()
    sc.close()
    del flush
    if rank != 0:
        return None
    t1_ms = float(np.mean(t1))
    cand_steps = V * S * T
    peaks = measured_peaks()
    peak = float(peaks.get("bf16_tflops_sustained", 1400.0)) * world
    achieved = FLOP_PER_CANDIDATE_STEP["fleet"] * cand_steps / (mean_ms * 1e-3) / 1e12
    overhead = mean_ms - t1_ms / world
    limiter = ("none: the plan time is within 5 % of the one-GPU time / N" if overhead <= 0.05 * mean_ms else
               "the all-gather of the per-vehicle tuples" if exch_ms >= 0.5 * overhead else
               "per-plan work that does not shrink with N (the per-vehicle history encoder, the combine and "
               "launch latency)")
    return {
        "workload": f"fleet SkyJEPA learned MPPI, {V} vehicles x {S} candidates x {T} steps, bf16 tcgen05 rollout, "
                    "per-vehicle masses",
        "parallelism": f"1 vehicle group x {world} candidate shards ({S // world} candidates of every vehicle "
                       "per rank)",
        "collective": "NCCL all_gather_into_tensor of per-vehicle MPPI tuples (min score, sum of weights, best key, "
                      f"weighted action sums): {V} x {4 + T * 4} floats per rank per plan" if world > 1 else "none",
        "n_gpus": world,
        "steps": steps,
        "ms_per_plan": round(mean_ms, 4),
        "latency_ms": {"p50": round(p50, 4), "p95": round(p95, 4)},
        "fleet_plans_per_s": round(1e3 / mean_ms, 3),
        "candidate_steps_per_s": round(cand_steps * 1e3 / mean_ms, 1),
        "t1_ms": round(t1_ms, 4),
        "exchange_ms": round(exch_ms, 4),
        "exchange_share": round(exch_ms / mean_ms, 4),
        "overhead_ms_vs_t1_over_n": round(overhead, 4),
        "limiter": limiter,
        "roofline": {"bound": "tensor", "achieved": round(achieved, 3), "peak": round(peak, 1), "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4),
                     "peak_source": "MEASURED_PEAKS bf16_tflops_sustained (of measured) x n_gpus"},
        "timing": "CUDA events on the planner's stream, L2 flushed between plans, max over ranks",
        "nccl": {"version": ".".join(str(v) for v in torch.cuda.nccl.version()) if world > 1 else None,
                 "ranks": dist.get_world_size() if world > 1 else 1, "log": NCCL_LOG},
        "clocks": clocks.summary(),
    }


# ------------------------------------------------------------ fleet workload

def run_fleet(args, rank, world, local_rank):
    """Fleet-scale learned MPPI: V vehicles x S candidates x T steps with
    per-vehicle physical parameters, split over the ranks by vehicles and/or
    candidate ranges (lewm_b200.fleet); one step = one plan of the whole fleet."""
    import datetime
    import torch
    import torch.distributed as dist
    import lewm_b200 as L
    from lewm_b200 import fleet as F
    from lewm_b200 import workloads as W

    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", init_method="env://", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    V, S, T = args.vehicles, args.samples, args.horizon
    parts = F.partition(V, S, world, args.shard)
    group = F.new_groups(parts) if world > 1 else None
    part = parts[rank]
    v0, v1 = part.vehicles
    full = W.fleet(seed=23, vehicles=V, samples=S, horizon=T)
    ctx = L.Context(local_rank)
    stream = ctx.torch_stream()
    sl = slice(v0, v1)
    sc = L.SkyJepaScorer(ctx, full.model, full.weights, full.state_mean, full.state_std, full.action_mean,
                         full.action_std, full.cost, full.dt)
    hist, act, refs, ref_a, masses = (full.state_history[sl].copy(), full.action_history[sl].copy(),
                                      full.reference_states[sl].copy(), full.reference_actions[sl].copy(),
                                      full.masses[sl].copy())
    sc.set_precision(args.precision)
    set_ctx = lambda: sc.set_context(hist, act, refs, ref_a, vehicle_mass=masses)
    set_ctx()
    fp = F.FleetPlanner(ctx, part, sc, full.mppi, group)
    fp.planner.set_warm_start_sequence(full.warm_start[sl])
    flush = torch.empty(256 * 1024 * 1024 // 4, device="cuda")

    def one_plan():
        return fp.plan_device()

    if args.loop:
        # the whole control step on the device: history shift + references +
        # prior into the scorer's context, the prior as warm start, the plan,
        # every vehicle's plant (10 substeps of 5 ms) with its first action
        nv = v1 - v0
        p_sh, p_ah, p_rs, p_ra = sc.context_device()
        raw = np.frombuffer(b"".join(bytes(d) for d in full.domains[sl]), dtype=np.float32).reshape(nv, -1)
        d_dom = torch.as_tensor(raw.copy()).cuda()
        d_x = torch.as_tensor(hist[:, -1].copy()).cuda()
        d_m = torch.as_tensor(np.stack([np.full(4, d.hover_force(), np.float32) for d in full.domains[sl]])).cuda()
        loop = {"k": 0, "last": None}
        torch.cuda.synchronize()

        def one_plan():  # noqa: F811 - one control step replaces one plan
            st = L.FleetStep()
            st.batch, st.horizon, st.history = nv, T, full.model.history_steps
            st.time, st.dt = 0.05 * loop["k"], 0.05
            st.reference_kind, st.radius, st.period = 2, 2.0, 8.0
            st.prior_domain = L.Domain.default()
            st.trim, st.state = None, d_x.data_ptr()
            st.last_action, st.last_action_stride = loop["last"], 4
            st.state_history, st.action_history, st.reference_states, st.reference_actions = p_sh, p_ah, p_rs, p_ra
            L.fleet_control_step_device(ctx, st)
            fp.planner.set_warm_start_device(p_ra, nv)
            r = fp.plan_device()
            L.plant_step_device(ctx, d_dom.data_ptr(), d_x.data_ptr(), d_m.data_ptr(), r.first_action, 4, nv,
                                0.005, 10)
            loop["k"] += 1
            loop["last"] = r.first_action
            return r

    for _ in range(args.warmup):
        one_plan()
    ctx.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    n0 = ctx.launch_count()
    times, kernel_ms = [], []
    clocks = ClockSampler(local_rank)
    ctx.set_kernel_timing(True)  # CUDA events around the rollout launch on the library's stream
    with clocks:
        for _ in range(args.steps):
            with torch.cuda.stream(stream):
                flush.add_(1.0)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            one_plan()
            e.record(stream)
            e.synchronize()
            times.append(s.elapsed_time(e))
            kernel_ms.append(ctx.kernel_time_ms())
    ctx.set_kernel_timing(False)
    launches = (ctx.launch_count() - n0) // args.steps
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    # end to end: host context in, host first actions out
    e2e_times = []
    for _ in range(args.steps):
        ctx.synchronize()
        t0 = time.perf_counter()
        set_ctx()
        r = one_plan()
        with torch.cuda.stream(stream):  # the copy waits for the plan on the library's stream
            first = L.device_tensor(r.first_action, (v1 - v0, 4)).cpu()
        e2e_times.append((time.perf_counter() - t0) * 1e3)
    h2d = hist.nbytes + act.nbytes + refs.nbytes + ref_a.nbytes + masses.nbytes
    d2h = first.numel() * 4
    stats = torch.tensor([max(times), sum(times), float(np.mean(e2e_times)), float(np.mean(kernel_ms))],
                         dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    _, total_ms, e2e_mean, kernel_mean = stats.tolist()
    result = None
    if rank == 0:
        cand_steps = V * S * T
        ms = total_ms / args.steps
        plans_per_s = 1e3 / ms
        achieved = FLOP_PER_CANDIDATE_STEP["fleet"] * cand_steps / (ms * 1e-3) / 1e12
        if args.precision == "bf16":
            # the rollout kernel: this rank's share of the FLOP over its own device time (max over ranks)
            k_achieved = FLOP_PER_CANDIDATE_STEP["fleet"] * cand_steps / world / (kernel_mean * 1e-3) / 1e12
            peaks = measured_peaks()
            peak = float(peaks.get("bf16_tflops_sustained", 1400.0))
            roof = {"bound": "tensor", "kernel": "skyjepa_tc_kernel", "achieved": round(k_achieved, 3),
                    "peak": round(peak, 1), "unit": "TFLOP/s", "frac": round(k_achieved / peak, 4), "traffic": None,
                    "peak_source": "MEASURED_PEAKS bf16_tflops_sustained (of measured), one GPU",
                    "note": "achieved = algorithmic FLOP of the learned rollout on one rank / the rollout kernel's "
                            "CUDA-event time (max over ranks)",
                    "kernel_ms": round(kernel_mean, 4), "kernel_share_of_plan": round(kernel_mean / ms, 3),
                    "plan_achieved": round(achieved, 3),
                    "plan_frac": round(achieved / (peak * world), 4)}
        else:
            sgemm = sgemm_peak_tflops(torch)
            roof = {"bound": "fp32", "achieved": round(achieved, 3), "peak": round(sgemm * world, 2),
                    "unit": "TFLOP/s", "frac": round(achieved / (sgemm * world), 4), "traffic": None,
                    "peak_source": "cuBLAS SGEMM 8192^3 (TF32 off) measured in this run, x n_gpus"}
        result = {
            "metric": (f"fleet closed-loop control steps/s ({V} vehicles: context, warm start, plan of {S} "
                       f"candidates x {T} steps, 10 plant substeps per step, all on the device)" if args.loop else
                       f"fleet plan steps/s ({V} vehicles x {S} candidates x {T} steps per step); "
                       "candidate-steps/s alongside"),
            "value": round(plans_per_s, 4),
            "unit": "fleet plans/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 3),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": args.precision,
            "data": "synthetic (seeded random-init weights, sampled vehicle masses/arms/motor constants)",
            "config": {"workload": f"fleet SkyJEPA learned MPPI, {V} vehicles x {S} candidates x {T} steps, "
                                   "latent 256, TCN [128,128,128]/[4,4,4], prober 32x2, per-vehicle mass, "
                                   + ("bf16 weights on tcgen05 tensor cores" if args.precision == "bf16"
                                      else "f32"),
                       "parallelism": f"{part.vehicle_groups} vehicle groups x {part.candidate_shards} candidate "
                                      f"shards ({args.shard})",
                       "l2": "flushed between steps (256 MiB write outside the timed region)"},
            "candidate_steps_per_s": round(plans_per_s * cand_steps, 1),
            "latency_ms": {"p50": round(percentile(times, 0.5), 3), "p95": round(percentile(times, 0.95), 3)},
            "e2e": {"value": round(1e3 / e2e_mean, 4), "unit": "fleet plans/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h)},
            "gpu_launches": int(launches * args.steps),
            "roofline": roof,
            "clocks": clocks.summary(),
        }
        if args.cpu_baseline:
            result["cpu_baseline"] = cpu_baseline_fleet(full, args.cpu_seconds)
    fp.close()
    sc.close()
    ctx.close()
    if world > 1:
        dist.destroy_process_group()
    return result


def cpu_baseline_fleet(w, budget_s: float):
    """The oracle on a bounded sample of the fleet: whole-vehicle plans (all S
    candidates x T steps) one vehicle at a time until the budget is spent;
    reported as candidate-steps/s and the fleet plans/s it implies."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import dataclasses
    import oracle as O
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    m = O.SkyJepaModel(w.model, w.weights)
    done, t_used = 0, 0.0
    while t_used < budget_s and done < w.batch:
        b = slice(done, done + 1)
        c = m.score_ctx((w.state_mean, w.state_std, w.action_mean, w.action_std), w.state_history[b],
                        w.action_history[b], w.reference_states[b], w.reference_actions[b], w.cost, w.dt,
                        masses=w.masses[b])
        t0 = time.perf_counter()
        O.mppi_plan(dataclasses.replace(w.mppi), 1, (O.SKYJEPA_FN, c), seed=w.mppi.seed,
                    warm_start=w.warm_start[b])
        t_used += time.perf_counter() - t0
        done += 1
    per_vehicle = t_used / done
    cand_steps = w.samples * w.horizon
    return {"value": round(1.0 / (per_vehicle * w.batch), 6), "unit": "fleet plans/s", "cores": threads,
            "kind": "port", "candidate_steps_per_s": round(cand_steps / per_vehicle, 1),
            "sample": f"{done} whole-vehicle plans ({w.samples} x {w.horizon}) of the fleet, oracle C "
                      f"restatement, {threads} OpenMP threads; fleet rate = vehicle rate / {w.batch}"}


# ------------------------------------------------------------ LeWM workloads

def lewm_flop_per_candidate_step(c) -> float:
    """Algorithmic FLOP of one rolled-out candidate step (one-frame window:
    the attention output is V, so only the V projection is counted)."""
    D, hid, inner = c.embed_dim, c.pred_hidden_dim, c.heads * c.dim_head
    mac = c.action_dim * c.smoothed_dim + c.smoothed_dim * c.action_mlp_scale * D + c.action_mlp_scale * D * D
    mac += c.depth * (6 * hid * hid + 2 * inner * hid + 2 * c.mlp_dim * hid)
    mac += 2 * D * c.pred_proj_hidden
    return 2.0 * mac


def run_lewm(args, rank, world, local_rank):
    """LeWM planning: `lewm-vector` = CEM over 300 x 5 candidates with a
    16-d observation; `lewm-image` = MPPI over 1024 x 10 candidates whose
    observation and goal are NV12 frames preprocessed and encoded by the ViT
    inside every plan.  Replicas for N > 1 (one vehicle does not shard)."""
    import datetime
    import torch
    import torch.distributed as dist
    import lewm_b200 as L
    from lewm_b200 import workloads as W

    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", init_method="env://", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    image = args.workload == "lewm-image"
    w = W.lewm_image(seed=31 + rank) if image else W.lewm_vector(seed=31 + rank)
    ctx = L.Context(local_rank)
    stream = ctx.torch_stream()
    sc = L.LewmScorer(ctx, w.config, w.weights)
    sc.set_precision(args.precision)
    planner = (L.MppiPlanner if image else L.CemPlanner)(ctx, w.planner)
    D = w.config.embed_dim
    if image:
        prep = L.ImagePreprocess.imagenet_224()
        s_img = w.config.image_size
        host_y = torch.from_numpy(np.concatenate([w.y_plane, w.goal_y])).pin_memory()
        host_uv = torch.from_numpy(np.concatenate([w.uv_plane, w.goal_uv])).pin_memory()
        dev_y = torch.empty(host_y.shape, dtype=torch.uint8, device="cuda")
        dev_uv = torch.empty(host_uv.shape, dtype=torch.uint8, device="cuda")
        h2d = host_y.numel() + host_uv.numel()
    else:
        host_obs = torch.from_numpy(np.concatenate([w.obs, w.goal_obs])).pin_memory()
        dev_obs = torch.empty(host_obs.shape, device="cuda")
        h2d = host_obs.numel() * 4
    with torch.cuda.stream(stream):
        if image:
            dev_y.copy_(host_y)
            dev_uv.copy_(host_uv)
        else:
            dev_obs.copy_(host_obs)
    ctx.synchronize()

    def encode_and_plan(upload: bool):
        if image:
            if upload:
                with torch.cuda.stream(stream):
                    dev_y.copy_(host_y, non_blocking=True)
                    dev_uv.copy_(host_uv, non_blocking=True)
            # one control step: NV12 preprocessing straight into the ViT's patch
            # matrix, the encoder beside sampling and the AdaLN tables, then the plan
            return planner.plan_nv12_device(sc, dev_y, dev_uv, w.batch, 1, s_img, s_img, "bt601-video", prep)
        with torch.cuda.stream(stream):
            if upload:
                dev_obs.copy_(host_obs, non_blocking=True)
            emb = sc.encode_vector(dev_obs)
            sc.set_context_device(emb[:1, None, :].contiguous(), emb[1:].contiguous())
        return planner.plan_device(sc)

    flush = torch.empty(256 * 1024 * 1024 // 4, device="cuda")
    for _ in range(args.warmup):
        encode_and_plan(False)
    ctx.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    n0 = ctx.launch_count()
    times = []
    clocks = ClockSampler(local_rank)
    with clocks:
        for _ in range(args.steps):
            with torch.cuda.stream(stream):
                flush.add_(1.0)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            encode_and_plan(False)
            e.record(stream)
            e.synchronize()
            times.append(s.elapsed_time(e))
    launches = (ctx.launch_count() - n0) // args.steps
    e2e_times = []
    for _ in range(args.steps):
        ctx.synchronize()
        t0 = time.perf_counter()
        r = encode_and_plan(True)
        with torch.cuda.stream(stream):
            seq = L.device_tensor(r.sequence, (1, w.horizon, w.config.action_dim)).cpu()
        e2e_times.append((time.perf_counter() - t0) * 1e3)
    stats = torch.tensor([sum(times), float(np.mean(e2e_times))], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    total_ms, e2e_mean = stats.tolist()
    result = None
    if rank == 0:
        iters = w.planner.iterations
        cand_steps = w.samples * w.horizon * iters
        ms = total_ms / args.steps
        plans_per_s = world * 1e3 / ms
        flop = lewm_flop_per_candidate_step(w.config) * cand_steps
        achieved = flop / (percentile(times, 0.5) * 1e-3) / 1e12
        if args.precision == "bf16":
            peak = float(measured_peaks().get("bf16_tflops", 1590.0))
            roof = {"bound": "tensor", "peak_source": "MEASURED_PEAKS bf16_tflops burst (of measured)"}
        else:
            peak = sgemm_peak_tflops(torch)
            roof = {"bound": "fp32", "peak_source": "cuBLAS SGEMM 8192^3 (TF32 off) measured in this run"}
        name = ("LeWM image MPPI: NV12 224x224 obs + goal -> preprocess -> ViT-Tiny (patch 16, 12 x 192) -> "
                "projector; predictor depth 6, 16 x 64 heads, MLP 2048; 1024 candidates x 10 steps, lambda 0.5"
                if image else
                "LeWM vector CEM: 16-d obs + goal -> VectorMlp 512 -> 192; predictor depth 4, 8 x 32 heads, MLP 768; "
                "300 candidates x 5 steps, 30 elites, 3 iterations")
        result = {
            "metric": "plan steps/s (one plan per step, observation/goal encoding included); candidate-steps/s "
                      "and p50/p95 plan latency alongside",
            "value": round(plans_per_s, 3), "unit": "plans/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": args.precision,
            "data": "synthetic (seeded random-init weights, seeded observations / NV12 noise frames)",
            "config": {"workload": name, "parallelism": f"replicas x{world}",
                       "gemms": ("bf16 weights and inputs on tcgen05 tensor cores, f32 accumulation and activations"
                                 if args.precision == "bf16" else "f32 CUDA cores"),
                       "l2": "flushed between steps (256 MiB write outside the timed region)"},
            "candidate_steps_per_s": round(plans_per_s * cand_steps, 1),
            "latency_ms": {"p50": round(percentile(times, 0.5), 4), "p95": round(percentile(times, 0.95), 4)},
            "e2e": {"value": round(world * 1e3 / e2e_mean, 3), "unit": "plans/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(seq.numel() * 4)},
            "gpu_launches": int(launches * args.steps),
            "roofline": {"bound": roof["bound"], "achieved": round(achieved, 3), "peak": round(peak, 2),
                         "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "traffic": None,
                         "peak_source": roof["peak_source"],
                         "note": "achieved = predictor FLOP per plan (encoders excluded) / p50 plan time"},
            "clocks": clocks.summary(),
        }
        if args.cpu_baseline:
            result["cpu_baseline"] = cpu_baseline_lewm(w, image, args.cpu_seconds)
    # pinned host buffers used on the library's stream must be released while
    # that stream still exists (the host allocator records events on it)
    ctx.synchronize()
    if image:
        del host_y, host_uv, dev_y, dev_uv
    else:
        del host_obs, dev_obs
    del seq, r
    torch.cuda.synchronize()
    planner.close()
    sc.close()
    ctx.close()
    if world > 1:
        dist.destroy_process_group()
    return result


def cpu_baseline_lewm(w, image: bool, budget_s: float):
    """The oracle's LeWM plan on the host cores (encoding included)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    m = O.LewmModel(w.config, w.weights)
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or not times:
        t0 = time.perf_counter()
        if image:
            pix = O.preprocess_nv12(np.concatenate([w.y_plane, w.goal_y]), np.concatenate([w.uv_plane, w.goal_uv]), 0,
                                    224, 224, mean=(0.485, 0.456, 0.406), std=(0.229, 0.224, 0.225))
            emb = m.encode_pixels(pix)
            ctxo = m.score_ctx(emb[:1, None, :], emb[1:])
            O.mppi_plan(w.planner, 1, (O.LEWM_FN, ctxo), seed=w.planner.seed)
        else:
            emb = m.encode_vector(np.concatenate([w.obs, w.goal_obs]))
            ctxo = m.score_ctx(emb[:1, None, :], emb[1:])
            O.cem_plan(w.planner, 1, (O.LEWM_FN, ctxo), seed=w.planner.seed)
        times.append(time.perf_counter() - t0)
        if len(times) >= 50:
            break
    mean = float(np.mean(times))
    return {"value": round(1.0 / mean, 5), "unit": "plans/s", "cores": threads, "kind": "port",
            "sample": f"{len(times)} full plans (encoding included), oracle C restatement, {threads} OpenMP threads"}


# ------------------------------------------------------------ media workload

# DRAM bytes (read + write) of one staged-kernel launch at 32 full-HD frames,
# f32 output, from a one-pass ncu capture (dram__bytes_read.sum +
# dram__bytes_write.sum) of that launch.  The writes
# fall short of the output size by what is still in the L2 when the kernel ends.
MEDIA_DRAM_BYTES = {("nv12", False, 32): 101.31e6 + 736.08e6, ("rgb", False, 32): 202.08e6 + 736.31e6}


def run_media(args, rank, world, local_rank):
    """NV12 -> normalised NCHW (Nv12Preprocessor, src/media/mod.rs:196-273) for
    a batch of full-HD frames at their own size (ImageNet mean / std): one
    read of the NV12 planes, one write of the planar output per pixel — the
    preprocessing kernel against the HBM roofline.  Inputs and outputs
    (~0.9 GB f32) exceed the L2, so no flush is needed between steps."""
    import torch
    import lewm_b200 as L
    torch.cuda.set_device(local_rank)
    B, H, W = args.frames, 1080, 1920
    bf16 = args.precision == "bf16"
    fmt = args.media_format
    channels = {"nv12": 1.5, "rgb": 3, "rgba": 4}[fmt]
    ctx = L.Context(local_rank)
    stream = ctx.torch_stream()
    g = torch.Generator().manual_seed(7 + rank)
    if fmt == "nv12":
        host_y = torch.randint(0, 256, (B, H, W), dtype=torch.uint8, generator=g).pin_memory()
        host_uv = torch.randint(0, 256, (B, H // 2, W // 2, 2), dtype=torch.uint8, generator=g).pin_memory()
    else:
        host_y = torch.randint(0, 256, (B, H, W, int(channels)), dtype=torch.uint8, generator=g).pin_memory()
        host_uv = torch.empty(0, dtype=torch.uint8).pin_memory()
    dev_y, dev_uv = host_y.cuda(), host_uv.cuda()
    out = torch.empty((B, 3, H, W), dtype=torch.bfloat16 if bf16 else torch.float32, device="cuda")
    cfg = L.ImagePreprocess.make(H, W, (0.485, 0.456, 0.406), (0.229, 0.224, 0.225))
    torch.cuda.synchronize()

    def step():
        if fmt == "nv12":
            L.preprocess_nv12_device(ctx, dev_y, dev_uv, B, H, W, "bt601-video", cfg, out, bf16=bf16)
        else:
            L.preprocess_packed_device(ctx, dev_y, B, H, W, fmt, cfg, out, 0, 0, bf16)

    for _ in range(args.warmup):
        step()
    ctx.synchronize()
    n0 = ctx.launch_count()
    times = []
    clocks = ClockSampler(local_rank)
    with clocks:
        for _ in range(args.steps):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            step()
            e.record(stream)
            e.synchronize()
            times.append(s.elapsed_time(e))
    launches = ctx.launch_count() - n0
    e2e = []
    host_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    for _ in range(max(3, args.steps // 10)):
        ctx.synchronize()
        t0 = time.perf_counter()
        with torch.cuda.stream(stream):
            dev_y.copy_(host_y, non_blocking=True)
            dev_uv.copy_(host_uv, non_blocking=True)
        step()
        with torch.cuda.stream(stream):
            host_out.copy_(out, non_blocking=True)
        ctx.synchronize()
        e2e.append(time.perf_counter() - t0)
    ms = float(np.median(times))
    px = B * H * W
    bytes_per_call = px * (channels + (6 if bf16 else 12))
    achieved = bytes_per_call / (ms * 1e-3) / 1e9
    peak = float(measured_peaks().get("hbm_gbs", 6650.0))
    result = {
        "metric": f"frames/s of {fmt.upper()} -> normalised NCHW preprocessing (1920x1080, batch {B}, same-size output)",
        "value": round(world * B * 1e3 / ms, 1), "unit": "frames/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8->" + ("bf16" if bf16 else "f32"),
        "data": f"synthetic (seeded uniform {fmt.upper()})",
        "config": {"workload": f"{'NV12 bt601-video' if fmt == 'nv12' else fmt.upper()} {W}x{H} x {B} -> NCHW "
                               f"{'bf16' if bf16 else 'f32'}, ImageNet mean/std", "parallelism": f"replicas x{world}",
                   "l2": "not flushed: inputs + outputs exceed the L2"},
        "e2e": {"value": round(world * B / float(np.median(e2e)), 1), "unit": "frames/s",
                "h2d_bytes_per_step": int(host_y.numel() + host_uv.numel()),
                "d2h_bytes_per_step": int(out.numel() * out.element_size())},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": MEDIA_DRAM_BYTES.get((fmt, bf16, B)),
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch of the same "
                                       "workload",
                     "peak_source": "MEASURED_PEAKS hbm_gbs (of measured)",
                     "note": f"achieved = ({channels} B of {fmt.upper()} read + output bytes written) per pixel "
                             "/ p50 time"},
        "clocks": clocks.summary(),
    }
    if args.cpu_baseline and rank == 0 and fmt == "nv12":
        result["cpu_baseline"] = cpu_baseline_media(host_y[:2].numpy(), host_uv[:2].numpy(), args.cpu_seconds)
    del host_y, host_uv, host_out
    ctx.close()
    return result if rank == 0 else None


def cpu_baseline_media(y, uv, budget_s: float):
    """The oracle's C NV12 -> NCHW conversion on the host cores: one frame per
    call, the calls spread over a thread per core (ctypes releases the GIL),
    repeated for about `budget_s` seconds."""
    from concurrent.futures import ThreadPoolExecutor
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    threads = os.cpu_count() or 1
    B, H, W = y.shape
    mean, std = (0.485, 0.456, 0.406), (0.229, 0.224, 0.225)
    outs = [np.empty((1, 3, H, W), np.float32) for _ in range(threads)]

    def one(i):
        O.preprocess_nv12(y[i % B][None], uv[i % B][None], 0, H, W, mean=mean, std=std, out=outs[i % threads])

    frames, t0 = 0, time.perf_counter()
    with ThreadPoolExecutor(threads) as pool:
        while True:
            list(pool.map(one, range(threads)))
            frames += threads
            dt = time.perf_counter() - t0
            if dt >= budget_s:
                break
    return {"value": round(frames / dt, 2), "unit": "frames/s", "cores": threads, "kind": "port",
            "sample": f"{frames} full-HD NV12 frames through the oracle's C preprocessing, one frame per call "
                      f"on {threads} threads"}


# -------------------------------------------------------- closed-loop scenarios

REFERENCE_KINDS = {"hover": 0, "circle": 1, "figure-eight": 2}


def closed_loop_setup(args):
    """The session configuration, the model and the scenario list of the
    closed-loop bench (lewm-bench-skyjepa.rs:215-262): hover / circle /
    figure-eight references x (the nominal domain + `random_domains` sampled
    domains), each flown for `steps` control steps of 50 ms."""
    import lewm_b200 as L
    from lewm_b200 import workloads as W
    cfg = L.SessionConfig.paper()
    cfg.dynamics = L.DYNAMICS["nominal_physics" if args.dynamics == "nominal" else "learned"]
    sky = None
    if args.dynamics == "learned":
        sky = W.skyjepa(seed=37, config=L.SkyJepaConfig.paper())
    domains = [("nominal", L.Domain.default())]
    domains += [(f"sampled-{i}", L.Domain.sample(9001 + 7919 * i)) for i in range(args.random_domains)]
    scenarios = [(kind, name, dom) for kind in REFERENCE_KINDS for name, dom in domains]
    return cfg, sky, scenarios


def run_closed_loop(args, rank, world, local_rank):
    """SkyJEPA closed-loop control through the controller session: every
    control step plans (one synchronised call: context upload, MPPI, result
    download, as SkyJepaControllerSession::plan), the rotor plant advances
    10 substeps of 5 ms on the host with the planned action, and the session
    commits the observation.  Latency = wall time of the plan call."""
    import torch
    import lewm_b200 as L
    torch.cuda.set_device(local_rank)
    cfg, sky, scenarios = closed_loop_setup(args)
    ctx = L.Context(local_rank)
    hover = L.hover_state()
    if sky is None:
        sess = L.SkyJepaSession(ctx, cfg, hover)
    else:
        sess = L.SkyJepaSession(ctx, cfg, hover, sky.model, sky.weights, sky.state_mean, sky.state_std,
                                sky.action_mean, sky.action_std)
    dt = cfg.dt
    refs0 = L.reference_horizon("hover", 0.0, dt, cfg.horizon, 2.0, 8.0)
    for _ in range(args.warmup):  # SkyJepaControllerSession::warm_up: plan, then reset
        sess.plan(refs0)
    times, rmses, launches = [], [], 0
    n0 = ctx.launch_count()
    kinds = {v: k for k, v in REFERENCE_KINDS.items()}
    clocks = ClockSampler(local_rank)
    with clocks:
        for kind, _name, dom in scenarios:
            x = L.hover_state()
            motors = np.full(4, dom.mass * dom.gravity / 4, np.float32)
            sess.reset_with_action(x, motors)  # the plant's nominal hover action
            err2 = 0.0
            for step in range(args.steps):
                t = step * dt
                refs = L.reference_horizon(kind, t, dt, cfg.horizon, 2.0, 8.0)
                t0 = time.perf_counter()
                plan = sess.plan(refs)
                times.append((time.perf_counter() - t0) * 1e3)
                for _ in range(10):
                    L.plant_step(dom, x, motors, plan.action, dt / 10)
                sess.commit_observation(x, plan.action)
                ref = L.reference_horizon(kind, t, dt, 1, 2.0, 8.0)[0]
                err2 += float(np.sum((x[:3] - ref[:3]) ** 2))
            rmses.append((err2 / args.steps) ** 0.5)
    launches = ctx.launch_count() - n0
    sess.close()
    ctx.close()
    if rank != 0:
        return None
    mean = float(np.mean(times))
    T, S = cfg.horizon, cfg.samples
    model = ("nominal rotor physics (10 substeps)" if sky is None else
             "SkyJEPA paper-derived model (latent 24, TCN [8,8,16]/[4,4,8], prober 32x2), random-init weights")
    result = {
        "metric": "closed-loop plan latency p95 (ms) and plans/s; 512 candidates x 15 steps, 1 MPPI iteration, "
                  "one synchronised session plan per 50 ms control step",
        "value": round(world * 1e3 / mean, 3), "unit": "plans/s", "n_gpus": world, "steps": len(times),
        "warmup": args.warmup, "ms_per_step": round(mean, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded random-init weights, generated references, sampled domains)",
        "config": {"workload": f"closed-loop SkyJEPA MPPI session, {model}; {len(scenarios)} scenarios "
                               f"(hover / circle / figure-eight x nominal + {args.random_domains} sampled domains) "
                               f"x {args.steps} control steps",
                   "parallelism": f"replicas x{world}", "l2": "not flushed: the session's working set is "
                   "far below L2; the plant and the host bookkeeping run between plans"},
        "latency_ms": {"p50": round(percentile(times, 0.5), 4), "p95": round(percentile(times, 0.95), 4),
                       "p99": round(percentile(times, 0.99), 4), "max": round(max(times), 4)},
        "candidate_steps_per_s": round(world * 1e3 / mean * S * T, 1),
        "tracking": {"position_rmse_m_median": round(float(np.median(rmses)), 4),
                     "position_rmse_m_max": round(float(np.max(rmses)), 4),
                     "scenarios_within_0.75m": int(sum(r <= 0.75 for r in rmses))},
        "reference_published_p95_ms": {"random-weight SkyJEPA MPPI": 8.931, "nominal-physics MPPI": 3.215,
                                       "hardware": "RTX 4090 (shared)"},
        "e2e": {"value": round(world * 1e3 / mean, 3), "unit": "plans/s",
                "h2d_bytes_per_step": int(4 * (T * 18 + T * 4 + T * 4 + 10 * 18 + 9 * 4)),
                "d2h_bytes_per_step": int(4 * (4 + T * 4 + S + 1))},
        "gpu_launches": int(launches),
        "clocks": clocks.summary(),
    }
    if args.cpu_baseline:
        result["cpu_baseline"] = cpu_baseline_closed_loop(args, args.cpu_seconds)
    return result


def cpu_baseline_closed_loop(args, budget_s: float):
    """The oracle's session (the same closed loop) on the host cores, for a
    bounded number of control steps of the first scenarios."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    import lewm_b200 as L
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    cfg, sky, scenarios = closed_loop_setup(args)
    sess = O.SkyJepaSession(cfg, L.hover_state(), None if sky is None else
                            (sky.model, sky.weights, (sky.state_mean, sky.state_std, sky.action_mean, sky.action_std)))
    times = []
    t_end = time.perf_counter() + budget_s
    for kind, _name, dom in scenarios:
        x = L.hover_state()
        motors = np.full(4, dom.mass * dom.gravity / 4, np.float32)
        sess.reset_with_action(x, motors)
        for step in range(args.steps):
            refs = O.reference_horizon(REFERENCE_KINDS[kind], step * cfg.dt, cfg.dt, cfg.horizon, 2.0, 8.0)
            t0 = time.perf_counter()
            seq, _, _ = sess.plan(refs)
            times.append((time.perf_counter() - t0) * 1e3)
            for _ in range(10):
                O.plant_step(dom, x, motors, seq[0], cfg.dt / 10)
            sess.commit_observation(x, seq[0])
            if time.perf_counter() > t_end:
                break
        if time.perf_counter() > t_end:
            break
    mean = float(np.mean(times))
    return {"value": round(1e3 / mean, 4), "unit": "plans/s", "cores": threads, "kind": "port",
            "sample": f"{len(times)} closed-loop session plans (oracle session, C planner and scorer, "
                      f"{threads} OpenMP threads)",
            "latency_ms": {"p50": round(percentile(times, 0.5), 3), "p95": round(percentile(times, 0.95), 3)}}


# ----------------------------------------------------------------- CPU arm

def cpu_baseline(kind: str, budget_s: float, threads: int = 0):
    """The oracle (C restatement of the reference's CPU path) on the host cores,
    on the workload built from the oracle alone (oracle/workload.py: the same
    arrays as the product's generator, without loading the product)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    import workload as W
    threads = threads or os.cpu_count() or 1
    O.set_threads(threads)
    if kind == "skyjepa":
        w = W.skyjepa(seed=17)
        m = O.SkyJepaModel(w.model, w.weights)
        c = m.score_ctx((w.state_mean, w.state_std, w.action_mean, w.action_std), w.state_history,
                        w.action_history, w.reference_states, w.reference_actions, w.cost, w.dt)
        scorer = (O.SKYJEPA_FN, c)
    else:
        w = W.nominal(seed=17)
        scorer = (O.NOMINAL_FN, O.nominal_ctx(w.initial, w.motors, w.reference_states, w.reference_actions, w.cost,
                                              w.dt, w.trim))
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 2:
        t0 = time.perf_counter()
        O.mppi_plan(w.mppi, 1, scorer, seed=w.mppi.seed, warm_start=w.warm_start)
        times.append(time.perf_counter() - t0)
        if len(times) >= 200:
            break
    mean = float(np.mean(times))
    return {"value": round(1.0 / mean, 4), "unit": "plans/s", "cores": threads, "kind": "port",
            "sample": f"{len(times)} full plans of the same workload (512 x 15, 1 iteration), "
                      f"oracle C restatement, {threads} OpenMP threads",
            "latency_ms": {"p50": round(percentile([t * 1e3 for t in times], 0.5), 3),
                           "p95": round(percentile([t * 1e3 for t in times], 0.95), 3)}}


def run_reference(args, rank, world):
    if rank != 0:
        return None
    if args.workload == "fleet":
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import workload as OW  # the fleet built from the oracle alone
        base = cpu_baseline_fleet(OW.fleet(seed=23, vehicles=args.vehicles, samples=args.samples,
                                           horizon=args.horizon), args.cpu_seconds)
        return {"impl": "reference",
                "metric": f"fleet plan steps/s ({args.vehicles} vehicles x {args.samples} candidates x "
                          f"{args.horizon} steps per step); candidate-steps/s alongside",
                "value": base["value"], "unit": "fleet plans/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(1e3 / base["value"], 3), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded random-init weights, sampled vehicle masses/arms/motor constants)",
                "config": {"workload": "fleet SkyJEPA learned MPPI", "parallelism": "host CPU"},
                "candidate_steps_per_s": base["candidate_steps_per_s"], "cpu_baseline": base,
                "e2e": {"value": base["value"], "unit": "fleet plans/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
    if args.workload == "closed-loop":
        base = cpu_baseline_closed_loop(args, args.cpu_seconds)
        return {"impl": "reference", "metric": "closed-loop plan latency p95 (ms) and plans/s; 512 candidates x 15 "
                "steps, 1 MPPI iteration, one synchronised session plan per 50 ms control step",
                "value": base["value"], "unit": "plans/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(1e3 / base["value"], 3), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded random-init weights, generated references, sampled domains)",
                "config": {"workload": f"closed-loop SkyJEPA MPPI session ({args.dynamics})",
                           "parallelism": "host CPU"},
                "latency_ms": base["latency_ms"], "cpu_baseline": base,
                "e2e": {"value": base["value"], "unit": "plans/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if args.workload == "media":
        g = np.random.default_rng(7)
        y = g.integers(0, 256, (2, 1080, 1920), dtype=np.uint8)
        uv = g.integers(0, 256, (2, 540, 960, 2), dtype=np.uint8)
        base = cpu_baseline_media(y, uv, args.cpu_seconds)
        return {"impl": "reference",
                "metric": "frames/s of NV12 -> normalised NCHW preprocessing (1920x1080, batch 32, same-size output)",
                "value": base["value"], "unit": "frames/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(32e3 / base["value"], 3), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "u8->f32", "data": "synthetic (seeded uniform NV12)",
                "config": {"workload": "NV12 bt601-video 1920x1080 x 32 -> NCHW f32, ImageNet mean/std",
                           "parallelism": "host CPU"},
                "cpu_baseline": base,
                "e2e": {"value": base["value"], "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if args.workload.startswith("lewm"):
        from lewm_b200 import workloads as W
        image = args.workload == "lewm-image"
        w = W.lewm_image(seed=31) if image else W.lewm_vector(seed=31)
        base = cpu_baseline_lewm(w, image, args.cpu_seconds)
        return {"impl": "reference", "metric": "plan steps/s (one plan per step, observation/goal encoding "
                "included); candidate-steps/s and p50/p95 plan latency alongside",
                "value": base["value"], "unit": "plans/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(1e3 / base["value"], 3), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded random-init weights, seeded observations / NV12 noise frames)",
                "config": {"workload": args.workload, "parallelism": "host CPU"},
                "candidate_steps_per_s": round(base["value"] * w.samples * w.horizon * w.planner.iterations, 1),
                "cpu_baseline": base,
                "e2e": {"value": base["value"], "unit": "plans/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    base = cpu_baseline(args.workload, args.cpu_seconds)
    # each timed step is one full plan on the host cores
    return {
        "impl": "reference",
        "metric": "plan steps/s (one plan of 512 candidates x 15 steps per step); candidate-steps/s and "
                  "p50/p95 plan latency alongside",
        "value": base["value"],
        "unit": "plans/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(1e3 / base["value"], 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded random-init weights, generated figure-eight references)",
        "config": default_workload_config(args.workload, world),
        "timing": "wall clock around each full plan on the host cores",
        "candidate_steps_per_s": round(base["value"] * 512 * 15, 1),
        "latency_ms": base["latency_ms"],
        "cpu_baseline": base,
        "e2e": {"value": base["value"], "unit": "plans/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["skyjepa", "nominal", "fleet", "lewm-vector", "lewm-image", "closed-loop",
                                           "media"],
                    default="skyjepa")
    ap.add_argument("--shard", choices=["auto", "vehicles", "candidates"], default="auto")
    ap.add_argument("--vehicles", type=int, default=256)
    ap.add_argument("--samples", type=int, default=4096)
    ap.add_argument("--horizon", type=int, default=30)
    ap.add_argument("--loop", action="store_true",
                    help="fleet: time whole control steps on the device (context, warm start, plan, plant)")
    ap.add_argument("--precision", choices=["f32", "bf16"], default=None,
                    help="fleet and lewm-image: bf16 weights on the tensor cores (their default) or f32; "
                         "lewm-vector: f32 (default) or bf16")
    ap.add_argument("--dynamics", choices=["learned", "nominal"], default="learned",
                    help="closed-loop: the paper-derived SkyJEPA model (random init) or the nominal rotor physics")
    ap.add_argument("--random-domains", type=int, default=2,
                    help="closed-loop: sampled domains beside the nominal one (the reference bench uses 20)")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--frames", type=int, default=32, help="media workload: full-HD frames per batch")
    ap.add_argument("--media-format", choices=["nv12", "rgb", "rgba"], default="nv12",
                    help="media workload: NV12 planes or packed RGB / RGBA frames")
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--no-fleet-record", dest="fleet_record", action="store_false",
                    help="default workload: skip the fleet record (256 x 4096 x 30 by candidate shards over all "
                         "ranks, one NCCL all-gather per plan) added to the JSON line")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.precision is None:  # the precision each workload's configuration names
        args.precision = "bf16" if args.workload in ("fleet", "lewm-image") else "f32"
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        out = run_reference(args, rank, world)
    elif args.workload == "fleet":
        out = run_fleet(args, rank, world, local_rank)
    elif args.workload.startswith("lewm"):
        out = run_lewm(args, rank, world, local_rank)
    elif args.workload == "closed-loop":
        out = run_closed_loop(args, rank, world, local_rank)
    elif args.workload == "media":
        out = run_media(args, rank, world, local_rank)
    else:
        out = run_ours(args, rank, world, local_rank)
    if rank == 0 and out is not None:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
