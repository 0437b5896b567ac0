#!/usr/bin/env python
"""Benchmark of the streaming step on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config NAME]

A step is one event of one stream through ``Runtime::step`` (the reference's
unit, reference bench/Main.cpp:223). The default workload is configs[1] of the
benchmark definition, "c2-main-fp32": Main fp32, single stream, d512 L8 H8
(head_dim 64) F2048 W128, 32 features, seeded N(0, 0.02) weights and N(0, 1)
events (synthetic; no dataset exists for this model).

Arms (both print the same metric/unit/config):
  --impl b200 (default)
    value   device-resident steps/s: the trace is preloaded in HBM and stepped
            by one resident kernel (st_device_trace_resident); CUDA events on
            the runtime's stream bracket exactly K steps; max over ranks.
    e2e     the public API with host buffers: Runtime.step on the persistent
            mailbox backend, K host calls, each copying the event in through
            mapped pinned memory and reading the score back; host clock.
    roofline, cpu_baseline (CPU oracle, 1 thread, bounded sample), clocks.
  --impl reference
    The reference's CPU step. Its Eigen implementation (src/cpu/Cpu.cpp)
    cannot be built here (no Eigen), so the C restatement in oracle/ is timed
    with every host thread, on a bounded sample; rank 0 only.
Multi-GPU (torchrun): the single-stream configs do not shard, so every rank
runs an independent replica stream (weak scaling, no collective on the step
path); value = total steps of all ranks / max device time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from streaming_transformer_b200 import Backend, Runtime, RuntimeOptions  # noqa: E402
from streaming_transformer_b200 import metrics, synthetic  # noqa: E402

METRIC = "p50 µs/step per stream; aggregate steps/s at 1/2/4/8 B200; % of BW roofline"
FALLBACK_HBM_GBS = 6650.0
L2_BYTES = 126 * 1024 * 1024


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20000)
    p.add_argument("--warmup", type=int, default=500)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--config", default="c2-main-fp32", choices=sorted(synthetic.CONFIGS))
    p.add_argument("--window", type=int, default=0, help="override the window (C3 sweep)")
    p.add_argument("--streams", type=int, default=1,
                   help="independent streams per GPU (C4/C5-A: the total is streams x GPUs, partitioned by rank)")
    p.add_argument("--cpu-seconds", type=float, default=15.0, help="CPU baseline sample budget")
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


def workload(args):
    config, mode = synthetic.CONFIGS[args.config]
    if args.window:
        config = synthetic.config_with_window(config, args.window)
    return config, mode


def config_json(args, config, mode, working_set, world=1):
    s = max(1, args.streams)
    per_gpu = "single stream per GPU" if s == 1 else f"{s} streams per GPU"
    return {
        "workload": f"{args.config}: {mode} {per_gpu}, d{config.width} L{config.layers} "
                    f"H{config.heads} hd{config.head_dim} F{config.ffn} W{config.window}, "
                    f"{config.features} features",
        "model": "local-causal pre-RMSNorm transformer (streaming step)",
        "streams_per_gpu": s,
        "global_batch": s * world,
        "seq_len": config.window,
        "parallelism": "streams partitioned across GPUs (independent, no collective)" if s > 1
                       else "replicas (independent streams, no collective)",
        "data": "seeded N(0,0.02) weights, unit norm gains, N(0,1) events",
        "l2": ("working set %.1f MB > 126 MB L2, no flush" % (working_set / 1e6)) if working_set > L2_BYTES
              else ("working set %.1f MB fits in L2; no flush between steps (streaming state carries "
                    "over step to step by design)" % (working_set / 1e6)),
    }


def measured_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        peaks = json.loads(path.read_text())
        return float(peaks["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs (of measured)"
    except (OSError, ValueError, KeyError):
        return FALLBACK_HBM_GBS, "profiling-recipe fallback 6.65 TB/s (of fallback)"


def kernel_name(info):
    """The device-loop kernel the runtime runs for the timed trace."""
    if info.get("batched"):
        return "k3_rounds"
    return "k4_flow" if info.get("flow") else "k2_trace"


def kernel_label(info, mode, streams):
    name = kernel_name(info)
    if name == "k3_rounds":
        return f"k3_rounds ({mode}, batched round of {streams} streams)"
    if name == "k4_flow":
        return (f"k4_flow ({mode}, {info.get('clusters')} clusters of {info.get('cluster')} CTAs, "
                "tagged-record exchanges, producer-warp weight ring)")
    return f"k2_trace ({mode}, {'weight ring' if info.get('weight_ring') else 'direct loads'})"


def measured_traffic(config_name, kernel):
    """DRAM bytes per step of `kernel` on `config_name` from a committed ncu
    capture (profiles/traffic.json), or None when none was taken for it."""
    path = ROOT / "profiles" / "traffic.json"
    try:
        entry = json.loads(path.read_text())[config_name]
        if entry.get("kernel", "k2_trace") != kernel:
            return None, None
        return float(entry["dram_bytes_per_step"]), entry.get("source", "")
    except (OSError, ValueError, KeyError):
        return None, None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples every 200 ms while running."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.device)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, loaded_only=True):
        rows = []
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[4:8]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, flags in rows for i, f in enumerate(flags) if f.lower() == "active"})
        sm = [r[0] for r in rows]
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                "samples": len(rows)}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def time_cpu_oracle(model, events, threads, budget_s, max_steps):
    """Oracle steps/s on `threads` host threads over a bounded sample from reset."""
    from oracle.oracle import Oracle  # CPU baseline only
    o = Oracle(model, threads=threads)
    t0 = time.perf_counter()
    o.run(events[:2])
    per = max((time.perf_counter() - t0) / 2, 1e-6)
    n = int(max(4, min(max_steps, budget_s / per, len(events))))
    o.reset()
    t0 = time.perf_counter()
    o.run(events[:n])
    dt = time.perf_counter() - t0
    return n / dt, n, dt


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    config, mode = workload(args)
    model = synthetic.make_model(config, mode, seed=42)
    from oracle.oracle import Oracle, cpu_count  # the reference arm times the CPU restatement
    threads = cpu_count()
    o = Oracle(model, threads=threads)
    # One step is one event, as on the device arm: W warm-up events (they also
    # fill the window) then K timed events in stream order, each run capped so
    # the whole arm ends within a few minutes.
    probe = synthetic.make_events(2, config.features, seed=122)
    t0 = time.perf_counter()
    o.run(probe)
    per = max((time.perf_counter() - t0) / 2, 1e-6)
    o.reset()
    warm = int(min(args.warmup, 30.0 / per))
    timed = int(max(1, min(args.steps, 150.0 / per)))
    events = synthetic.make_events(warm + timed, config.features, seed=123)
    o.run(events[:warm])
    t0 = time.perf_counter()
    o.run(events[warm:])
    dt = time.perf_counter() - t0
    o.close()
    steps_per_s = timed / dt
    ws = metrics.weight_bytes(config, mode) + 2 * config.layers * config.width * config.window * metrics.ELEM_BYTES[mode]
    sample = (f"{timed} consecutive events of the {args.config} trace after {warm} warm-up events, "
              f"C restatement of the reference CPU step (reference Eigen src/cpu/Cpu.cpp needs Eigen3, absent), "
              f"{threads} threads, {dt:.1f} s")
    if timed < args.steps:
        sample += f"; capped from {args.steps} steps to bound the run"
    if args.streams > 1:
        sample += "; streams are independent, so stream-steps/s is the single-stream rate"
    line = {
        "impl": "reference", "metric": METRIC, "value": steps_per_s, "unit": "steps/s", "n_gpus": args.gpus,
        "steps": timed, "warmup": warm, "ms_per_step": 1000.0 / steps_per_s, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": mode, "data": "synthetic",
        "config": config_json(args, config, mode, ws, world),
        "cpu_baseline": {"value": steps_per_s, "unit": "steps/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": steps_per_s, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def combine_ranks(values, dist=None, group=None):
    """Max over ranks of each host-side timing (a CPU tensor over the host
    group); identity on one process."""
    import torch
    t = torch.tensor(list(values), dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return [float(x) for x in t]


def run_b200(args):
    import torch
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dist = host = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
        # Host-side coordination (barriers, max over ranks) runs over gloo: an
        # NCCL barrier synchronizes the whole device, which would wait for the
        # resident persistent worker of the e2e phase until its idle budget
        # ends it. The step path itself has no collective (replicas).
        host = dist.new_group(backend="gloo", timeout=timedelta(seconds=120))

    def barrier(device_wide=True):
        # While the persistent worker is resident a device-wide synchronize
        # would wait for that kernel, so the e2e phase synchronizes torch's own
        # stream only.
        if device_wide:
            torch.cuda.synchronize()
        else:
            torch.cuda.current_stream().synchronize()
        if dist:
            dist.barrier(group=host)

    config, mode = workload(args)
    model = synthetic.make_model(config, mode, seed=42)
    K, W = max(1, args.steps), max(3, args.warmup)
    S = max(1, args.streams)
    # stream g = rank * S + s has its own seeded trace
    events = np.stack([synthetic.make_events(K + W, config.features, seed=123 + rank * S + s) for s in range(S)],
                      axis=1)  # [K + W, S, features]
    e2e_lat = []
    with ClockSampler(local) as clocks:
        # One stream: the persistent mailbox (lowest latency). Several streams:
        # FUSED, one batched-round launch per st_step_batch call.
        backend = Backend.PERSISTENT if S == 1 else Backend.FUSED
        rt = Runtime(model, RuntimeOptions(backend=backend, blocks=0, device=local), streams=S)
        step = (lambda e: rt.step(e[0])) if S == 1 else rt.step_batch
        try:
            # ---- e2e through the public API: host events in, host scores out
            for e in events[:W]:
                step(e)
            rt.reset()
            barrier(device_wide=False)
            t_start = time.perf_counter()
            for e in events[W:W + K]:
                t0 = time.perf_counter_ns()
                step(e)
                e2e_lat.append((time.perf_counter_ns() - t0) / 1000.0)
            e2e_wall = time.perf_counter() - t_start
            barrier(device_wide=False)
            # ---- device-resident: trace preloaded in HBM, one resident kernel
            dev_events = torch.from_numpy(np.ascontiguousarray(events)).cuda()
            torch.cuda.synchronize()
            rt.device_trace_resident(dev_events.data_ptr(), W)       # warm-up (untimed)
            barrier()
            us, launches = rt.device_trace_resident(dev_events[W:].data_ptr(), K)  # us per round of S streams
            barrier()
            info = rt.info()
        finally:
            rt.close()
    elapsed_s = us * K / 1e6
    max_elapsed, max_e2e = combine_ranks([elapsed_s, e2e_wall], dist, host)
    if dist:
        dist.destroy_process_group()
    if rank != 0:
        return 0
    value = world * S * K / max_elapsed
    peak, peak_src = measured_peak()
    alg = metrics.trace_bytes(config, mode, K, streams=S)
    achieved = alg / K / (us * 1e-6) / 1e9
    traffic, traffic_src = measured_traffic(args.config, kernel_name(info))
    ws = metrics.weight_bytes(config, mode) + S * 2 * config.layers * config.width * config.window * metrics.ELEM_BYTES[mode]
    line = {
        "metric": METRIC, "value": value, "unit": "steps/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": max_elapsed * 1000.0 / K, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": mode, "data": "synthetic",
        "config": config_json(args, config, mode, ws, world),
        "p50_us_per_step_device": us,
        "e2e": {"value": world * S * K / max_e2e, "unit": "steps/s", "h2d_bytes_per_step": 4 * config.features * S,
                "d2h_bytes_per_step": 4 * S, "p50_us": metrics.nearest_rank(e2e_lat, 0.5),
                "p99_us": metrics.nearest_rank(e2e_lat, 0.99),
                "path": ("Runtime.step -> st_step, persistent mailbox, mapped pinned input/score, host clock"
                         if S == 1 else "Runtime.step_batch -> st_step_batch, one batched-round launch (FUSED), "
                         "pinned copies of the S inputs and scores, host clock")},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic,
                     "kernel": kernel_label(info, mode, S),
                     "algorithmic_bytes_per_step": alg / K, "peak_source": peak_src,
                     "traffic_source": traffic_src},
        "gpu_launches": launches,
        "clocks": clocks.summary(),
        "runtime": {"blocks": info.get("blocks"), "threads": info.get("threads"),
                    "registers_per_thread": info.get("registers_per_thread"),
                    "barriers_per_step": info.get("barriers_per_step"), "batched": info.get("batched"),
                    "batched_grid": info.get("batched_grid"), "batched_splits": info.get("batched_splits")},
    }
    if world == 1 and not args.no_cpu_baseline:
        sps, n, dt = time_cpu_oracle(model, events[:, 0], 1, args.cpu_seconds, K)
        line["cpu_baseline"] = {
            "value": sps, "unit": "steps/s", "cores": 1, "kind": "port",
            "sample": f"{n} events from reset, C restatement of the reference CPU step, 1 thread, {dt:.1f} s"}
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
