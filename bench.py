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
Steady state: the device arm first steps max(--warmup, window) untimed events
from reset, so every timed step attends over a full window, then times K
events that continue from that state (st_device_trace_continue).

Multi-GPU (torchrun): the single-stream configs do not shard, so every rank
runs an independent replica stream (weak scaling, no collective on the step
path); value = total steps of all ranks / max device time. With --streams S > 1
the S streams are the job's total and are partitioned evenly over the ranks
(S / N each; strong scaling, as the benchmark's C4 line defines it).

Unless --no-c4 is given (or the workload is C4 itself), the line also carries a
"c4" record: Large bf16 with 256 streams in total partitioned over the N GPUs,
stepped by the batched round from a full window, aggregate stream-steps/s
against the per-GPU-count roofline (every GPU reads the whole weights once per
round plus its own streams' K/V). With N >= 2 GPUs (unless --no-c5b) it also
carries a "c5b" record: one Large fp32 stream (W512) tensor-parallel over the N
GPUs (st_create_tp: each GPU its share of the heads and ffn rows, exchanges
over NVLink inside the kernel), device steps/s from a full window, against the
roofline of one GPU's shard of the bytes.
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
                   help="independent streams in total, partitioned evenly over the GPUs (C4: 256); "
                        "1 = one replica stream per GPU")
    p.add_argument("--no-c4", action="store_true", help="skip the C4 256-stream partition record")
    p.add_argument("--c4-rounds", type=int, default=100, help="timed rounds of the C4 record (at most --steps)")
    p.add_argument("--no-c5b", action="store_true", help="skip the C5-B tensor-parallel record (N >= 2)")
    p.add_argument("--c5b-steps", type=int, default=200, help="timed steps of the C5-B record (at most --steps)")
    p.add_argument("--cpu-seconds", type=float, default=15.0, help="CPU baseline sample budget")
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


def workload(args):
    config, mode = synthetic.CONFIGS[args.config]
    if args.window:
        config = synthetic.config_with_window(config, args.window)
    return config, mode


def streams_per_rank(total, world):
    """Streams each rank steps: 1 (a replica) when total is 1, else total / world."""
    if total <= 1:
        return 1
    if total % world:
        raise SystemExit(f"--streams {total} does not split evenly over {world} GPUs")
    return total // world


def rank_streams(rank, S):
    """Global ids of the streams rank `rank` steps when every rank steps S: rank * S + s.
    Stream g's events come from seed seed_base + g, the same at any GPU count."""
    return [rank * S + s for s in range(S)]


def aggregate_rate(world, S, steps, max_elapsed):
    """Whole-job rate: every rank's S streams x steps over the slowest rank's time."""
    return world * S * steps / max_elapsed


def config_json(args, config, mode, working_set, world=1):
    total = max(1, args.streams)
    s = streams_per_rank(total, world)
    per_gpu = ("single stream per GPU" if total == 1 else
               f"{total} streams in total, {s} per GPU")
    return {
        "workload": f"{args.config}: {mode} {per_gpu}, d{config.width} L{config.layers} "
                    f"H{config.heads} hd{config.head_dim} F{config.ffn} W{config.window}, "
                    f"{config.features} features",
        "model": "local-causal pre-RMSNorm transformer (streaming step)",
        "streams_total": total if total > 1 else world,
        "streams_per_gpu": s,
        "global_batch": s * world,
        "seq_len": config.window,
        "steady_state": "timed steps follow max(warmup, window) untimed steps: every timed step attends a full window",
        "parallelism": "streams partitioned across GPUs (independent, no collective)" if total > 1
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
    if info.get("flow"):
        return info.get("resource_kernel", "k4_flow")
    return "k2_trace"


def kernel_label(info, mode, streams):
    name = kernel_name(info)
    if name == "k3_rounds":
        return f"k3_rounds ({mode}, batched round of {streams} streams)"
    if name == "k4_flow":
        return (f"{name} ({mode}, {info.get('clusters')} clusters of {info.get('cluster')} CTAs, "
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
    # as on the device arm, at least a full window of untimed events first
    warm = int(min(max(args.warmup, config.window), 30.0 / per))
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


def guarded_on_all_ranks(run, dist=None, group=None):
    """(result, error) of run() on every rank; the result is kept only when
    every rank's run succeeded, so all ranks report the same outcome (a failed
    record must not end the bench line, nor leave the ranks disagreeing)."""
    result, error = None, None
    try:
        result = run()
    except Exception as exc:
        error = f"{type(exc).__name__}: {exc}"[:400]
    if combine_ranks([0.0 if result else 1.0], dist, group)[0] > 0:
        result = None
        error = error or "the run failed on another rank"
    return result, error


def combine_ranks(values, dist=None, group=None):
    """Max over ranks of each host-side timing (a CPU tensor over the host
    group); identity on one process."""
    import torch
    t = torch.tensor(list(values), dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return [float(x) for x in t]


def c4_roofline(world, peak_gbs):
    """Per-GPU-count roofline of the C4 partition: every GPU reads the whole
    weights once per round plus its own streams' K/V over a full window and
    writes one K/V row per stream and layer; aggregate stream-steps/s."""
    config, mode = synthetic.CONFIGS["c4-large-bf16"]
    per_rank = 256 // world
    per_gpu_bytes = metrics.step_bytes(config, mode, config.window, streams=per_rank)
    round_s = per_gpu_bytes / (peak_gbs * 1e9)
    return 256 / round_s, int(per_gpu_bytes)


def run_rounds(model, config, S, rank, warm, timed, local, seed_base):
    """Batched rounds of S streams: `warm` untimed rounds from reset (filling the
    windows), then `timed` rounds continuing from that state. Returns
    (us per round, kernels launched in the timed region, runtime info)."""
    import torch
    events = np.stack([synthetic.make_events(warm + timed, config.features, seed=seed_base + g)
                       for g in rank_streams(rank, S)], axis=1)
    dev = torch.from_numpy(np.ascontiguousarray(events)).cuda()
    rt = Runtime(model, RuntimeOptions(backend=Backend.FUSED, blocks=0, device=local), streams=S)
    try:
        rt.device_trace_resident(dev.data_ptr(), warm)
        torch.cuda.synchronize()
        stride = S * config.features
        us, launches = rt.device_trace_continue(dev[warm:].data_ptr(), timed)
        info = rt.info()
    finally:
        rt.close()
    del dev
    return us, launches, info, stride


def run_tp_stream(world, rank, local, steps, host):
    """C5-B: one Large fp32 stream over all ranks' GPUs; (us per step, launches, info)."""
    import torch
    from streaming_transformer_b200.tp import torch_tensor_parallel
    config, mode = synthetic.CONFIGS["c5-large-fp32"]
    model = synthetic.make_model(config, mode, seed=42)
    warm = config.window
    events = synthetic.make_events(warm + steps, config.features, seed=321)  # one stream: the same on every GPU
    dev = torch.from_numpy(events).cuda()
    rt = Runtime(model, RuntimeOptions(backend=Backend.FUSED, blocks=0, device=local),
                 tp=torch_tensor_parallel(host))
    try:
        rt.device_trace_resident(dev.data_ptr(), warm)
        torch.cuda.synchronize()
        us, launches = rt.device_trace_continue(dev[warm:].data_ptr(), steps)
        info = rt.info()
    finally:
        rt.close()
    return us, launches, info, config, mode


def c5b_roofline(world, peak_gbs):
    """Bytes one GPU of the tensor-parallel stream reads per step (its 1/N of
    the weights and of the heads' K/V) at the measured peak."""
    config, mode = synthetic.CONFIGS["c5-large-fp32"]
    e = metrics.ELEM_BYTES[mode]
    per_gpu = metrics.weight_bytes(config, mode) / world + 2 * config.layers * config.width * (config.window + 1) * e / world
    return per_gpu / (peak_gbs * 1e9) * 1e6, int(per_gpu)


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
        # ends it. The step path itself has no collective.
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
    total = max(1, args.streams)
    S = streams_per_rank(total, world)
    # Untimed device steps before the timed region: at least a full window.
    Wd = max(W, config.window)
    # stream g = rank * S + s has its own seeded trace
    events = np.stack([synthetic.make_events(K + Wd, config.features, seed=123 + g) for g in rank_streams(rank, S)],
                      axis=1)  # [K + Wd, S, features]
    e2e_lat = []
    with ClockSampler(local) as clocks:
        # One stream: the persistent mailbox (lowest latency). Several streams:
        # FUSED, one batched-round launch per st_step_batch call.
        backend = Backend.PERSISTENT if S == 1 else Backend.FUSED
        rt = Runtime(model, RuntimeOptions(backend=backend, blocks=0, device=local), streams=S)
        step = (lambda e: rt.step(e[0])) if S == 1 else rt.step_batch
        try:
            # ---- e2e through the public API: host events in, host scores out.
            # The warm-up fills the window, so the timed calls are steady state.
            for e in events[:Wd]:
                step(e)
            barrier(device_wide=False)
            t_start = time.perf_counter()
            for e in events[Wd:Wd + K]:
                t0 = time.perf_counter_ns()
                step(e)
                e2e_lat.append((time.perf_counter_ns() - t0) / 1000.0)
            e2e_wall = time.perf_counter() - t_start
            barrier(device_wide=False)
            # ---- device-resident: trace preloaded in HBM, one resident kernel;
            # Wd untimed steps from reset, then K timed steps from that state
            dev_events = torch.from_numpy(np.ascontiguousarray(events)).cuda()
            torch.cuda.synchronize()
            rt.device_trace_resident(dev_events.data_ptr(), Wd)       # warm-up (untimed)
            barrier()
            us, launches = rt.device_trace_continue(dev_events[Wd:].data_ptr(), K)  # us per round of S streams
            barrier()
            info = rt.info()
        finally:
            rt.close()
        del dev_events
        c4 = None
        if not args.no_c4 and args.config != "c4-large-bf16":
            c4_config, c4_mode = synthetic.CONFIGS["c4-large-bf16"]
            c4_model = synthetic.make_model(c4_config, c4_mode, seed=42)
            c4_S = 256 // world
            c4_K = max(1, min(K, args.c4_rounds))
            barrier()
            c4_us, c4_launches, c4_info, _ = run_rounds(c4_model, c4_config, c4_S, rank, c4_config.window, c4_K,
                                                        local, 7000)
            barrier()
            c4 = (c4_us, c4_K, c4_S, c4_launches, c4_info, c4_config, c4_mode)
        c5b = None
        c5b_error = None
        if world > 1 and not args.no_c5b:
            c5b_K = max(1, min(K, args.c5b_steps))
            barrier()
            c5b, c5b_error = guarded_on_all_ranks(
                lambda: run_tp_stream(world, rank, local, c5b_K, host) + (c5b_K,), dist, host)
            barrier()
    elapsed_s = us * K / 1e6
    times = [elapsed_s, e2e_wall] + ([c4[0] * c4[1] / 1e6] if c4 else []) + ([c5b[0]] if c5b else [])
    maxed = combine_ranks(times, dist, host)
    max_elapsed, max_e2e = maxed[0], maxed[1]
    if dist:
        dist.destroy_process_group()
    if rank != 0:
        return 0
    value = aggregate_rate(world, S, K, max_elapsed)
    peak, peak_src = measured_peak()
    alg = metrics.trace_bytes(config, mode, K, start=Wd, streams=S)
    achieved = alg / K / (us * 1e-6) / 1e9
    traffic, traffic_src = measured_traffic(args.config, kernel_name(info))
    ws = metrics.weight_bytes(config, mode) + S * 2 * config.layers * config.width * config.window * metrics.ELEM_BYTES[mode]
    line = {
        "metric": METRIC, "value": value, "unit": "steps/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": max_elapsed * 1000.0 / K, "higher_is_better": True,
        "scaling": "strong" if total > 1 else "weak",
        "vs_baseline": None, "dtype": mode, "data": "synthetic",
        "config": config_json(args, config, mode, ws, world),
        "mean_us_per_step_device": us,
        "device_warmup_steps": Wd,
        "e2e": {"value": aggregate_rate(world, S, K, max_e2e), "unit": "steps/s", "h2d_bytes_per_step": 4 * config.features * S,
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
    if c4:
        c4_us, c4_K, c4_S, c4_launches, c4_info, c4_config, c4_mode = c4
        c4_value = aggregate_rate(world, c4_S, c4_K, maxed[2])
        roof, per_gpu_bytes = c4_roofline(world, peak)
        line["c4"] = {
            "workload": (f"c4-large-bf16: 256 streams in total, {c4_S} per GPU on {world} GPU(s), d1024 L12 H16 "
                         f"F4096 W256 bf16, batched round, {c4_config.window} untimed rounds then {c4_K} timed"),
            "value": c4_value, "unit": "stream-steps/s", "scaling": "strong", "streams_total": 256,
            "streams_per_gpu": c4_S, "rounds": c4_K, "ms_per_round": maxed[2] * 1000.0 / c4_K,
            "roofline_stream_steps_per_s": roof, "roofline_frac": c4_value / roof,
            "per_gpu_bytes_per_round": per_gpu_bytes, "peak_source": peak_src,
            "kernel": kernel_label(c4_info, c4_mode, c4_S), "gpu_launches": c4_launches,
            "tensor_cores": c4_info.get("batched_tensor_cores"),
        }
    if c5b:
        c5b_us, c5b_launches, c5b_info, c5b_config, c5b_mode, c5b_K = c5b
        c5b_us = maxed[-1]
        roof_us, per_gpu_bytes = c5b_roofline(world, peak)
        line["c5b"] = {
            "workload": (f"c5-large-fp32 phase B: one stream, d1024 L12 H16 F4096 W512 fp32, tensor-parallel over "
                         f"{world} GPUs ({16 // world} heads and {4096 // world} ffn rows each), {c5b_config.window} "
                         f"untimed steps then {c5b_K} timed"),
            "value": 1e6 / c5b_us, "unit": "steps/s", "us_per_step": c5b_us, "scaling": "strong",
            "roofline_us_per_step": roof_us, "roofline_frac": roof_us / c5b_us,
            "per_gpu_bytes_per_step": per_gpu_bytes, "peak_source": peak_src,
            "kernel": f"k4_flow tensor-parallel ({c5b_info.get('clusters')} clusters of {c5b_info.get('cluster')})",
            "gpu_launches": c5b_launches,
            "exchanges": "out-projection records and down sums stored into every GPU's buffers over NVLink, "
                         "polled locally (no collective library on the step path)",
        }
    if c5b_error:
        line["c5b"] = {"workload": f"c5-large-fp32 phase B: one stream tensor-parallel over {world} GPUs",
                       "error": c5b_error}
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
