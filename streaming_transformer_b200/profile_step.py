"""Run a short device-only trace of one configuration, for profilers.

    python -m streaming_transformer_b200.profile_step --config c2-main-fp32 \
        --backend cuda --events 4 [--warmup 2] [--window W] [--timeline | --phases]

Builds the seeded synthetic model of the configuration, steps ``--warmup``
events, then ``--events`` events with st_device_trace (one resident kernel for
the fused/persistent backends, the per-phase kernel sequence for cuda/graph),
and prints the device microseconds per step. Intended to run under
``ncu --clock-control none`` with a small event count; it never starts the
persistent mailbox worker (a kernel that waits for the host must not be
replayed by a profiler).
"""
from __future__ import annotations

import argparse
import json

from . import BACKEND_NAMES, Backend, Runtime, RuntimeOptions, synthetic


def main() -> None:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--config", default="c2-main-fp32", choices=sorted(synthetic.CONFIGS))
    p.add_argument("--backend", default="cuda", choices=["cuda", "graph", "fused", "persistent"])
    p.add_argument("--events", type=int, default=4)
    p.add_argument("--warmup", type=int, default=2)
    p.add_argument("--window", type=int, default=0)
    p.add_argument("--blocks", type=int, default=0)
    p.add_argument("--streams", type=int, default=1, help="streams (more than 1: the batched round)")
    p.add_argument("--steady", action="store_true",
                   help="the timed launch continues from the warm-up's state (device-resident events) instead of "
                        "starting from reset; with --warmup >= window every timed step attends a full window")
    p.add_argument("--timeline", action="store_true",
                   help="per-phase breakdown from CTA 0's clock64() marks (scaled to the measured step time); "
                        "with --streams > 1, the batched round's phases over its last rounds")
    p.add_argument("--phases", action="store_true",
                   help="flow kernel: per-phase cycle sums of every CTA (diagnostic build), median over the "
                        "CTAs that own a head and over the FFN-only CTAs, us per step at --sm-mhz")
    p.add_argument("--sm-mhz", type=float, default=1965.0, help="SM clock for --phases (cycles to us)")
    a = p.parse_args()
    config, mode = synthetic.CONFIGS[a.config]
    if a.window:
        config = synthetic.config_with_window(config, a.window)
    backend = BACKEND_NAMES[a.backend]
    if backend == Backend.PERSISTENT:
        backend = Backend.FUSED  # same device loop, no host-driven worker
    model = synthetic.make_model(config, mode, seed=42)
    if a.streams > 1:
        events = synthetic.make_stream_events(a.streams, a.warmup + a.events, config.features)
    else:
        events = synthetic.make_events(a.warmup + a.events, config.features, seed=123)
    with Runtime(model, RuntimeOptions(backend=backend, blocks=a.blocks), streams=a.streams) as rt:
        if a.steady:
            import numpy as np
            import torch
            dev = torch.from_numpy(np.ascontiguousarray(events, dtype=np.float32)).cuda()
            if a.warmup:
                rt.device_trace_resident(dev.data_ptr(), a.warmup)
            torch.cuda.synchronize()
            us, _ = rt.device_trace_continue(dev[a.warmup:].data_ptr(), a.events)
        else:
            if a.warmup:
                rt.device_trace(events[: a.warmup])
            us = rt.device_trace(events[a.warmup:])
        out = {"config": a.config, "backend": backend.name.lower(), "events": a.events, "streams": a.streams,
               "us_per_step": us, "blocks": rt.info()["blocks"]}
        if a.timeline and a.streams > 1:
            out.update(round_breakdown(rt, events, config, a.sm_mhz))
        elif a.timeline:
            out["phases_us"] = timeline_breakdown(rt, events[a.warmup:], config, us)
        if a.phases:
            out.update(phase_sums(rt, events[a.warmup:], config, a.sm_mhz))
        print(json.dumps(out))


# Tags of the device marks (TimelineTag in csrc/st_step.cuh); each mark is
# clock64() << 8 | tag and charges the interval since the previous mark to its tag.
TAGS = {1: "step_start", 2: "input", 3: "norm1", 4: "ring_wait", 5: "warp_gemv", 6: "qkv_rows", 7: "qkv_shared",
        8: "kv_wait", 9: "merge_heads", 10: "logits_softmax", 11: "pv_broadcast", 12: "partials_shared",
        13: "out_rows", 14: "sync_cluster_arrive", 15: "sync_grid_wait", 16: "residual_heads", 17: "norm2",
        18: "gate_up_rows", 19: "down_partial", 20: "cluster_reduce", 21: "residual_clusters", 22: "step_end",
        23: "ring_release_fill"}


# Phase tags of the flow kernel's cycle sums (FlowMark in csrc/st_flow.cuh); slot 0
# holds the step count, slot 24 the ring waits already inside the phases.
FLOW_TAGS = {1: "step", 2: "input", 4: "qkv", 5: "qkv_recv", 6: "attention", 7: "partials_recv",
             8: "merge", 9: "out", 10: "gather1", 11: "publish2", 12: "norm2", 13: "gate_up", 14: "down",
             15: "down_reduce_recv", 16: "down_publish", 17: "gather2", 18: "publish1", 19: "score",
             20: "kv_prefetch_issue", 21: "norm1_scale", 22: "norm1_gain", 3: "norm1_barrier",
             24: "(ring_wait, inside the phases)"}


def phase_sums(rt, events, config, sm_mhz):
    """Per-phase us per step of the flow kernel's diagnostic build: every CTA sums
    the cycles of each phase over the run (st_device_timeline_cta, cta -1)."""
    import ctypes

    import numpy as np

    from .runtime import _check, _fptr, library
    info = rt.info()
    if not info.get("flow"):
        raise SystemExit("--phases needs the flow kernel (one stream at a benchmark shape, fused backend)")
    grid, cs = info["flow_grid"], info["cluster"]
    e = np.ascontiguousarray(events, dtype=np.float32)
    cap = grid * 32
    marks = np.zeros(cap, dtype=np.int64)
    used = ctypes.c_size_t(0)
    _check(library().st_device_timeline_cta(rt._h, _fptr(e), e.shape[0], -1,
                                            marks.ctypes.data_as(ctypes.POINTER(ctypes.c_longlong)), cap,
                                            ctypes.byref(used)), rt._h)
    m = marks.reshape(grid, 32).astype(np.float64)
    per = m[:, 1:] / np.maximum(m[:, :1], 1) / sm_mhz  # us per step; column i is tag i + 1
    heads = config.heads // int(info.get("tp_size", 1) or 1)
    groups = {"head_ctas": [c for c in range(grid) if c // cs < heads],
              "ffn_only_ctas": [c for c in range(grid) if c // cs >= heads]}
    out = {"sm_mhz": sm_mhz, "steps": int(np.median(m[:, 0]))}
    for label, ctas in groups.items():
        if not ctas:
            continue
        med = np.median(per[ctas], axis=0)
        phases = {FLOW_TAGS.get(i + 1, f"tag{i + 1}"): round(float(med[i]), 2)
                  for i in np.argsort(-med) if med[i] > 0.005}
        total = float(sum(v for k, v in phases.items() if not k.startswith("(")))
        out[label] = {"ctas": len(ctas), "total_us": round(total, 2), "phases_us": phases}
    return out


# Phase tags of the batched round (BatchTag in csrc/st_batch.cuh): each mark
# ends the named phase; "sync" is the wait at a grid barrier.
ROUND_TAGS = {40: "input", 41: "qkv_gemm", 42: "attention", 43: "out_gemm", 44: "residual_norm2",
              45: "gate_up_gemm", 46: "swiglu", 47: "down_gemm", 48: "residual_norm1", 49: "grid_barrier_wait",
              50: "attention_qkv_finish"}


def round_breakdown(rt, events, config, sm_mhz, rounds_kept=40):
    """Per-phase us per round of the batched round from thread 0 of CTA 0, over
    the last ``rounds_kept`` rounds of a run of all ``events`` from reset (the
    windows are full when the run is longer than the window)."""
    import numpy as np
    count = events.shape[0]
    per_round = 12 * config.layers + 4
    cap = 16 * max(1 << 16, count * per_round * 2)
    row = rt.device_timeline(events, capacity=cap, cta=0, warp=0)
    tags = (row & 0xFF).astype(int)
    clocks = row >> 8
    starts = np.flatnonzero(tags == 40)
    if len(starts) < 2:
        return {"round_phases_us": {}}
    keep = min(rounds_kept, len(starts) - 1)
    lo, hi = starts[-keep - 1], starts[-1]
    acc = {}
    for k in range(lo + 1, hi + 1):
        name = ROUND_TAGS.get(int(tags[k]), f"tag{int(tags[k])}")
        acc[name] = acc.get(name, 0) + int(clocks[k] - clocks[k - 1])
    scale = 1.0 / (keep * sm_mhz)
    phases = {n: round(v * scale, 1) for n, v in sorted(acc.items(), key=lambda kv: -kv[1])}
    return {"rounds_kept": keep, "round_us": round((clocks[hi] - clocks[lo]) * scale, 1),
            "round_phases_us": phases}


def timeline_breakdown(rt, events, config, us_per_step):
    """Per-step total of each tag's intervals (median over steps), scaled so one
    step sums to the measured device time per step."""
    import numpy as np
    raw = rt.device_timeline(events).astype(np.int64)
    raw = raw[(raw & 0xFF) != 24]  # chunk issue times are not phase boundaries
    tags = raw & 0xFF
    clocks = raw >> 8
    starts = np.flatnonzero(tags == 1)
    per_step = []
    for i in range(len(starts) - 1):
        seg = slice(starts[i], starts[i + 1] + 1)
        c, t = clocks[seg], tags[seg]
        totals = {}
        for k in range(1, len(c)):
            name = TAGS.get(int(t[k]), f"tag{int(t[k])}")
            if k == len(c) - 1:
                name = "end_of_step"
            totals[name] = totals.get(name, 0) + int(c[k] - c[k - 1])
        per_step.append((int(c[-1] - c[0]), totals))
    if not per_step:
        return {}
    cycles = float(np.median([p[0] for p in per_step]))
    scale = us_per_step / cycles
    names = sorted({n for _, t in per_step for n in t}, key=lambda n: -np.median([t.get(n, 0) for _, t in per_step]))
    out = {n: round(float(np.median([t.get(n, 0) for _, t in per_step])) * scale, 3) for n in names}
    out["implied_sm_mhz"] = round(cycles / us_per_step, 1)
    return out


if __name__ == "__main__":
    main()
