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
    p.add_argument("--timeline", action="store_true",
                   help="per-phase breakdown from CTA 0's clock64() marks (scaled to the measured step time)")
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
    events = synthetic.make_events(a.warmup + a.events, config.features, seed=123)
    with Runtime(model, RuntimeOptions(backend=backend, blocks=a.blocks)) as rt:
        if a.warmup:
            rt.device_trace(events[: a.warmup])
        us = rt.device_trace(events[a.warmup:])
        out = {"config": a.config, "backend": backend.name.lower(), "events": a.events,
               "us_per_step": us, "blocks": rt.info()["blocks"]}
        if a.timeline:
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
FLOW_TAGS = {1: "step", 2: "input", 3: "norm1", 4: "qkv", 5: "qkv_recv", 6: "attention", 7: "partials_recv",
             8: "merge", 9: "out", 10: "gather1", 11: "publish2", 12: "norm2", 13: "gate_up", 14: "down",
             15: "down_reduce_recv", 16: "down_publish", 17: "gather2", 18: "publish1", 19: "score",
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
