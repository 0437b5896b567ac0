"""Run a short device-only trace of one configuration, for profilers.

    python -m streaming_transformer_b200.profile_step --config c2-main-fp32 \
        --backend cuda --events 4 [--warmup 2] [--window W]

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
        print(json.dumps(out))


LAYER_MARKS = ["norm1", "qkv_rows", "qkv_shared", "attention", "partials_shared", "out_partial",
               "grid_sync_A", "residual_heads", "norm2", "gate_up", "down_partial", "cluster_reduce",
               "grid_sync_B", "residual_clusters"]


def timeline_breakdown(rt, events, config, us_per_step):
    """Median duration of each phase (time since the previous mark) over the
    steps, scaled so one step sums to the measured device time per step."""
    import numpy as np
    marks = rt.device_timeline(events).astype(np.int64)
    per_step = 2 + len(LAYER_MARKS) * config.layers
    steps = len(marks) // per_step
    names = ["step_start", "input"] + [f"{n}" for _ in range(config.layers) for n in LAYER_MARKS]
    durations = {}
    cycles_per_step = []
    for s in range(steps):
        m = marks[s * per_step:(s + 1) * per_step]
        nxt = marks[(s + 1) * per_step] if (s + 1) * per_step < len(marks) else None
        if nxt is not None:
            cycles_per_step.append(nxt - m[0])
        for i in range(1, per_step):
            durations.setdefault(names[i], []).append(m[i] - m[i - 1])
    scale = us_per_step / float(np.median(cycles_per_step)) if cycles_per_step else 1.0 / 1965.0
    summary = {}
    for name, vals in durations.items():
        v = np.asarray(vals, dtype=np.float64)
        per_layer = name in LAYER_MARKS
        # layer marks appear config.layers times per step: report the per-step total
        summary[name] = round(float(np.median(v.reshape(steps, -1).sum(1) if per_layer else v)) * scale, 3)
    summary["other (end of step)"] = round(us_per_step - sum(summary.values()), 3)
    return summary


if __name__ == "__main__":
    main()
