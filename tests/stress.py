"""Long persistent-mailbox stress run checked against the CPU oracle at sampled steps.

The reference's stress gate (reference scripts/validate.py:55-75) runs a million
events through the persistent backend with a reset every 10007 events and
compares the GPU's results with a CPU replay of the whole trace (bench/Oracle.cpp,
snapshots every 4096 events). A full CPU replay of a million Large steps takes
hours, so this run checks by state hand-off instead: after a sampled step k the
GPU state (position, K/V ring, hidden) is read with ``Runtime.snapshot``, loaded
into the oracle (``Oracle.load_state``), and the next ``replay`` events are stepped
on both sides; their scores and the state after them must agree under the
reference numerical policy (tests/policy.py). Every snapshot's position is also
checked against the count of steps since the last reset (no drift), and every
score of the run must be finite.

    python tests/stress.py [--config c5-large-fp32] [--commands 1000000]
                           [--reset-every 10007] [--samples 16] [--replay 3]
                           [--blocks 0] [--json out.json]

Prints one JSON line. Exit 0 when every check passed, 2 on a numerical or drift
failure, 1 on an error (reference bench/Main.cpp:464-469).
"""
from __future__ import annotations

import argparse
import json
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
for p in (str(ROOT), str(ROOT / "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

from oracle.oracle import Oracle, cpu_count  # noqa: E402
from policy import score_errors, state_errors  # noqa: E402
from streaming_transformer_b200 import Backend, Runtime, RuntimeOptions, synthetic  # noqa: E402


def sample_points(commands: int, samples: int, replay: int) -> list[int]:
    """Steps after which the state is handed off: spread evenly over the run,
    the last one early enough that its replay window fits."""
    last = commands - replay - 1
    if samples <= 0 or last < 0:
        return []
    if samples == 1:
        return [last]
    return sorted({int(round(j * last / (samples - 1))) for j in range(samples)})


def resets_before(i: int, reset_every: int) -> bool:
    """The reference's --reset-every N: reset before event i when i is a positive multiple of N."""
    return reset_every > 0 and i > 0 and i % reset_every == 0


def run(config: str = "c5-large-fp32", commands: int = 1_000_000, reset_every: int = 10007,
        samples: int = 16, replay: int = 3, blocks: int = 0, seed: int = 123,
        oracle_threads: int = 0) -> dict:
    cfg, mode = synthetic.CONFIGS[config]
    model = synthetic.make_model(cfg, mode)
    events = synthetic.make_events(commands, cfg.features, seed)
    points = sample_points(commands, samples, replay)
    starts = {k: j for j, k in enumerate(points)}
    ends = {k + replay: k for k in points}
    mixed = mode

    rt = Runtime(model, RuntimeOptions(backend=Backend.PERSISTENT, blocks=blocks))
    oracle = Oracle(model, threads=oracle_threads or cpu_count())
    scores = np.empty(commands, dtype=np.float32)
    host_ns = np.empty(commands, dtype=np.int64)
    checks, failures = [], []
    last_reset = 0
    handed = {}
    clock = time.perf_counter_ns
    step = rt.step
    t_run = time.perf_counter()
    try:
        for i in range(commands):
            if resets_before(i, reset_every):
                rt.reset()
                last_reset = i
            t0 = clock()
            scores[i] = step(events[i])
            host_ns[i] = clock() - t0
            if i in starts:
                snap = rt.snapshot()
                want = i + 1 - last_reset
                if snap.position != want:
                    failures.append(dict(kind="position", step=i, position=snap.position, expected=want))
                oracle.load_state(snap.position, snap.keys, snap.values, snap.hidden)
                handed[i] = snap.keys.shape
            if i in ends:
                k = ends[i]
                ref = []
                for e in range(k + 1, i + 1):
                    if resets_before(e, reset_every):
                        oracle.reset()
                    ref.append(oracle.step(events[e]))
                snap = rt.snapshot()
                shape = handed.pop(k)
                result = dict(step=k, replayed=replay,
                              scores=score_errors(scores[k + 1:i + 1], np.array(ref, np.float32),
                                                  cfg.layers, mixed))
                state = {}
                for name, gpu, cpu in (("keys", snap.keys, oracle.keys().reshape(shape)),
                                       ("values", snap.values, oracle.values().reshape(shape)),
                                       ("hidden", snap.hidden[:, None, :],
                                        oracle.hidden().reshape(snap.hidden.shape)[:, None, :])):
                    per_layer = [state_errors(gpu[l], cpu[l], l, mixed) for l in range(cfg.layers)]
                    state[name] = dict(passed=all(r["passed"] for r in per_layer),
                                       max_abs=max(r["max_abs"] for r in per_layer))
                result["state"] = state
                result["position"] = dict(gpu=snap.position, oracle=oracle.position)
                ok = (result["scores"]["passed"] and all(s["passed"] for s in state.values())
                      and snap.position == oracle.position)
                checks.append(result)
                if not ok:
                    failures.append(dict(kind="parity", **result))
        wall = time.perf_counter() - t_run
    finally:
        rt.close()
        oracle.close()

    nonfinite = int(np.count_nonzero(~np.isfinite(scores)))
    if nonfinite:
        failures.append(dict(kind="nonfinite", count=nonfinite))
    us = host_ns / 1e3
    return {
        "config": config, "mode": mode, "backend": "persistent", "blocks": blocks,
        "commands": commands, "reset_every": reset_every, "resets": (commands - 1) // reset_every
        if reset_every > 0 else 0,
        "samples_checked": len(checks), "replay_per_sample": replay,
        "max_score_abs_err": max((c["scores"]["max_abs"] for c in checks), default=0.0),
        "max_state_abs_err": max((s["max_abs"] for c in checks for s in c["state"].values()), default=0.0),
        "nonfinite_scores": nonfinite,
        "host_us_per_step": {"p50": float(np.percentile(us, 50)), "p99": float(np.percentile(us, 99)),
                             "max": float(us.max())},
        "wall_seconds": wall, "steps_per_s_including_checks": commands / wall,
        "passed": not failures, "failures": failures[:5],
    }


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--config", default="c5-large-fp32", choices=sorted(synthetic.CONFIGS))
    ap.add_argument("--commands", type=int, default=1_000_000)
    ap.add_argument("--reset-every", type=int, default=10007)
    ap.add_argument("--samples", type=int, default=16)
    ap.add_argument("--replay", type=int, default=3)
    ap.add_argument("--blocks", type=int, default=0)
    ap.add_argument("--seed", type=int, default=123)
    ap.add_argument("--json", default=None, help="also write the result to this file")
    a = ap.parse_args(argv)
    try:
        out = run(a.config, a.commands, a.reset_every, a.samples, a.replay, a.blocks, a.seed)
    except Exception as exc:  # reference bench/Main.cpp:464-469: errors exit 1
        print(json.dumps({"error": f"{type(exc).__name__}: {exc}"}))
        return 1
    line = json.dumps(out)
    print(line)
    if a.json:
        Path(a.json).write_text(line + "\n")
    return 0 if out["passed"] else 2


if __name__ == "__main__":
    sys.exit(main())
