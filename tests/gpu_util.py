"""Helpers shared by the GPU tests: replay an event trace through a Runtime and
through the CPU oracle and compare under the reference policy."""
from __future__ import annotations

import numpy as np

from oracle.oracle import Oracle
from policy import check_scores, check_state
from streaming_transformer_b200 import Backend, Runtime, RuntimeOptions

BACKENDS = [Backend.CUDA, Backend.GRAPH, Backend.FUSED, Backend.PERSISTENT]


def replay(runtime, events, resets=(), state_events=(), hidden_events=None):
    scores, hidden, keys, values, positions = [], {}, {}, {}, {}
    for i, event in enumerate(events):
        if i in resets:
            runtime.reset()
        scores.append(runtime.step(event))
        want_hidden = hidden_events is None or i in hidden_events
        if want_hidden or i in state_events:
            snap = runtime.snapshot()
            positions[i] = snap.position
            if want_hidden:
                hidden[i] = snap.hidden
            if i in state_events:
                keys[i], values[i] = snap.keys, snap.values
    return np.array(scores, dtype=np.float32), hidden, keys, values, positions


def expected_position(i, resets):
    before = [r for r in resets if r <= i]
    return i + 1 - (max(before) if before else 0)


def compare_to_oracle(model, events, options, resets=(), check_every=1):
    """Run the runtime and the oracle side by side; compare scores and full state."""
    rt = Runtime(model, options)
    o = Oracle(model)
    mode = model.mode
    try:
        got, want = [], []
        for i, event in enumerate(events):
            if i in resets:
                rt.reset()
                o.reset()
            got.append(rt.step(event))
            want.append(o.step(event))
            if i % check_every == 0 or i == len(events) - 1:
                snap = rt.snapshot()
                assert snap.position == o.position, (i, snap.position, o.position)
                check_state(snap.hidden[:, None, :], o.hidden()[:, None, :], mode, f"hidden {i}")
                check_state(snap.keys, o.keys(), mode, f"keys {i}")
                check_state(snap.values, o.values(), mode, f"values {i}")
        check_scores(np.array(got), np.array(want), model.config.layers, mode, "scores")
        return np.array(got), np.array(want)
    finally:
        rt.close()
