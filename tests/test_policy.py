"""The numerical policy (tests/policy.py) must pass rounding noise and fail real
mistakes: a K/V row written to the wrong ring slot, two heads swapped, a state
carried with a wrong value. Every mistake is planted in the oracle's state on
the CPU; no GPU is involved."""
from __future__ import annotations

import numpy as np
import pytest

from oracle.oracle import Oracle
from policy import check_scores, check_state, fp32_relative_errors, l2_gate
from streaming_transformer_b200 import synthetic


def _stepped(name: str, extra: int = 5):
    config, mode = synthetic.CONFIGS[name]
    model = synthetic.make_model(config, mode, seed=7)
    oracle = Oracle(model)
    events = synthetic.make_events(config.window + extra, config.features, seed=11)
    scores = oracle.run(events)
    return config, mode, model, oracle, scores


def test_fp32_bound_passes_last_bit_noise():
    config, mode, _, oracle, scores = _stepped("c1-small-fp32")
    keys = oracle.keys()
    rng = np.random.default_rng(3)
    noisy = keys * (1 + rng.choice([-1.0, 1.0], size=keys.shape) * 2.0 ** -23)
    check_state(noisy.astype(np.float32), keys, mode, "keys with one-ulp noise")
    check_scores(scores * np.float32(1 + 2.0 ** -23), scores, config.layers, mode, "scores")


def test_fp32_bound_fails_a_row_in_the_wrong_slot():
    config, mode, _, oracle, _ = _stepped("c1-small-fp32")
    keys = oracle.keys()
    wrong = keys.copy()
    slot = oracle.position % config.window  # the next slot to be written
    # the newest row lands one slot late: slot - 1 keeps its old row
    wrong[1, 2, slot] = keys[1, 2, slot - 1]
    with pytest.raises(AssertionError):
        check_state(wrong, keys, mode, "keys")
    rel = fp32_relative_errors(wrong[1], keys[1])
    assert not rel["passed"] and rel["relative_l2"] > 1e-3


def test_mixed_gate_fails_swapped_heads_even_at_depth():
    config, mode = synthetic.CONFIGS["c4-large-bf16"]
    rng = np.random.default_rng(5)
    layer = config.layers - 1  # the widest depth-scaled gate
    values = rng.standard_normal((config.heads, config.window, config.width // config.heads)).astype(np.float32)
    swapped = values.copy()
    swapped[[0, 1]] = values[[1, 0]]
    assert l2_gate(mode, layer) == pytest.approx(0.016 * 3)
    stacked_ref = np.stack([values] * config.layers)
    stacked_bad = stacked_ref.copy()
    stacked_bad[layer] = swapped
    with pytest.raises(AssertionError):
        check_state(stacked_bad, stacked_ref, mode, "values")


def test_planted_state_mistake_propagates_to_failure():
    """Two oracles step the same events from the same state, except that the
    second lost one value row of layer 0 (a missed ring write, left zero): the
    policy must flag the scores and states of the steps that attend it."""
    config, mode, model, oracle, _ = _stepped("c1-small-fp32")
    position = oracle.position
    keys, values, hidden = oracle.keys(), oracle.values(), oracle.hidden()
    planted = Oracle(model)
    lost = values.copy()
    lost[0, 1, (position - 3) % config.window] = 0
    planted.load_state(position, keys, lost, hidden)
    events = synthetic.make_events(3, config.features, seed=99)
    want = np.array([oracle.step(e) for e in events], dtype=np.float32)
    got = np.array([planted.step(e) for e in events], dtype=np.float32)
    failed = []
    for what, a, b in (("hidden", planted.hidden(), oracle.hidden()),
                       ("keys", planted.keys(), oracle.keys())):
        try:
            check_state(a, b, mode, what)
        except AssertionError:
            failed.append(what)
    try:
        check_scores(got, want, config.layers, mode, "scores")
    except AssertionError:
        failed.append("scores")
    assert {"hidden", "keys"} <= set(failed), failed
