"""Persistent-mailbox stress runs with state hand-off checks (tests/stress.py).

Short versions of the million-command gate (reference scripts/validate.py:55-75:
persistent backend, blocks 1 and 4, a reset every 10007 events): the run crosses
at least two resets, hands the GPU state to the CPU oracle at sampled steps and
compares the replayed scores and state under the reference policy.
"""
import pytest

import stress

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("config,commands,blocks", [
    ("c2-main-fp32", 25_000, 0),
    ("c3-main-bf16", 25_000, 0),
    ("c1-small-fp32", 3_000, 4),
])
def test_stress_with_state_hand_off(config, commands, blocks):
    reset_every = 10007 if commands > 20_000 else 1009
    out = stress.run(config, commands=commands, reset_every=reset_every, samples=6, replay=2, blocks=blocks)
    assert out["samples_checked"] == 6
    assert out["resets"] >= 2
    assert out["nonfinite_scores"] == 0
    assert out["passed"], out["failures"]
