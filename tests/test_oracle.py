"""Pin the CPU oracle (oracle/st_oracle.c) before trusting it as the GPU checker.

* against every committed golden (tests/golden): the reference's own expected
  archives (fixtures/small-*/expected) and reference/model.py outputs at the
  reference and the B200 benchmark shapes, under the reference policy;
* known-answer tests from the reference suite: roundHalf (tests/Native.cpp:20-21),
  adjacent-pair RoPE (tests/test_porting_contract.py:10-21), uniform attention
  equals the mean of retained values across eviction and reset
  (tests/test_porting_contract.py:24-51), trace on/off gives identical state
  (tests/Native.cpp:61-98).
"""
import math

import numpy as np
import pytest
import torch

from golden_io import ALL_CASES, Golden
from oracle.oracle import Oracle, round_bf16, round_half
from policy import check_scores, check_state
from streaming_transformer_b200.model import Model, ModelConfig
from streaming_transformer_b200 import synthetic


def replay(oracle, golden):
    scores, hidden, keys, values = [], {}, {}, {}
    for i, event in enumerate(golden.events):
        if i in golden.resets:
            oracle.reset()
        scores.append(oracle.step(event))
        if i in golden.hidden_events:
            hidden[i] = oracle.hidden()
        if i in golden.state_events:
            keys[i], values[i] = oracle.keys(), oracle.values()
    return np.array(scores, dtype=np.float32), hidden, keys, values


@pytest.mark.parametrize("case", ALL_CASES)
def test_oracle_matches_golden(case):
    g = Golden(case)
    o = Oracle(g.model)
    scores, hidden, keys, values = replay(o, g)
    c = g.model.config
    check_scores(scores, g.expected["scores"], c.layers, g.model.mode, case)
    for row, event in enumerate(g.hidden_events):
        check_state(hidden[event][:, None, :], g.expected["hidden"][row][:, None, :], g.model.mode,
                    f"{case} hidden {event}")
    for row, event in enumerate(g.state_events):
        for name, got in (("keys", keys[event]), ("values", values[event])):
            want = g.expected[name][row]
            got = got[g.state_layers]
            # one state vector = one [head, slot, head_dim] row; layer on axis 0
            check_state(got, want, g.model.mode, f"{case} {name} {event}")


def test_round_half_known_answers():
    assert round_half(1.0001) == 1.0
    assert math.isinf(round_half(1e10))
    assert round_half(65504.0) == 65504.0
    assert math.isinf(round_half(65520.0))
    assert round_half(65519.0) == 65504.0


def test_round_half_matches_ieee_binary16():
    rng = np.random.default_rng(7)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32) * 10 ** rng.uniform(-9, 5, 20000).astype(np.float32),
                        np.array([0.0, -0.0, 2 ** -24, 2 ** -25, 3 * 2 ** -26, 2 ** -14, 6.1e-5, 1 + 2 ** -11,
                                  1 + 3 * 2 ** -11, 2049.0, 2051.0], dtype=np.float32)]).astype(np.float32)
    want = x.astype(np.float16).astype(np.float32)
    got = np.array([round_half(float(v)) for v in x], dtype=np.float32)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def test_round_bf16_matches_torch():
    rng = np.random.default_rng(8)
    x = (rng.standard_normal(20000) * 10 ** rng.uniform(-30, 30, 20000)).astype(np.float32)
    x = np.concatenate([x, np.array([1 + 2 ** -8, 1 + 3 * 2 ** -8, 3.4e38, -3.4e38, 0.0], dtype=np.float32)])
    want = torch.from_numpy(x).bfloat16().float().numpy()
    got = np.array([round_bf16(float(v)) for v in x], dtype=np.float32)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def tiny_model(mode="fp32", window=5, zero_qk=False, seed=3):
    c = ModelConfig(layers=2, width=8, heads=2, ffn=16, window=window, features=32, epsilon=1e-5)
    t = synthetic.make_tensors(c, seed, std=0.3)
    if zero_qk:
        for l in range(c.layers):
            t[f"layers.{l}.q"][:] = 0
            t[f"layers.{l}.k"][:] = 0
    return Model.from_tensors(c, mode, t)


def test_rope_uses_adjacent_pairs():
    m = tiny_model()
    o = Oracle(m)
    events = synthetic.make_events(8, 32, 5)
    for i in range(7):
        o.step(events[i])
    _, trace = o.step_traced(events[7])  # position 7
    d = m.config.head_dim
    pre = trace["layers.0.q.linear"]
    got = trace["layers.0.q"]
    for h in range(m.config.heads):
        for i in range(0, d, 2):
            angle = 7 * 10000.0 ** (-i / d)
            a, b = pre[h * d + i], pre[h * d + i + 1]
            assert abs(got[h * d + i] - (a * math.cos(angle) - b * math.sin(angle))) < 1e-6
            assert abs(got[h * d + i + 1] - (a * math.sin(angle) + b * math.cos(angle))) < 1e-6


@pytest.mark.parametrize("mode", ["fp32", "mixed", "bf16"])
@pytest.mark.parametrize("window", [1, 5])
def test_uniform_attention_is_mean_of_retained_values(mode, window):
    m = tiny_model(mode, window, zero_qk=True)
    o = Oracle(m)
    events = synthetic.make_events(4 * window + 3, 32, 173)
    history = [[] for _ in range(m.config.layers)]
    for i, event in enumerate(events):
        if i == 2 * window + 1:
            o.reset()
            history = [[] for _ in range(m.config.layers)]
        _, trace = o.step_traced(event)
        for l in range(m.config.layers):
            history[l].append(trace[f"layers.{l}.v"])
            want = np.stack(history[l][-window:]).astype(np.float64).mean(0).astype(np.float32)
            if mode == "mixed":
                want = want.astype(np.float16).astype(np.float32)
            got = trace[f"layers.{l}.attention"]
            tol = 2e-3 if mode == "mixed" else (8e-3 if mode == "bf16" else 1e-6)
            np.testing.assert_allclose(got, want, atol=tol, rtol=tol)


@pytest.mark.parametrize("case", ["ref-small-fp32", "ref-small-mixed", "ref-main-mixed"])
def test_trace_capture_preserves_state(case):
    g = Golden(case)
    a, b = Oracle(g.model), Oracle(g.model)
    count = min(len(g.events), 3 * g.model.config.window + 9)
    for i in range(count):
        if i == 2 * g.model.config.window + 3:
            a.reset()
            b.reset()
        s1 = a.step(g.events[i])
        s2, trace = b.step_traced(g.events[i])
        assert s1 == s2
        pre = trace["input.pre_cast"]
        want = pre.astype(np.float16).astype(np.float32) if g.model.mode == "mixed" else pre
        np.testing.assert_array_equal(trace["input.linear"], want)
    np.testing.assert_array_equal(a.keys(), b.keys())
    np.testing.assert_array_equal(a.values(), b.values())
    np.testing.assert_array_equal(a.hidden(), b.hidden())


def test_threads_do_not_change_results():
    g = Golden("c1-small-fp32")
    a, b = Oracle(g.model, threads=1), Oracle(g.model, threads=4)
    for event in g.events[:10]:
        assert a.step(event) == b.step(event)
    np.testing.assert_array_equal(a.keys(), b.keys())


def test_load_state_hand_off_replays_identically():
    g = Golden("ref-small-fp32")
    a = Oracle(g.model)
    for event in g.events[:70]:
        a.step(event)
    b = Oracle(g.model)
    b.load_state(a.position, a.keys(), a.values(), a.hidden())
    for event in g.events[70:90]:
        assert a.step(event) == b.step(event)
    assert a.position == b.position == 90


def test_streaming_differs_from_recomputed_window():
    # Recomputing only the last W raw events loses higher-layer history
    # (reference tests/test_reference.py:33-35).
    m = tiny_model(window=5)
    events = synthetic.make_events(40, 32, 11)
    o = Oracle(m)
    last = [o.step(e) for e in events][-1]
    fresh = Oracle(m)
    naive = [fresh.step(e) for e in events[-5:]][-1]
    assert abs(naive - last) > 1e-4


def test_stress_sampling_and_reset_schedule():
    import stress
    pts = stress.sample_points(1_000_000, 16, 3)
    assert len(pts) == 16 and pts[0] == 0 and pts[-1] == 1_000_000 - 4
    assert all(b > a for a, b in zip(pts, pts[1:]))
    assert stress.sample_points(3, 4, 3) == []
    assert [i for i in range(30_100) if stress.resets_before(i, 10007)] == [10007, 20014, 30021]
    assert not any(stress.resets_before(i, 0) for i in range(100))
