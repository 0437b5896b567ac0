"""Far positions, ragged histories and poisoned slots through state hand-off.

Reference patterns (tests/Primitives.cu:15-98, 190-218): positions up to 1e6,
windows 1..512, poisoned unused ring slots and a poisoned other layer. Here the
state is loaded into the GPU runtime and the CPU oracle alike (st_load_state /
Oracle.load_state), one step runs, and results and state must agree.
"""
import numpy as np
import pytest

from oracle.oracle import Oracle
from policy import check_scores, check_state
from streaming_transformer_b200 import Backend, ModelConfig, Runtime, RuntimeOptions
from streaming_transformer_b200 import synthetic
from streaming_transformer_b200.model import round_storage

pytestmark = pytest.mark.gpu

POSITIONS = [0, 1, 30, 31, 32, 63, 64, 65, 254, 255, 256, 257, 511, 512, 1027, 10007, 1000000]


def random_state(c, mode, position, seed, poison=True):
    rng = np.random.default_rng(seed)
    shape = (c.layers, c.heads, c.window, c.head_dim)
    keys = rng.standard_normal(shape).astype(np.float32) * 0.5
    values = rng.standard_normal(shape).astype(np.float32) * 0.5
    valid = min(position + 1, c.window)
    if poison and valid < c.window:
        # Slots past the retained history must never be read.
        keys[:, :, valid:, :] = 10000.0
        values[:, :, valid:, :] = -10000.0
    keys = round_storage(keys, mode).reshape(shape)
    values = round_storage(values, mode).reshape(shape)
    hidden = round_storage(rng.standard_normal((c.layers, c.width)).astype(np.float32), mode).reshape(c.layers, c.width)
    return keys, values, hidden


@pytest.mark.parametrize("mode", ["fp32", "mixed", "bf16"])
@pytest.mark.parametrize("window,hd", [(1, 16), (7, 32), (32, 64), (64, 16), (256, 32), (512, 64)])
def test_far_positions_and_poisoned_slots(mode, window, hd):
    heads = 2
    c = ModelConfig(2, heads * hd, heads, 96, window, 32, 1e-5)
    model = synthetic.make_model(c, mode, seed=window + hd)
    events = synthetic.make_events(3, 32, seed=hd)
    rt = Runtime(model, RuntimeOptions(backend=Backend.FUSED, blocks=0))
    o = Oracle(model)
    try:
        for k, position in enumerate(POSITIONS):
            keys, values, hidden = random_state(c, mode, position, seed=k)
            # the step writes slot position % W; poison only truly unused slots
            rt.load_state(position, keys, values, hidden)
            o.load_state(position, keys, values, hidden)
            got = [rt.step(e) for e in events]
            want = [o.step(e) for e in events]
            snap = rt.snapshot()
            assert snap.position == o.position == position + len(events)
            check_scores(got, want, c.layers, mode, f"t={position}")
            check_state(snap.keys, o.keys(), mode, f"keys t={position}")
            check_state(snap.values, o.values(), mode, f"values t={position}")
            check_state(snap.hidden[:, None, :], o.hidden()[:, None, :], mode, f"hidden t={position}")
    finally:
        rt.close()


def test_rope_at_absolute_positions_matches_oracle():
    # reference tests/Primitives.cu:190-218: t in {0, 255, 10007, 1e6}, fp32 1e-5 + 1e-4 rel.
    c = ModelConfig(1, 128, 4, 64, 2, 32, 1e-5)
    model = synthetic.make_model(c, "fp32", seed=9)
    event = synthetic.make_events(1, 32, seed=10)[0]
    rt = Runtime(model, RuntimeOptions(backend=Backend.CUDA, blocks=0))
    o = Oracle(model)
    try:
        for t in (0, 255, 10007, 1000000):
            keys, values, hidden = random_state(c, "fp32", t, seed=t, poison=False)
            rt.load_state(t, keys, values, hidden)
            o.load_state(t, keys, values, hidden)
            got, want = rt.step(event), o.step(event)
            snap = rt.snapshot()
            slot = t % c.window
            np.testing.assert_allclose(snap.keys[:, :, slot], o.keys()[:, :, slot], atol=1e-5, rtol=1e-4)
            assert abs(got - want) <= 1e-5 + 1e-4 * abs(want)
    finally:
        rt.close()


def test_uniform_attention_is_mean_of_retained_values():
    # reference tests/test_porting_contract.py:24-51 on the GPU: zero Q/K weights
    # make attention the plain mean of the retained V rows, across eviction and reset.
    c = ModelConfig(2, 128, 2, 64, 5, 32, 1e-5)
    t = synthetic.make_tensors(c, 3, std=c.width ** -0.5)  # unit-scale activations, as randn/sqrt(cols)
    for l in range(c.layers):
        t[f"layers.{l}.q"][:] = 0
        t[f"layers.{l}.k"][:] = 0
    from streaming_transformer_b200 import Model
    model = Model.from_tensors(c, "fp32", t)
    events = synthetic.make_events(4 * c.window + 3, 32, seed=173)
    from gpu_util import compare_to_oracle
    compare_to_oracle(model, events, RuntimeOptions(backend=Backend.GRAPH, blocks=0), resets=(2 * c.window + 1,))
