"""GPU parity: every backend against the committed goldens and the CPU oracle.

Mirrors the reference's fixture matrix (reference scripts/validate.py:40-52:
sizes x modes x backend/grid variants, 3W+9 events with a reset before 2W+3)
and its stress pattern (reset every N, state checked at intervals). The
bar is the reference numerical policy (tests/policy.py): fp32 within
1e-5 abs + 1e-4 rel everywhere; fp16 "mixed" within mixed-depth-rms-v3;
bf16 within the same bounds with the declared bf16 relative-L2 gate.
"""
import numpy as np
import pytest

from golden_io import Golden
from gpu_util import BACKENDS, compare_to_oracle, expected_position, replay
from oracle.oracle import Oracle
from policy import check_scores, check_state
from streaming_transformer_b200 import Backend, ModelConfig, Runtime, RuntimeOptions
from streaming_transformer_b200 import synthetic

pytestmark = pytest.mark.gpu


def check_against_golden(g: Golden, options: RuntimeOptions, limit=None):
    events = g.events[:limit] if limit else g.events
    rt = Runtime(g.model, options)
    try:
        scores, hidden, keys, values, positions = replay(
            rt, events, g.resets, [e for e in g.state_events if e < len(events)],
            [e for e in g.hidden_events if e < len(events)])
    finally:
        rt.close()
    c = g.model.config
    n = len(events)
    check_scores(scores, g.expected["scores"][:n], c.layers, g.model.mode, g.name)
    for row, event in enumerate(g.hidden_events):
        if event < n:
            check_state(hidden[event][:, None, :], g.expected["hidden"][row][:, None, :], g.model.mode,
                        f"{g.name} hidden {event}")
            assert positions[event] == expected_position(event, g.resets)
    for row, event in enumerate(g.state_events):
        if event < n:
            check_state(keys[event][g.state_layers], g.expected["keys"][row], g.model.mode, f"{g.name} keys {event}")
            check_state(values[event][g.state_layers], g.expected["values"][row], g.model.mode,
                        f"{g.name} values {event}")
    return scores


@pytest.mark.parametrize("backend", BACKENDS, ids=lambda b: b.name.lower())
@pytest.mark.parametrize("case", ["ref-small-fp32", "ref-small-mixed", "ref-main-fp32", "ref-main-mixed"])
def test_reference_goldens(case, backend):
    check_against_golden(Golden(case), RuntimeOptions(backend=backend, blocks=0))


@pytest.mark.parametrize("case", ["c1-small-fp32", "c1-small-bf16", "c2-main-fp32"])
@pytest.mark.parametrize("backend", [Backend.GRAPH, Backend.PERSISTENT], ids=lambda b: b.name.lower())
def test_benchmark_shape_goldens(case, backend):
    check_against_golden(Golden(case), RuntimeOptions(backend=backend, blocks=0))


@pytest.mark.parametrize("blocks", [1, 4, 0])
@pytest.mark.parametrize("backend", [Backend.CUDA, Backend.FUSED, Backend.PERSISTENT], ids=lambda b: b.name.lower())
def test_grid_sizes(backend, blocks):
    # reference tests ran blocks 1/4/110; 0 = one CTA per SM here.
    check_against_golden(Golden("ref-small-mixed"), RuntimeOptions(backend=backend, blocks=blocks), limit=140)


@pytest.mark.parametrize("mapped", [False, True])
@pytest.mark.parametrize("backend", [Backend.CUDA, Backend.GRAPH, Backend.FUSED], ids=lambda b: b.name.lower())
def test_mapped_transport(backend, mapped):
    check_against_golden(Golden("ref-small-fp32"), RuntimeOptions(backend=backend, blocks=0, mapped=mapped), limit=80)


@pytest.mark.parametrize("mode", ["fp32", "mixed", "bf16"])
@pytest.mark.parametrize("window", [1, 7, 32, 33, 64, 128])
def test_window_sweep_against_oracle(mode, window):
    # Ragged valid lengths, ring wrap-around and a reset, head_dim 64.
    c = ModelConfig(2, 128, 2, 256, window, 32, 1e-6)
    model = synthetic.make_model(c, mode, seed=window)
    events = synthetic.make_events(2 * window + 12, 32, seed=window + 1)
    compare_to_oracle(model, events, RuntimeOptions(backend=Backend.FUSED, blocks=0),
                      resets=(window + 5,), check_every=max(1, window // 4))


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_main_shape_long_run_against_oracle(mode):
    # C2 / C3 shape (d512, L8, hd64, W128) over more than two ring revolutions.
    config, _ = synthetic.CONFIGS["c2-main-fp32"]
    model = synthetic.make_model(config, mode, seed=42)
    events = synthetic.make_events(300, 32, seed=7)
    compare_to_oracle(model, events, RuntimeOptions(backend=Backend.PERSISTENT, blocks=0), resets=(270,),
                      check_every=50)


@pytest.mark.parametrize("mode", ["fp32", "mixed"])
def test_odd_shapes_take_the_scalar_paths(mode):
    # features 33 and width 6 (head_dim 2) exercise unaligned rows.
    c = ModelConfig(2, 6, 3, 10, 5, 33, 1e-5)
    model = synthetic.make_model(c, mode, seed=5)
    events = synthetic.make_events(20, 33, seed=6)
    compare_to_oracle(model, events, RuntimeOptions(backend=Backend.FUSED, blocks=0), resets=(13,))


def test_fp32_is_bit_stable_across_runs_and_backends():
    # Fixed reduction orders: a kernel family gives the same bits on every run.
    # GRAPH runs the per-op kernels; FUSED and PERSISTENT run the single-stream
    # flow kernel at this shape, whose sums are associated differently, so the
    # two families agree within the fp32 policy rather than bit for bit.
    g = Golden("c1-small-fp32")
    runs = {}
    for backend in (Backend.GRAPH, Backend.FUSED, Backend.PERSISTENT, Backend.GRAPH, Backend.FUSED):
        rt = Runtime(g.model, RuntimeOptions(backend=backend, blocks=0))
        try:
            runs.setdefault(backend, []).append(np.array([rt.step(e) for e in g.events[:40]]))
        finally:
            rt.close()
    graph, fused, persistent = runs[Backend.GRAPH], runs[Backend.FUSED], runs[Backend.PERSISTENT]
    np.testing.assert_array_equal(graph[1].view(np.uint32), graph[0].view(np.uint32))
    for r in fused[1:] + persistent:
        np.testing.assert_array_equal(r.view(np.uint32), fused[0].view(np.uint32))
    check_scores(fused[0], graph[0], g.model.config.layers, "fp32", "flow vs per-op")


@pytest.mark.parametrize("backend", [Backend.PERSISTENT, Backend.FUSED], ids=lambda b: b.name.lower())
def test_main_shape_runs_are_bit_identical(backend):
    # The device-loop step exchanges partial sums between clusters while other
    # clusters still run; any race shows as runs that differ in the last bits
    # and drift apart through the K/V ring. 260 events cover two ring revolutions.
    config, _ = synthetic.CONFIGS["c2-main-fp32"]
    model = synthetic.make_model(config, "fp32", seed=42)
    events = synthetic.make_events(260, 32, seed=7)
    runs = []
    for _ in range(2):
        with Runtime(model, RuntimeOptions(backend=backend, blocks=0)) as rt:
            scores = np.array([rt.step(e) for e in events], dtype=np.float32)
            snap = rt.snapshot()
        runs.append((scores, snap.keys, snap.hidden))
    np.testing.assert_array_equal(runs[1][0].view(np.uint32), runs[0][0].view(np.uint32))
    np.testing.assert_array_equal(runs[1][1].view(np.uint32), runs[0][1].view(np.uint32))
    np.testing.assert_array_equal(runs[1][2].view(np.uint32), runs[0][2].view(np.uint32))


def test_device_trace_matches_step_by_step():
    g = Golden("ref-main-mixed")
    for backend in (Backend.GRAPH, Backend.FUSED, Backend.PERSISTENT):
        rt = Runtime(g.model, RuntimeOptions(backend=backend, blocks=0))
        try:
            us, scores = rt.device_trace(g.events[:100], return_scores=True)
            assert us > 0
            snap = rt.snapshot()
        finally:
            rt.close()
        check_scores(scores, g.expected["scores"][:100], g.model.config.layers, "mixed", backend.name)
        assert snap.position == 100
