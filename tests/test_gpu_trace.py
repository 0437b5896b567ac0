"""traceStep: per-op snapshots (reference tests/Lifecycle.cu:108-137,
bench/Diagnose.cpp:42-62). Every captured intermediate must agree with the CPU
oracle's capture of the same name, and tracing must not change execution."""
import numpy as np
import pytest

from golden_io import Golden
from oracle.oracle import Oracle
from policy import score_errors, state_errors
from streaming_transformer_b200 import Backend, Runtime, RuntimeOptions, StreamError

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", ["ref-small-fp32", "ref-main-fp32", "ref-main-mixed", "c1-small-bf16"])
def test_trace_matches_oracle_op_by_op(case):
    g = Golden(case)
    rt = Runtime(g.model, RuntimeOptions(backend=Backend.CUDA, blocks=0))
    o = Oracle(g.model)
    try:
        for i, event in enumerate(g.events[:6]):
            got = rt.trace_step(event)
            _, want = o.step_traced(event)
            for name, value in got.items():
                assert name in want, name
                if name == "score.linear":
                    r = score_errors(value, want[name], g.model.config.layers, g.model.mode)
                else:
                    layer = int(name.split(".")[1]) if name.startswith("layers.") else 0
                    r = state_errors(value, want[name], layer, g.model.mode)
                assert r["passed"], (case, i, name, r)
    finally:
        rt.close()


@pytest.mark.parametrize("blocks", [4, 0])
def test_traced_steps_preserve_execution(blocks):
    # reference tests/Lifecycle.cu:108-137: identical scores and identical state.
    g = Golden("ref-main-mixed")
    rt = Runtime(g.model, RuntimeOptions(backend=Backend.CUDA, blocks=blocks))
    try:
        scores = [rt.step(e) for e in g.events[:12]]
        state = rt.snapshot()
        rt.reset()
        for i, e in enumerate(g.events[:12]):
            trace = rt.trace_step(e)
            assert trace["layers.0.attention"].shape == (g.model.config.width,)
            assert scores[i] == trace["score.linear"][0]
        traced = rt.snapshot()
        assert traced.position == state.position
        np.testing.assert_array_equal(traced.keys, state.keys)
        np.testing.assert_array_equal(traced.values, state.values)
        np.testing.assert_array_equal(traced.hidden, state.hidden)
    finally:
        rt.close()


def test_trace_requires_cuda_backend():
    g = Golden("ref-small-fp32")
    rt = Runtime(g.model, RuntimeOptions(backend=Backend.GRAPH, blocks=0))
    try:
        with pytest.raises(StreamError):
            rt.trace_step(g.events[0])
    finally:
        rt.close()
