"""Several independent streams in one runtime (reference RuntimeOptions with
streams > 1, as in the reference's multi-stream benchmark configurations):
every backend, batched steps, per-stream state, a stream reset in the middle,
and the device-trace kernel, each stream checked against its own CPU oracle
under the reference policy. blocks=8 puts every head in one cluster, so one
CTA's weight chunks for a step outnumber the ring's slots and fill its whole
byte buffer."""
import numpy as np
import pytest

from oracle.oracle import Oracle
from policy import check_scores, check_state
from streaming_transformer_b200 import Backend, Runtime, RuntimeOptions, synthetic
from streaming_transformer_b200.model import ModelConfig

S = 3
CONFIG = ModelConfig(2, 128, 2, 256, 16, 32, 1e-5)  # head_dim 64, window 16


def traces(n):
    return np.stack([synthetic.make_events(n, CONFIG.features, seed=100 + s) for s in range(S)], axis=1)


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["fp32", "bf16"])
@pytest.mark.parametrize("backend", [Backend.CUDA, Backend.GRAPH, Backend.FUSED, Backend.PERSISTENT])
@pytest.mark.parametrize("blocks", [0, 8])
def test_batched_streams_match_their_oracles(mode, backend, blocks):
    model = synthetic.make_model(CONFIG, mode, seed=11)
    events = traces(40)
    rt = Runtime(model, RuntimeOptions(backend=backend, blocks=blocks), streams=S)
    oracles = [Oracle(model) for _ in range(S)]
    try:
        got, want = [], []
        for i, e in enumerate(events):
            if i == 25:  # reset stream 1 only
                rt.reset_stream(1)
                oracles[1].reset()
            got.append(rt.step_batch(e))
            want.append([o.step(e[s]) for s, o in enumerate(oracles)])
        got, want = np.array(got), np.array(want, dtype=np.float32)
        for s in range(S):
            check_scores(got[:, s], want[:, s], CONFIG.layers, mode, f"stream {s}")
            snap = rt.snapshot(s)
            assert snap.position == oracles[s].position
            check_state(snap.keys, oracles[s].keys(), mode, f"keys stream {s}")
            check_state(snap.values, oracles[s].values(), mode, f"values stream {s}")
            check_state(snap.hidden[:, None, :], oracles[s].hidden()[:, None, :], mode, f"hidden stream {s}")
    finally:
        rt.close()


@pytest.mark.gpu
@pytest.mark.parametrize("backend", [Backend.FUSED, Backend.PERSISTENT])
@pytest.mark.parametrize("blocks", [0, 8])
def test_device_trace_of_several_streams(backend, blocks):
    model = synthetic.make_model(CONFIG, "fp32", seed=12)
    events = traces(30)
    rt = Runtime(model, RuntimeOptions(backend=backend, blocks=blocks), streams=S)
    try:
        _, scores = rt.device_trace(events, return_scores=True)
        assert rt.snapshot(0).position == len(events)
    finally:
        rt.close()
    for s in range(S):
        o = Oracle(model)
        want = np.array([o.step(e) for e in events[:, s]], dtype=np.float32)
        check_scores(scores[:, s], want, CONFIG.layers, "fp32", f"trace stream {s}")
