"""Several independent streams in one runtime (reference RuntimeOptions with
streams > 1, as in the reference's multi-stream benchmark configurations):
every backend, batched steps, per-stream state, a stream reset in the middle,
and the device-trace kernel, each stream checked against its own CPU oracle
under the reference policy. blocks=8 puts every head in one cluster, so one
CTA's weight chunks for a step outnumber the ring's slots and fill its whole
byte buffer. ST_BATCHED=1 forces the batched round (every weight read once per
round for all streams), =0 the per-stream loop inside one launch."""
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
@pytest.mark.parametrize("blocks,batched", [(0, "0"), (8, "0"), (0, "1")])
def test_batched_streams_match_their_oracles(mode, backend, blocks, batched, monkeypatch):
    monkeypatch.setenv("ST_BATCHED", batched)
    model = synthetic.make_model(CONFIG, mode, seed=11)
    events = traces(40)
    rt = Runtime(model, RuntimeOptions(backend=backend, blocks=blocks), streams=S)
    assert rt.info()["batched"] == (batched == "1")
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
@pytest.mark.parametrize("blocks,batched", [(0, "0"), (8, "0"), (0, "1")])
def test_device_trace_of_several_streams(backend, blocks, batched, monkeypatch):
    monkeypatch.setenv("ST_BATCHED", batched)
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


WIDE = ModelConfig(2, 256, 4, 512, 24, 32, 1e-6)  # head_dim 64, window 24


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_batched_round_with_a_partial_stream_group(mode, monkeypatch):
    """40 streams: one full 32-stream GEMM group and a partial one; more events
    than the window, so the ring wraps; device trace and stepped rounds."""
    monkeypatch.setenv("ST_BATCHED", "1")
    n_streams, n_events = 40, 30
    model = synthetic.make_model(WIDE, mode, seed=21)
    events = np.stack([synthetic.make_events(n_events, WIDE.features, seed=300 + s) for s in range(n_streams)], axis=1)
    rt = Runtime(model, RuntimeOptions(backend=Backend.FUSED, blocks=0), streams=n_streams)
    try:
        assert rt.info()["batched"]
        _, traced = rt.device_trace(events, return_scores=True)
        rt.reset()
        stepped = np.array([rt.step_batch(e) for e in events])
        snaps = [rt.snapshot(s) for s in (0, 33, n_streams - 1)]
    finally:
        rt.close()
    np.testing.assert_array_equal(traced, stepped)  # same kernel, same order: bit-identical
    for s, snap in zip((0, 33, n_streams - 1), snaps):
        o = Oracle(model)
        want = np.array([o.step(e) for e in events[:, s]], dtype=np.float32)
        check_scores(stepped[:, s], want, WIDE.layers, mode, f"stream {s}")
        assert snap.position == n_events
        check_state(snap.keys, o.keys(), mode, f"keys stream {s}")
        check_state(snap.values, o.values(), mode, f"values stream {s}")
