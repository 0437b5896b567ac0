"""Persistent-worker lifecycle (reference tests/Lifecycle.cu:17-137) and the
mailbox protocol's bounded waits, exercised without any GPU fault: the idle
budget and max-events exits are ordinary, bounded device-side returns."""
import time

import numpy as np
import pytest

from golden_io import Golden
from oracle.oracle import Oracle
from streaming_transformer_b200 import Backend, Runtime, RuntimeOptions, StreamError

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode", ["fp32", "mixed"])
@pytest.mark.parametrize("blocks", [1, 4])
def test_reset_repeated_scores_and_restart(mode, blocks):
    g = Golden(f"ref-small-{mode}")
    W = g.model.config.window
    options = RuntimeOptions(backend=Backend.PERSISTENT, blocks=blocks)
    for restart in range(2):
        rt = Runtime(g.model, options)
        o = Oracle(g.model)
        event = np.zeros(g.model.config.features, dtype=np.float32)
        for i in range(3 * W + 9):
            if i in (1, W, 2 * W + 3):
                rt.reset()
                rt.reset()
                o.reset()
                assert rt.snapshot().position == 0
            # Repeated zero scores still advance and complete distinct sequence IDs.
            assert rt.step(event) == pytest.approx(o.step(event), abs=1e-6)
            assert rt.snapshot().position == o.position
        rt.stop()
        rt.stop()
        with pytest.raises(StreamError):
            rt.step(event)
        with pytest.raises(StreamError):
            rt.reset()
        rt.close()


@pytest.mark.parametrize("blocks", [1, 4])
def test_finite_event_exit(blocks):
    g = Golden("ref-small-fp32")
    event = np.zeros(g.model.config.features, dtype=np.float32)
    rt = Runtime(g.model, RuntimeOptions(backend=Backend.PERSISTENT, blocks=blocks, max_events=2))
    assert rt.step(event) == 0.0
    rt.reset()
    assert rt.step(event) == 0.0
    with pytest.raises(StreamError) as info:
        rt.step(event)
    assert info.value.status in ("WORKER_EXITED", "STOPPED")
    rt.stop()
    rt.close()


def test_idle_exit():
    g = Golden("ref-small-fp32")
    event = np.zeros(g.model.config.features, dtype=np.float32)
    rt = Runtime(g.model, RuntimeOptions(backend=Backend.PERSISTENT, idle_seconds=0.001))
    time.sleep(0.1)
    with pytest.raises(StreamError) as info:
        rt.step(event)
    assert info.value.status == "WORKER_EXITED"
    rt.stop()
    rt.close()


@pytest.mark.parametrize("blocks", [1, 4])
def test_sequence_exhaustion_still_allows_stop(blocks):
    g = Golden("ref-small-fp32")
    event = np.zeros(g.model.config.features, dtype=np.float32)
    rt = Runtime(g.model, RuntimeOptions(backend=Backend.PERSISTENT, blocks=blocks, initial_sequence=2 ** 64 - 3))
    assert rt.step(event) == 0.0
    with pytest.raises(StreamError) as info:
        rt.step(event)
    assert info.value.status == "EXHAUSTED"
    with pytest.raises(StreamError):
        rt.reset()
    rt.stop()
    rt.stop()
    rt.close()


def test_cooperative_grid_above_occupancy_is_rejected():
    g = Golden("ref-small-fp32")
    with pytest.raises(StreamError) as info:
        Runtime(g.model, RuntimeOptions(backend=Backend.PERSISTENT, blocks=100000))
    assert "occupancy" in str(info.value)


def test_backoff_polling_gives_identical_results():
    g = Golden("ref-small-mixed")
    out = []
    for backoff in (False, True):
        rt = Runtime(g.model, RuntimeOptions(backend=Backend.PERSISTENT, blocks=0, backoff=backoff))
        out.append([rt.step(e) for e in g.events[:30]])
        rt.close()
    assert out[0] == out[1]


def test_info_and_probe_describe_the_device():
    from streaming_transformer_b200 import probe
    p = probe()
    assert p["compute_major"] == 10 and p["sm_count"] > 0
    g = Golden("ref-small-fp32")
    rt = Runtime(g.model, RuntimeOptions(backend=Backend.PERSISTENT, blocks=0))
    info = rt.info()
    # one CTA per SM at most, whole clusters only (clusters of 8 pack per GPC)
    assert 0 < info["blocks"] <= p["sm_count"] and info["threads"] == 512
    assert info["blocks"] % info["cluster"] == 0 and info["clusters"] * info["cluster"] == info["blocks"]
    assert info["transport"] == "mapped-system-load-store"
    assert info["registers_per_thread"] > 0
    rt.close()


def test_snapshot_during_persistent_run_and_reset_stream_errors():
    g = Golden("ref-small-fp32")
    rt = Runtime(g.model, RuntimeOptions(backend=Backend.PERSISTENT, blocks=0))
    for e in g.events[:5]:
        rt.step(e)
    assert rt.snapshot().position == 5
    with pytest.raises(StreamError):
        rt.snapshot(stream=1)
    with pytest.raises(StreamError):
        rt.reset_stream(3)
    rt.close()


@pytest.mark.parametrize("backend", [Backend.FUSED, Backend.PERSISTENT], ids=lambda b: b.name.lower())
def test_bounded_device_wait_runs_out(backend, monkeypatch):
    """A device-side wait whose flag nothing sets: CTA 0 of the single-stream
    kernel withholds its layer-0 out-projection records (ST_TEST_DROP_RECORD),
    so every CTA's exchange-1 wait runs out its bound (shortened to 50 ms by
    ST_DEVICE_TIMEOUT_MS). The kernel must return with the error word set, the
    host must report DEVICE_TIMEOUT, the runtime must then refuse work and be
    destroyed cleanly, and the same context must serve a fresh runtime whose
    results match the oracle (reference tests/Lifecycle.cu:50-73; host-side
    detection src/cuda/Runtime.cu:417-426). Nothing faults or hangs the GPU."""
    from streaming_transformer_b200 import synthetic
    config, mode = synthetic.CONFIGS["c1-small-fp32"]
    model = synthetic.make_model(config, mode, seed=3)
    events = synthetic.make_events(3, config.features, seed=4)
    monkeypatch.setenv("ST_DEVICE_TIMEOUT_MS", "50")
    monkeypatch.setenv("ST_TEST_DROP_RECORD", "0")
    rt = None
    t0 = time.perf_counter()
    with pytest.raises(StreamError) as info:
        # FUSED meets the withheld record already in st_start's warm-up step
        rt = Runtime(model, RuntimeOptions(backend=backend, blocks=0))
        assert rt.info()["resource_kernel"] == "k4_flow"
        rt.step(events[0])
    assert info.value.status == "DEVICE_TIMEOUT", str(info.value)
    assert time.perf_counter() - t0 < 20.0
    if rt is not None:
        with pytest.raises(StreamError):
            rt.step(events[1])
        rt.close()
    monkeypatch.delenv("ST_DEVICE_TIMEOUT_MS")
    monkeypatch.delenv("ST_TEST_DROP_RECORD")
    o = Oracle(model)
    with Runtime(model, RuntimeOptions(backend=backend, blocks=0)) as fresh:
        got = np.array([fresh.step(e) for e in events])
    want = np.array([o.step(e) for e in events])
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6)
