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
