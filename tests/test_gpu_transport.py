"""Transport calibration (st_transport_bench; reference transportBench,
src/cuda/Runtime.cu:706-814) and scheduled-arrival replay through the public
API (st_replay_scheduled; reference bench/Main.cpp:282-343) on the GPU."""
import numpy as np
import pytest

from golden_io import Golden
from oracle.oracle import Oracle
from policy import check_scores
from streaming_transformer_b200 import Backend, Runtime, RuntimeOptions, transport_bench

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode", ["empty", "copy", "ping-pong", "gpu-ping"])
def test_host_transport_modes_round_trip(mode):
    r = transport_bench(mode, 300)
    assert r["mode"] == mode and r["events"] == 300 and r["failed"] == 0, r
    assert 0 < r["p50_us"] <= r["p99_us"] <= r["worst_us"] < 10000, r


def test_grid_barrier_mode_times_device_barriers():
    r = transport_bench("grid-barrier", 2000)
    assert r["mode"] == "grid-barrier" and r["failed"] == 0, r
    assert 100 < r["ns_per_barrier"] < 100000, r


def test_scheduled_replay_serves_every_arrival_and_matches_the_oracle():
    g = Golden("ref-small-fp32")
    events = g.events[:160]
    with Runtime(g.model, RuntimeOptions(backend=Backend.PERSISTENT, blocks=0)) as rt:
        report, samples, scores = rt.replay_scheduled(events, rate=2000.0, queue=4096, deadline_us=5000.0)
    assert report["completed"] == len(events) and report["dropped"] == 0, report
    o = Oracle(g.model)
    want = np.array([o.step(e) for e in events], dtype=np.float32)
    check_scores(scores, want, g.model.config.layers, g.model.mode, "scheduled replay")
    intended, enqueue, submit, complete = samples.T
    assert np.all(submit >= enqueue) and np.all(complete > submit)
    assert report["service"]["p50_us"] < 1000, report


def test_scheduled_replay_drops_arrivals_beyond_its_queue():
    g = Golden("ref-small-fp32")
    events = g.events[:120]
    with Runtime(g.model, RuntimeOptions(backend=Backend.PERSISTENT, blocks=0)) as rt:
        # 1 us between arrivals against tens of microseconds of service
        report, _, scores = rt.replay_scheduled(events, rate=1e6, queue=2)
    assert report["dropped"] > 0 and report["completed"] + report["dropped"] == len(events)
    assert int(np.isnan(scores).sum()) == report["dropped"]
