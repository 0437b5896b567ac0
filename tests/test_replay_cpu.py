"""Scheduled-arrival replay (st_replay_scheduled_with; reference
bench/Main.cpp:282-343) on the host, with a Python step function in place of
the GPU: arrival order, the four timestamps per event, drops when the queue is
full, and the report's accounting."""
import time

import numpy as np

from streaming_transformer_b200.runtime import replay_scheduled_with


def test_paced_arrivals_are_served_in_order_without_drops():
    events = np.arange(64 * 4, dtype=np.float32).reshape(64, 4)
    seen = []

    def step(e):
        seen.append(float(e[0]))
        return float(e.sum())

    report, samples, scores = replay_scheduled_with(step, events, rate=4000.0, queue=128)
    assert report["events"] == 64 and report["completed"] == 64 and report["dropped"] == 0
    assert seen == [float(4 * i) for i in range(64)]
    np.testing.assert_array_equal(scores, events.sum(axis=1))
    intended, enqueue, submit, complete = samples.T
    assert np.all(enqueue >= intended) and np.all(submit >= enqueue) and np.all(complete >= submit)
    np.testing.assert_allclose(np.diff(intended), 1e9 / 4000.0, rtol=1e-6)
    assert report["service"]["p50_us"] >= 0 and "p999_us" in report["arrival"]


def test_bursts_arrive_in_groups_of_sixteen():
    events = np.zeros((48, 2), dtype=np.float32)
    _, samples, _ = replay_scheduled_with(lambda e: 0.0, events, rate=10000.0, bursty=True)
    intended = samples[:, 0]
    for g in range(3):
        assert np.all(intended[16 * g:16 * (g + 1)] == intended[16 * g])
    np.testing.assert_allclose(intended[16] - intended[0], 16 * 1e9 / 10000.0, rtol=1e-6)


def test_a_full_queue_drops_arrivals_and_the_report_counts_them():
    events = np.ones((40, 2), dtype=np.float32)

    def slow(e):
        time.sleep(0.002)   # 2 ms per step against 0.1 ms between arrivals
        return 1.0

    report, samples, scores = replay_scheduled_with(slow, events, rate=10000.0, queue=1, deadline_us=100.0)
    dropped = np.isnan(scores)
    assert report["dropped"] == int(dropped.sum()) > 0
    assert report["completed"] + report["dropped"] == 40
    assert np.all(samples[dropped, 2:] == 0) and np.all(samples[~dropped, 3] > 0)
    assert report["deadline_misses"] > 0
