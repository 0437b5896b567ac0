"""bench.py's multi-rank host logic on CPU: two gloo ranks, max over ranks of
the per-rank timings (the device-side work of each rank is an independent
replica or stream partition, so this reduction is the only cross-rank step), and
the stream partition the C4 record and `--streams` use: which streams each rank
steps, which seeded traces they get, and the whole-job rate."""
import os
import socket
import sys
from pathlib import Path

import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    import torch.distributed as dist
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = [1.0 + rank, 10.0 - rank]  # rank-specific elapsed times
        out[rank] = bench.combine_ranks(mine, dist, None)
    finally:
        dist.destroy_process_group()


def test_max_over_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        assert all(p.exitcode == 0 for p in procs)
        assert out[0] == out[1] == [2.0, 10.0]


def _partition_rank(rank, world, port, out):
    import torch.distributed as dist
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        S = bench.streams_per_rank(256, world)
        ids = bench.rank_streams(rank, S)
        elapsed = [0.5 + 0.25 * rank]  # this rank's timed seconds for K rounds
        maxed = bench.combine_ranks(elapsed, dist, None)
        out[rank] = (S, ids, maxed[0], bench.aggregate_rate(world, S, 100, maxed[0]))
    finally:
        dist.destroy_process_group()


def test_stream_partition_over_two_gloo_ranks():
    """256 streams over 2 ranks: 128 each, disjoint ids covering 0..255 (so stream
    g gets seed base + g at any GPU count), and value = 2 x 128 x K / slowest time."""
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_partition_rank, args=(r, 2, port, out)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        assert all(p.exitcode == 0 for p in procs)
        (s0, ids0, max0, v0), (s1, ids1, max1, v1) = out[0], out[1]
        assert s0 == s1 == 128
        assert sorted(ids0 + ids1) == list(range(256)) and not set(ids0) & set(ids1)
        assert max0 == max1 == 0.75
        assert v0 == v1 == 2 * 128 * 100 / 0.75


def _guarded_rank(rank, world, port, fail_rank, out):
    import torch.distributed as dist
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        def run():
            if rank == fail_rank:
                raise RuntimeError("device wait ran out")
            return (1.0, rank)
        out[rank] = bench.guarded_on_all_ranks(run, dist, None)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fail_rank", [-1, 1])
def test_a_failed_record_is_dropped_on_every_rank(fail_rank):
    """The C5-B record's guard: when one rank's run raises, every rank drops the
    record and reports an error (the failing rank its own message); when none
    fails, every rank keeps its result."""
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_guarded_rank, args=(r, 2, port, fail_rank, out)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        assert all(p.exitcode == 0 for p in procs)
        if fail_rank < 0:
            assert out[0] == ((1.0, 0), None) and out[1] == ((1.0, 1), None)
        else:
            assert out[0] == (None, "the run failed on another rank")
            assert out[1] == (None, "RuntimeError: device wait ran out")


def test_partition_matches_one_gpu_and_rejects_uneven_splits():
    import bench
    assert bench.rank_streams(0, 256) == list(range(256))  # one GPU: the same stream ids
    assert bench.streams_per_rank(1, 8) == 1  # a single-stream config runs one replica per rank
    with pytest.raises(SystemExit):
        bench.streams_per_rank(256, 3)


def test_single_process_is_identity():
    import bench
    assert bench.combine_ranks([3.0, 4.0]) == [3.0, 4.0]
