"""bench.py's multi-rank host logic on CPU: two gloo ranks, max over ranks of
the per-rank timings (the device-side work of each rank is an independent
replica, so this reduction is the only cross-rank step)."""
import os
import socket
import sys
from pathlib import Path

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


def test_single_process_is_identity():
    import bench
    assert bench.combine_ranks([3.0, 4.0]) == [3.0, 4.0]
