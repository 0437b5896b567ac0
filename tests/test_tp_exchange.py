"""Host side of tensor parallelism on CPU: the handle all-gather two gloo ranks
use to connect their runtimes (streaming_transformer_b200.tp) returns every
rank's blob in rank order, including binary blobs of the handle's size."""
import multiprocessing as mp
import os
import socket

import pytest


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from streaming_transformer_b200.tp import torch_tensor_parallel
    dist.init_process_group("gloo", rank=rank, world_size=world)
    tp = torch_tensor_parallel()
    blob = bytes([rank]) * 100 + bytes(range(156))  # 256 bytes, every byte value present
    got = tp.exchange(blob)
    out.put((rank, tp.rank, tp.size, [b[:1] for b in got], all(len(b) == 256 for b in got)))
    dist.destroy_process_group()


def test_handles_gather_in_rank_order():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, tp_rank, tp_size, firsts, sizes in results:
        assert tp_rank == rank and tp_size == 2 and sizes
        assert firsts == [b"\x00", b"\x01"]
