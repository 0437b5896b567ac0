"""Host side of tensor parallelism (one stream over several GPUs of a node).

Each GPU of the stream is driven by its own process (torchrun: one rank per
GPU). The runtimes connect by exchanging small handles (the layout they were
built with and an IPC handle of their record buffers); after that the GPUs'
kernels talk to each other directly over NVLink and the host only keeps the
ranks' calls in step: every call that runs the model is made by all ranks,
with the same inputs, in the same order.
"""
from __future__ import annotations

from .runtime import TensorParallel


def torch_exchange(group=None):
    """An all-gather of byte strings among the stream's processes over
    torch.distributed (any backend; gloo needs no GPU)."""
    import torch.distributed as dist

    def exchange(blob: bytes) -> list[bytes]:
        out = [None] * dist.get_world_size(group)
        dist.all_gather_object(out, bytes(blob), group=group)
        return [bytes(b) for b in out]

    return exchange


def torch_tensor_parallel(group=None) -> TensorParallel:
    """This process's place in a stream spanning every rank of ``group``."""
    import torch.distributed as dist
    return TensorParallel(rank=dist.get_rank(group), size=dist.get_world_size(group), exchange=torch_exchange(group))
