"""Sequence sharding of a multi-sequence batch over the GPUs of one node.

The reference decodes one sequence at a time and has no batch path; its sequences are independent
(each has its own KV cache rows, tinyllama.cpp:122-138), so a batch is split by sequence: rank r of
a world of size G takes a contiguous range of sequences, runs them with its own model replica
(Model.generate_batch, all of its sequences in one fused decode step), and the ranks' rows are
concatenated at the end. The data path has no collective; the only exchange is the final gather
of the generated ids to rank 0 (host objects through torch.distributed, NCCL or gloo).
"""
from __future__ import annotations

import datetime


def shard_range(n_seq: int, world: int, rank: int) -> tuple[int, int]:
    """(start, count) of rank's sequences: contiguous ranges in rank order whose sizes differ by at
    most one (the first n_seq % world ranks take one extra)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if n_seq < 0:
        raise ValueError("negative batch")
    base, extra = divmod(n_seq, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def generate_sharded(model, prompts, n_gen: int, group=None):
    """Greedy decode of a [batch, n_prompt] int32 prompt array sharded by sequence over the
    process group; returns the [batch, n_gen] ids on rank 0 and None on the other ranks.

    `model` is this rank's replica (anything with generate_batch(prompts, n_gen) -> [b, n_gen]).
    A rank whose shard is empty takes part in the gather with an empty block. Errors of a rank
    (an exception in its shard) are raised on that rank; the others see the gather fail within
    the process group's timeout instead of waiting for good."""
    import numpy as np
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    p = np.ascontiguousarray(prompts, np.int32)
    if p.ndim != 2:
        raise ValueError("prompts must be [batch, n_prompt]")
    start, count = shard_range(p.shape[0], world, rank)
    local = model.generate_batch(p[start:start + count], n_gen) if count else np.zeros((0, n_gen), np.int32)
    local = np.ascontiguousarray(local, np.int32)
    parts = [None] * world if rank == 0 else None
    dist.gather_object((start, local), parts, dst=0, group=group)
    if rank != 0:
        return None
    out = np.zeros((p.shape[0], n_gen), np.int32)
    for s, block in parts:
        out[s:s + block.shape[0]] = block
    return out


def init_group(backend: str, timeout_s: float = 60.0):
    """torch.distributed.init_process_group from the torchrun environment (MASTER_ADDR should be
    127.0.0.1 on this node) with a short timeout, so that ranks waiting for a failed rank end
    with an error."""
    import torch.distributed as dist
    if not dist.is_initialized():
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s))
    return dist.get_rank(), dist.get_world_size()
