"""Data-parallel sharding of independent robot streams over the GPUs of one
node (one process per GPU).

Every stream owns its KV ring, suffix and x_t, so a rank serves a contiguous
block of streams batched along B with no collective on the hot path.  The
only exchange is the gather of the finished action chunks to rank 0 after a
chunk (the multi-stream configuration's final NCCL gather).
"""
from __future__ import annotations

import torch


def shard_range(n_streams: int, rank: int, world: int) -> tuple[int, int]:
    """(first stream, count) served by `rank`; the first n_streams % world
    ranks take one stream more."""
    if n_streams < 1 or world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad sharding: {n_streams} streams, rank {rank} of {world}")
    base, rem = divmod(n_streams, world)
    return rank * base + min(rank, rem), base + (1 if rank < rem else 0)


def gather_chunks(local: torch.Tensor, n_streams: int, dist, group=None) -> torch.Tensor:
    """All ranks' action chunks [n_local, ...] -> [n_streams, ...] in stream
    order (returned on every rank).  Shards of unequal size are padded to the
    largest one for the collective, which every rank enters once."""
    world = dist.get_world_size(group)
    counts = [shard_range(n_streams, r, world)[1] for r in range(world)]
    rank = dist.get_rank(group)
    if local.shape[0] != counts[rank]:
        raise ValueError(f"rank {rank} holds {local.shape[0]} streams, expected {counts[rank]}")
    pad = max(counts)
    buf = local.new_zeros((pad,) + tuple(local.shape[1:]))
    buf[: local.shape[0]].copy_(local)
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    return torch.cat([p[:c] for p, c in zip(parts, counts)], dim=0)
