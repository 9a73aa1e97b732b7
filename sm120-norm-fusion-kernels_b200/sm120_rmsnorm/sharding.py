"""Row / sequence sharding for one process per GPU.

The fused normalisation path is data-parallel: every row (residual add +
RMSNorm) and every token (Q/K norm + RoPE + KV store) is independent, so N
GPUs split the rows -- or the decode sequences -- and each runs the operator
on its own slice with no collective on the data path. For the KV variant each
rank owns its own paged cache, so its slot_mapping indexes rank-local blocks.

The helpers here only compute the split; they never communicate.
"""
from __future__ import annotations

import torch


def shard_bounds(total: int, world_size: int, rank: int) -> tuple[int, int]:
    """Contiguous ``[start, stop)`` of ``total`` units owned by ``rank``.

    Shards differ in size by at most one unit and the first ``total %
    world_size`` ranks take the larger ones.
    """
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} is not in a world of size {world_size}")
    if total < 0:
        raise ValueError("total must be non-negative")
    base, extra = divmod(total, world_size)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard(tensor: torch.Tensor, world_size: int, rank: int, dim: int = 0) -> torch.Tensor:
    """This rank's slice of ``tensor`` along ``dim`` (a view; contiguous for dim 0
    of a contiguous tensor)."""
    start, stop = shard_bounds(tensor.shape[dim], world_size, rank)
    return tensor.narrow(dim, start, stop - start)


def shard_decode_batch(world_size: int, rank: int, *per_token: torch.Tensor) -> list[torch.Tensor]:
    """Slice per-token tensors (query, key, value, positions, slot_mapping)
    consistently: every tensor gets the same token range of this rank."""
    if not per_token:
        return []
    tokens = per_token[0].shape[0]
    for t in per_token:
        if t.shape[0] != tokens:
            raise ValueError("per-token tensors must share their first dimension")
    start, stop = shard_bounds(tokens, world_size, rank)
    return [t[start:stop] for t in per_token]
