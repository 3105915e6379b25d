"""Partitioning FA-KLA work across GPUs.

Every (batch b, head h) sequence is independent (the reference processes them
in parallel with no interaction, cpu_kernels.cpp:68), so a multi-GPU run
needs no collective on the data path: each rank takes a contiguous block of
batch rows or of heads. For a head shard the rank also takes the matching
rows of the feature map (W[h0*M:h1*M], bias[h0*M:h1*M]); q and k rows stay
whole because the map mixes all heads of a row.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch


def shard_range(n: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous, balanced [start, stop) of n units for `rank` of `world`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def head_shard(weight: torch.Tensor, bias: Optional[torch.Tensor], heads: int, world: int, rank: int):
    """(h0, h1, W rows, bias rows) of this rank's heads."""
    h0, h1 = shard_range(heads, world, rank)
    m = weight.shape[0] // heads
    w = weight[h0 * m:h1 * m].contiguous()
    b = None if bias is None else bias[h0 * m:h1 * m].contiguous()
    return h0, h1, w, b


def batch_shard(batch: int, world: int, rank: int) -> Tuple[int, int]:
    return shard_range(batch, world, rank)
