"""Batch sharding across GPUs.

The projection is independent per matrix, so a batch of N matrices splits
into contiguous slices, one per rank, with no exchange on the data path.
Slices differ in size by at most one matrix; rank r gets
[N*r//world, N*(r+1)//world).
"""
from __future__ import annotations


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    if world < 1 or not (0 <= rank < world) or n < 0:
        raise ValueError(f"bad shard request n={n} rank={rank} world={world}")
    return n * rank // world, n * (rank + 1) // world


def shard_sizes(n: int, world: int) -> list[int]:
    return [b - a for a, b in (shard_range(n, r, world) for r in range(world))]
