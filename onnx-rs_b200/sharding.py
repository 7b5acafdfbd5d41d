"""Batch sharding across GPUs of one node: each rank runs a contiguous slice of
the batch on its own full weight replica; no data-path collective.  The
"concat" is the ranks' outputs placed side by side in batch order."""
from __future__ import annotations

from typing import List, Tuple


def shard_range(global_batch: int, world: int, rank: int) -> Tuple[int, int]:
    """[start, stop) of `rank`'s images; the batch must split evenly (256/world)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if global_batch % world:
        raise ValueError(f"global batch {global_batch} does not split evenly over {world} ranks")
    per = global_batch // world
    return rank * per, (rank + 1) * per


def all_ranges(global_batch: int, world: int) -> List[Tuple[int, int]]:
    return [shard_range(global_batch, world, r) for r in range(world)]
