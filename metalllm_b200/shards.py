"""(batch x head) shard planning for running the attention hot path on
several GPUs of one node, one process per GPU.

Every (b, h) pair is independent in flashAttentionForward, computeD and
flashAttentionBackward (attention.metal:74-76, 219-221 decode one head per
threadgroup), so the flat index bh = b*H + h is split into equal contiguous
ranges and no data crosses between GPUs.  A rank only needs the batch rows
its range touches; it calls the *_shard entry points with its range expressed
relative to that local batch slice.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class ShardPlan:
    rank: int
    world: int
    bh_begin: int       # global flat range [bh_begin, bh_end)
    bh_end: int
    b_begin: int        # local batch slice [b_begin, b_end) of the global batch
    b_end: int
    local_bh_begin: int  # the range relative to the local slice
    local_bh_end: int

    @property
    def local_batch(self) -> int:
        return self.b_end - self.b_begin

    @property
    def shards(self) -> int:
        return self.bh_end - self.bh_begin


def plan(B: int, H: int, world: int, rank: int) -> ShardPlan:
    """Contiguous, balanced split of the B*H shards over `world` ranks
    (the first B*H % world ranks get one extra shard)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    total = B * H
    base, extra = divmod(total, world)
    begin = rank * base + min(rank, extra)
    end = begin + base + (1 if rank < extra else 0)
    if end > begin:
        b0 = begin // H
        b1 = (end - 1) // H + 1
    else:
        b0 = b1 = min(begin // H, B)
    return ShardPlan(rank, world, begin, end, b0, b1, begin - b0 * H, end - b0 * H)


def plan_all(B: int, H: int, world: int) -> list[ShardPlan]:
    return [plan(B, H, world, r) for r in range(world)]
