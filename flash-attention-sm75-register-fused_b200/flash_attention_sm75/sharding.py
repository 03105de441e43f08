"""Partition of the independent (batch, head) units of an attention forward
across ranks — the only multi-GPU structure this path has (no exchange step).

GQA: query heads that share a KV head form one unit group, so a rank never
needs a KV head it does not own and no K/V row is duplicated across ranks.
"""
from dataclasses import dataclass
from typing import List, Tuple


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    groups: List[Tuple[int, int]]  # (batch, kv_head) pairs owned by this rank
    group_size: int                # query heads per KV head

    @property
    def query_units(self) -> List[Tuple[int, int]]:
        """(batch, query_head) pairs of this rank, in repeat_interleave order."""
        g = self.group_size
        return [(b, hk * g + i) for (b, hk) in self.groups for i in range(g)]


def shard_units(B: int, Hq: int, Hkv: int, world: int, rank: int) -> Shard:
    """Contiguous split of the B*Hkv KV-head groups over ``world`` ranks;
    the first ``(B*Hkv) % world`` ranks get one extra group."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    if Hkv <= 0 or Hq % Hkv != 0:
        raise ValueError(f"Q heads ({Hq}) not divisible by K/V heads ({Hkv})")
    total = B * Hkv
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    count = base + (1 if rank < extra else 0)
    groups = [divmod(u, Hkv) for u in range(start, start + count)]
    return Shard(rank, world, groups, Hq // Hkv)


def batch_range(B_per_rank: int, rank: int) -> Tuple[int, int]:
    """Weak scaling: rank r owns global batch entries [r*B, (r+1)*B)."""
    return rank * B_per_rank, (rank + 1) * B_per_rank
