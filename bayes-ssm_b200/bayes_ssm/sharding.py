"""Chain sharding across ranks.

The recurrence is independent per chain (one (batch, head) sequence), so a
data-parallel job splits the N chains into contiguous shards with no
exchange on the data path.  ``bench.py`` runs weak scaling (every rank owns a
full 16384-chain workload); these helpers cover the strong-scaling split of
one global batch.
"""
from __future__ import annotations


def chain_shard(n: int, world: int, rank: int) -> slice:
    """Contiguous slice of ``range(n)`` owned by ``rank`` (sizes differ by <= 1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"invalid rank {rank} for world size {world}")
    if n < 0:
        raise ValueError("n must be nonnegative")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return slice(lo, lo + base + (1 if rank < extra else 0))


def shard_sizes(n: int, world: int) -> list[int]:
    return [chain_shard(n, world, r).stop - chain_shard(n, world, r).start for r in range(world)]


__all__ = ["chain_shard", "shard_sizes"]
