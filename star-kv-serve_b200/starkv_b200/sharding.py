"""Head-sharded tensor parallelism for the decode path.

Each rank keeps the K codes and K up-projection rows of its own KV heads and the
whole V latent (one V code is shared by every head, checkpoint.py:140-153, so
head sharding cannot split it). Heads are dealt so every rank has the same
number of heads (the query / o_proj shards stay equal) and K bytes per token are
balanced: longest-processing-time first on the per-head K width, each head to
the least-loaded rank that still has room.
"""
from __future__ import annotations


def align16(r: int) -> int:
    return -(-int(r) // 16) * 16


def lpt_shard(ranks: list[int], world: int) -> list[list[int]]:
    """Partition head indices into `world` equal-size groups balancing sum(align16(rank))."""
    H = len(ranks)
    if H % world:
        raise ValueError(f"{H} heads do not split over {world} ranks")
    cap = H // world
    order = sorted(range(H), key=lambda h: (-align16(ranks[h]), h))
    load = [0] * world
    groups: list[list[int]] = [[] for _ in range(world)]
    for h in order:
        r = min((g for g in range(world) if len(groups[g]) < cap), key=lambda g: (load[g], g))
        groups[r].append(h)
        load[r] += align16(ranks[h])
    return [sorted(g) for g in groups]


def shard_loads(ranks: list[int], groups: list[list[int]]) -> list[int]:
    return [sum(align16(ranks[h]) for h in g) for g in groups]
