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


def k_offsets(ranks: list[int]) -> list[int]:
    """Start lane of each head's K codes in a row: heads packed at 16-lane widths."""
    offs, o = [], 0
    for r in ranks:
        offs.append(o)
        o += align16(r)
    return offs


def shard_lanes(ranks: list[int], heads: list[int]) -> tuple[list[int], list[int], int, list[int]]:
    """K layout of a rank that keeps KV heads `heads` (in that order).

    Returns (local ranks, local offsets, local K width, lanes) where ``lanes[i]`` is
    the lane of the full row that local lane ``i`` holds: a rank's cache rows are
    ``[K codes at lanes | V codes]`` and its ``k_up`` rows are ``k_up[lanes]``.
    """
    full = k_offsets(ranks)
    local_ranks, local_offsets, lanes = [], [], []
    for h in heads:
        w = align16(ranks[h])
        local_ranks.append(int(ranks[h]))
        local_offsets.append(len(lanes))
        lanes.extend(range(full[h], full[h] + w))
    return local_ranks, local_offsets, len(lanes), lanes


def query_heads(heads: list[int], group: int) -> list[int]:
    """Query heads served by KV heads `heads` (GQA group size `group`), in order: the
    rank's query / v_up_by_q / output rows."""
    return [h * group + j for h in heads for j in range(group)]
