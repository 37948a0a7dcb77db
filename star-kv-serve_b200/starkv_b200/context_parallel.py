"""Context-parallel decode: each rank decodes, for all heads, its share of every
sequence (its contiguous run of 256-token tiles) with
``paged_starkv_decode(..., context=(rank, world))`` or
``paged_quant_decode(..., context=...)``, and the ranks' partial results are
combined exactly:

    M = max_r m_r,   out = sum_r exp(m_r - M) out_r / sum_r exp(m_r - M) l_r

(out_r is the rank's unnormalised, already lifted output, m_r / l_r its per-head
logit max and softmax denominator). Every rank reads 1/world of the K and V codes,
including the V latent that head sharding has to replicate.

A rank's partial lives in one packed f32 buffer ``[out n*H*128 | m n*H | l n*H]``;
the exchange is a single NCCL all-gather of those buffers (about 1 MB each for 64
sequences x 32 heads) and the combination one native kernel
(``starkv_cp_combine``).
"""
from __future__ import annotations

import torch

from . import _lib
from .collectives import all_gather_into_

_PACK = 130   # floats per (sequence, head): 128 output values, max, denominator


def partial_views(n: int, H: int, device, buf: torch.Tensor | None = None):
    """(out [n, H, 128], m [n, H], l [n, H]) views of one packed f32 buffer."""
    size = n * H * _PACK
    if buf is None:
        buf = torch.empty(size, dtype=torch.float32, device=device)
    assert buf.dtype == torch.float32 and buf.is_contiguous() and buf.numel() >= size
    nh = n * H
    return (buf[:nh * 128].view(n, H, 128), buf[nh * 128:nh * 129].view(n, H), buf[nh * 129:nh * 130].view(n, H))


def _packed(out: torch.Tensor, m: torch.Tensor, l: torch.Tensor) -> torch.Tensor:
    n, H = m.shape
    nh = n * H
    if (out.is_contiguous() and m.is_contiguous() and l.is_contiguous()
            and m.data_ptr() == out.data_ptr() + 4 * nh * 128 and l.data_ptr() == m.data_ptr() + 4 * nh):
        return torch.as_strided(out, (nh * _PACK,), (1,))
    return torch.cat([out.reshape(-1), m.reshape(-1), l.reshape(-1)])


def _combine_parts(parts: torch.Tensor, world: int, n: int, H: int, dtype, result=None) -> torch.Tensor:
    if result is None:
        result = torch.empty((n, H, 128), dtype=dtype, device=parts.device)
    st = _lib.lib().starkv_cp_combine(parts.data_ptr(), world, n, H, result.data_ptr(), _lib.i64s(result.stride()),
                                      _lib.dtype_code(result), _lib.stream_ptr(parts.device))
    _lib.check(st, "cp_combine")
    return result


_gather_bufs: dict = {}


def gather_partials(out: torch.Tensor, m: torch.Tensor, l: torch.Tensor, group=None) -> torch.Tensor:
    """All ranks of `group`: one all-gather of the packed partials; returns the
    rank-major buffer [world * n*H*130] (reused between calls of the same size)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    local = _packed(out, m, l)
    key = (local.device, local.dtype, world, local.numel())
    gathered = _gather_bufs.get(key)
    if gathered is None:
        gathered = _gather_bufs[key] = torch.empty(world * local.numel(), dtype=local.dtype, device=local.device)
    all_gather_into_(gathered, local, group=group)
    return gathered


def combine(out: torch.Tensor, m: torch.Tensor, l: torch.Tensor, group=None, dtype=torch.bfloat16,
            result: torch.Tensor | None = None) -> torch.Tensor:
    """All ranks of `group` call this with their partial (out, m, l) on the GPU;
    every rank gets the combined [n, H, 128] output in `dtype`."""
    import torch.distributed as dist
    n, H = m.shape
    gathered = gather_partials(out, m, l, group)
    return _combine_parts(gathered, dist.get_world_size(group), n, H, dtype, result)


def combine_local(parts: list[tuple[torch.Tensor, torch.Tensor, torch.Tensor]], dtype=torch.bfloat16) -> torch.Tensor:
    """The same combination for partial results held by one process (tests, one GPU)."""
    n, H = parts[0][1].shape
    stacked = torch.cat([_packed(*p) for p in parts])
    return _combine_parts(stacked, len(parts), n, H, dtype)


# ---------------------------------------------------------------------------
# Page round-robin placement (growing sequences).
#
# The split above divides a sequence whose length is known. A served sequence grows
# by one token per step, and its tokens must not move between ranks as it grows, so
# the whole model stores page p of every sequence (tokens 16p .. 16p+15) on rank
# p % world. On its rank a page is local page p // world, and the rank's pages of a
# sequence form one contiguous local sequence that the decode kernels read like any
# other. Only the rotary rows differ: the score kernel takes row i of the table for
# local token i, so each rank passes a table whose row i holds the rotary row of that
# token's global position. The keys are then rotated at their true positions, and
# the partial results combine exactly as above.
# ---------------------------------------------------------------------------

def page_owner(pos, world: int, block_size: int = 16):
    """Rank that stores global position `pos` (int or tensor)."""
    return (pos // block_size) % world


def local_index(pos, world: int, block_size: int = 16):
    """Index of global position `pos` in its owner's local sequence."""
    return (pos // block_size // world) * block_size + pos % block_size


def global_position(i, rank: int, world: int, block_size: int = 16):
    """Global position of local token `i` of `rank` (the inverse of local_index)."""
    return ((i // block_size) * world + rank) * block_size + i % block_size


def local_len(L, rank: int, world: int, block_size: int = 16):
    """Tokens of a sequence of length `L` (int or tensor) that `rank` stores."""
    full, rem = L // block_size, L % block_size
    n_full = (full - rank + world - 1) // world            # owned whole pages among 0 .. full-1
    tail = rem * ((full % world) == rank)                 # the partial last page, if owned
    return n_full * block_size + tail


def local_rotary_table(cos_sin_cache: torch.Tensor, rank: int, world: int, block_size: int = 16) -> torch.Tensor:
    """[ceil(P / world) rounded to pages, 128] table whose row i is row
    global_position(i) of `cos_sin_cache` ([P, 128]); rows past P repeat its last
    row and are never read for a sequence shorter than P."""
    P = cos_sin_cache.shape[0]
    rows = -(-P // (block_size * world)) * block_size
    i = torch.arange(rows, device=cos_sin_cache.device)
    return cos_sin_cache[global_position(i, rank, world, block_size).clamp(max=P - 1)].contiguous()


class PageSplitTables:
    """One rank's block tables under the page split, for sequences that grow.

    A serving engine keeps one of these per rank. `extend` appends tokens to
    sequences and returns the local cache slots to write them at. A slot is -1 where
    another rank owns the token's page; the cache-write kernels send such a slot to
    the reserved null block. A rank takes a local block only when one of its pages
    starts. `decode_metadata` returns the local block table, sequence lengths and
    their bound for a decode call over the rank's pages. `release` frees a finished
    sequence's blocks for reuse. Block 0 is never handed out: it stays the null
    block."""

    def __init__(self, rank: int, world: int, num_blocks: int, block_size: int = 16):
        if not 0 <= rank < world:
            raise ValueError(f"rank {rank} outside a world of {world}")
        self.rank, self.world, self.block_size = rank, world, block_size
        self.free = list(range(num_blocks - 1, 0, -1))     # pop() hands out low ids first
        self.blocks: dict = {}                              # sequence id -> local block ids
        self.lens: dict = {}                                # sequence id -> global length

    def blocks_needed(self, seq_id, count: int = 1) -> int:
        """Local blocks this rank would take to append `count` tokens to `seq_id`;
        changes nothing."""
        L = self.lens.get(seq_id, 0)
        held = len(self.blocks.get(seq_id, []))
        return -(-int(local_len(L + count, self.rank, self.world, self.block_size)) // self.block_size) - held

    def can_extend(self, seq_id, count: int = 1) -> bool:
        """Whether this rank has the blocks for `extend(seq_id, count)`; changes nothing.
        The ranks of a group must agree before any of them extends (each rank's need
        differs), see extend_agreed / extend_on_all_ranks."""
        return self.blocks_needed(seq_id, count) <= len(self.free)

    def extend(self, seq_id, count: int = 1) -> list[int]:
        """Append `count` tokens to `seq_id` (created on first use); returns the local
        slot of each new token, -1 where another rank stores it. Refuses with
        RuntimeError, changing nothing, when this rank is short of blocks; that keeps
        one rank consistent, not the group (another rank may already have extended),
        so a serving engine extends through extend_agreed."""
        L = self.lens.get(seq_id, 0)
        bs = self.block_size
        need = self.blocks_needed(seq_id, count)
        if need > len(self.free):   # refuse before changing anything
            raise RuntimeError(f"rank {self.rank}: sequence {seq_id!r} needs {need} more cache blocks, "
                               f"{len(self.free)} free")
        blocks = self.blocks.setdefault(seq_id, [])
        blocks.extend(self.free.pop() for _ in range(need))
        out = []
        for pos in range(L, L + count):
            if page_owner(pos, self.world, bs) != self.rank:
                out.append(-1)
            else:
                li = local_index(pos, self.world, bs)
                out.append(blocks[li // bs] * bs + li % bs)
        self.lens[seq_id] = L + count
        return out

    def local_len(self, seq_id) -> int:
        return int(local_len(self.lens.get(seq_id, 0), self.rank, self.world, self.block_size))

    def decode_metadata(self, seq_ids, device=None, max_blocks: int | None = None):
        """(block_table int32 [n, max_blocks], seq_lens int32 [n], max_seq_len) of the
        rank's local sequences, for paged_starkv_decode / paged_quant_decode."""
        lens = [self.local_len(s) for s in seq_ids]
        width = max_blocks or max([len(self.blocks.get(s, [])) for s in seq_ids] + [1])
        bt = torch.zeros(len(seq_ids), width, dtype=torch.int32)
        for i, s in enumerate(seq_ids):
            b = self.blocks.get(s, [])
            if len(b) > width:
                raise ValueError(f"sequence {s!r} holds {len(b)} blocks here, more than max_blocks={width}")
            bt[i, :len(b)] = torch.tensor(b, dtype=torch.int32)
        return (bt.to(device) if device is not None else bt,
                torch.tensor(lens, dtype=torch.int32, device=device), max(lens + [1]))

    def release(self, seq_id) -> None:
        """Forget a finished sequence and free its blocks."""
        self.free.extend(reversed(self.blocks.pop(seq_id, [])))
        self.lens.pop(seq_id, None)


def extend_on_all_ranks(tables: list[PageSplitTables], seq_id, count: int = 1) -> list[list[int]]:
    """Extend `seq_id` on every rank's tables held in one process (ranks emulated
    on one GPU, tests): every rank is checked first, so either all extend or none
    does (RuntimeError, nothing changed)."""
    short = [t.rank for t in tables if not t.can_extend(seq_id, count)]
    if short:
        raise RuntimeError(f"sequence {seq_id!r}: rank(s) {short} short of cache blocks; no rank extended")
    return [t.extend(seq_id, count) for t in tables]


def extend_agreed(table: PageSplitTables, seq_id, count: int = 1, group=None) -> list[int]:
    """Extend `seq_id` on this rank only if every rank of the group can: the ranks
    agree with one MIN all-reduce of can_extend (a tensor on the backend's device)
    before any of them changes its tables. If any rank is short, every rank raises
    RuntimeError with its tables unchanged, so the group stays consistent. Every rank
    must call it for the same (seq_id, count), in the same order."""
    import torch.distributed as dist
    ok = torch.tensor([1 if table.can_extend(seq_id, count) else 0], dtype=torch.int32)
    if dist.get_backend(group) == "nccl":
        ok = ok.cuda()
    dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
    if int(ok.item()) == 0:
        raise RuntimeError(f"sequence {seq_id!r}: a rank of the group is short of cache blocks; no rank extended")
    return table.extend(seq_id, count)
