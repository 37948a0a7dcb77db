"""Paged decode over the 3.2-bit STAR-KV cache, on the sm_100a library.

Drop-in for ``starkv_serve/kernels/paged_quant.py``: the format constants and
host helpers keep the reference's names and meaning (OUTLIER_RATIO, HADAMARD_SEED,
EPS, HEAD_DIM, n_outlier, block_hadamard, QuantRow, k_tables), and the three
operators keep their signatures:

* ``pack_kv``            paged_quant.py:205-216 -> ``starkv_pack_kv_q32``
* ``fold_q``             paged_quant.py:241-255 -> ``starkv_fold_q``
* ``paged_quant_decode`` paged_quant.py:357-411 -> ``starkv_paged_decode_q32``

The format is kv_quant.py's (kv_quant.py:13-24): per token, each KV head's leading
int(0.2 * rank) channels at 4 bits and the rest at 3 bits, each block with one
symmetric bf16 scale; the V latent likewise with its outlier bytes first. The
quantizer is kv_quant._q (kv_quant.py:111-121) bit for bit: IEEE division and
round-half-even. The block Hadamard is folded into the weights by the loader, so
decode never applies an inverse rotation (checkpoint.py:96-103, 118-123).
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass

import torch

from .. import _lib, context_parallel, workspace

OUTLIER_RATIO = 0.2
HADAMARD_SEED = 1234
EPS = 1e-5
HEAD_DIM = 128


def n_outlier(rank: int) -> int:
    """Outlier channels of a block of ``rank`` channels (paged_quant.py:46-47)."""
    return int(OUTLIER_RATIO * rank)


def block_hadamard(rank: int, n_out: int, generator: torch.Generator) -> torch.Tensor:
    """rank x rank orthonormal T = diag(H_outlier, H_inlier), float64 on the CPU.

    Same construction and random stream as paged_quant.py:50-68: each block is a
    Sylvester Hadamard on its largest power-of-two leading part (identity on the
    rest), rows scaled by random signs drawn with ``torch.rand(m, generator)``.
    """
    T = torch.eye(rank, dtype=torch.float64, device="cpu")
    for start, size in ((0, n_out), (n_out, rank - n_out)):
        if size <= 1:
            continue
        m = 1 << (size.bit_length() - 1)
        H = torch.ones(1, 1, dtype=torch.float64)
        while H.shape[0] < m:
            H = torch.cat([torch.cat([H, H], 1), torch.cat([H, -H], 1)], 0)
        u = torch.rand(m, generator=generator, device="cpu")
        signs = torch.where(u < 0.5, -1.0, 1.0).to(torch.float64)
        T[start:start + m, start:start + m] = signs[:, None] * H / math.sqrt(m)
    return T


@dataclass(frozen=True)
class QuantRow:
    """Byte layout of one token of a 3.2-bit layer (paged_quant.py:71-111)::

      [0, ks_off)        K codes, lanes 2k and 2k+1 in byte k
      [ks_off, vs_off)   K scales, (outlier, inlier) bf16 per KV head
      [vs_off, vq_off)   V scales, (outlier, inlier) bf16
      [vq_off, ...)      V codes, outlier channels first; row padded to 16 bytes
    """
    k_width: int
    num_kv_heads: int
    v_rank: int

    @property
    def v_nout(self) -> int:
        return n_outlier(self.v_rank)

    @property
    def ks_off(self) -> int:
        return self.k_width // 2

    @property
    def vs_off(self) -> int:
        return self.ks_off + 4 * self.num_kv_heads

    @property
    def vq_off(self) -> int:
        return self.vs_off + 4

    @property
    def v_nbo(self) -> int:
        return (self.v_nout + 1) // 2

    @property
    def v_bytes(self) -> int:
        return self.v_nbo + (self.v_rank - self.v_nout + 1) // 2

    @property
    def nbytes(self) -> int:
        return -(-(self.vq_off + self.v_bytes) // 16) * 16


def k_tables(ranks: list[int], device) -> tuple[torch.Tensor, torch.Tensor, tuple]:
    """(outlier lanes per head, head of every K lane, per-16-lane-tile (head,
    outlier lanes in the tile, last tile of its head)) -- paged_quant.py:114-131."""
    nouts = [n_outlier(r) for r in ranks]
    lanes, head, t_out, last = [], [], [], []
    for h, (r, no) in enumerate(zip(ranks, nouts)):
        tiles = -(-r // 16)
        lanes.extend([h] * (16 * tiles))
        for j in range(tiles):
            head.append(h)
            t_out.append(max(0, min(16, no - 16 * j)))
            last.append(int(j == tiles - 1))

    def t(v):
        return torch.tensor(v, dtype=torch.int32, device=device)
    return t(nouts), t(lanes), (t(head), t(t_out), t(last))


# ---------------------------------------------------------------------------
# write side
# ---------------------------------------------------------------------------

def pack_kv(k_codes, v_codes, cache, slot_mapping, row: QuantRow, k_ranks, k_offsets, k_nouts,
            status: torch.Tensor | None = None):
    """Quantize the step's codes into their slots of ``cache`` [num_blocks, block_size, row bytes]."""
    n = k_codes.shape[0]
    assert k_codes.stride(-1) == 1 and v_codes.stride(-1) == 1
    assert cache.dtype == torch.uint8 and cache.stride(-1) == 1
    if n == 0:
        return
    a = _lib.PackArgs()
    a.k_codes, a.k_stride0, a.k_dtype = k_codes.data_ptr(), k_codes.stride(0), _lib.dtype_code(k_codes)
    a.v_codes, a.v_stride0, a.v_dtype = v_codes.data_ptr(), v_codes.stride(0), _lib.dtype_code(v_codes)
    a.cache, a.cache_stride = cache.data_ptr(), _lib.i64s(cache.stride()[:2])
    a.num_blocks, a.block_size = cache.shape[0], cache.shape[1]
    a.slot_mapping, a.slot_dtype = slot_mapping.data_ptr(), _lib.dtype_code(slot_mapping)
    a.n, a.num_kv_heads, a.k_width, a.v_rank = n, row.num_kv_heads, row.k_width, row.v_rank
    a.k_ranks, a.k_offsets, a.k_nouts = k_ranks.data_ptr(), k_offsets.data_ptr(), k_nouts.data_ptr()
    a.ks_off, a.vs_off, a.vq_off = row.ks_off, row.vs_off, row.vq_off
    a.v_nout, a.v_nbo, a.v_bytes = row.v_nout, row.v_nbo, row.v_bytes
    a.status = None if status is None else status.data_ptr()
    _lib.check(_lib.lib().starkv_pack_kv_q32(a, _lib.stream_ptr(cache.device)), "pack_kv")


# ---------------------------------------------------------------------------
# decode
# ---------------------------------------------------------------------------

def fold_q(q, k_up, head_of_lane, scale, *, status=None):
    """q [n, H, 128] (RoPE applied), U^T [W, 128] -> A|B [n, W, 128] f16 with the
    logit scale folded in (paged_quant.py:241-255):

      A[r,i] = q_i U[r,i] + q_{i+64} U[r,i+64]      B[r,i] = q_{i+64} U[r,i] - q_i U[r,i+64]

    ``status`` (optional device int32 tensor): a ``head_of_lane`` entry outside
    ``[0, H)`` gives a zero row and is recorded there as STARKV_EBOUNDS (105)."""
    n, W = q.shape[0], k_up.shape[0]
    assert q.stride(-1) == 1 and k_up.stride(-1) == 1
    ab = torch.empty(n, W, HEAD_DIM, device=q.device, dtype=torch.float16)
    qs = (C.c_int64 * 3)(*q.stride())
    us = (C.c_int64 * 2)(*k_up.stride())
    st = _lib.lib().starkv_fold_q(q.data_ptr(), qs, _lib.dtype_code(q), k_up.data_ptr(), us, _lib.dtype_code(k_up),
                                  head_of_lane.data_ptr(), n, q.shape[1], W, float(scale), ab.data_ptr(),
                                  _lib.ptr(status), _lib.stream_ptr(q.device))
    _lib.check(st, "fold_q")
    return ab


def paged_quant_decode(
    query: torch.Tensor,          # [n, H, 128], RoPE already applied
    kv_cache: torch.Tensor,       # [num_blocks, block_size, row.nbytes] uint8 (inner stride 1)
    block_table: torch.Tensor,    # [n, max_blocks] int32
    seq_lens: torch.Tensor,       # [n] int32, including the token just written
    max_seq_len: int,             # host-side bound on seq_lens (max_model_len in a CUDA graph)
    row: QuantRow,
    k_up: torch.Tensor,           # [k_width, 128]  U^T, heads side by side
    head_of_lane: torch.Tensor,   # [k_width] int32
    k_tiles: tuple,               # per-16-lane-tile (head, outlier lanes, is last) from k_tables
    v_up_by_q: torch.Tensor,      # [H, v_rank, 128]
    cos_sin_cache: torch.Tensor,  # [max_positions, 128] = cat(cos, sin)
    scale: float,
    target_v_programs: int = 2048,   # accepted for compatibility; work split is automatic
    *,
    out: torch.Tensor | None = None,
    ws: torch.Tensor | None = None,
    context: tuple[int, int] | None = None,
    partial: torch.Tensor | None = None,
):
    """Returns the attention output per query head, ``[n, H, 128]`` in ``v_up_by_q.dtype``.

    With ``context=(rank, world)`` the call decodes only this rank's share of every
    sequence (context-parallel decode, starkv_b200.context_parallel) and returns
    ``(out, m, l)``: ``out`` f32 ``[n, H, 128]`` unnormalised, ``m`` / ``l`` f32
    ``[n, H]`` the rank's per-head logit max and softmax denominator.
    The three are views of one packed f32 buffer (``partial``, allocated when not
    given; see ``context_parallel.partial_views``)."""
    n, H, D = query.shape
    # the reference's own preconditions (paged_quant.py:374-376)
    assert D == HEAD_DIM and H == row.num_kv_heads, "4-bit decode: MHA, head_dim 128"
    assert kv_cache.dtype == torch.uint8 and kv_cache.shape[-1] == row.nbytes
    assert cos_sin_cache.shape[-1] == D and cos_sin_cache.shape[0] >= max_seq_len
    if context is not None:
        out, m_out, l_out = context_parallel.partial_views(query.shape[0], query.shape[1], query.device, partial)
    if out is None:
        out = torch.empty((n, H, D), dtype=v_up_by_q.dtype, device=query.device)
    if n == 0:
        return (out, m_out.fill_(float("-inf")), l_out.zero_()) if context is not None else out
    th, tn, tlast = k_tiles
    need = workspace.bytes_needed(n, H, H, row.k_width, row.v_rank, max_seq_len)
    if ws is None:
        ws = workspace.get(query.device, need)
    a = _lib.DecodeArgs()
    a.query, a.q_stride, a.q_dtype = query.data_ptr(), _lib.i64s(query.stride()), _lib.dtype_code(query)
    a.kv_cache, a.cache_stride, a.cache_dtype = kv_cache.data_ptr(), _lib.i64s(kv_cache.stride()), _lib.U8
    a.num_blocks, a.block_size = kv_cache.shape[0], kv_cache.shape[1]
    a.block_table, a.bt_stride, a.max_blocks = block_table.data_ptr(), _lib.i64s(block_table.stride()), \
        block_table.shape[1]
    a.seq_lens = seq_lens.data_ptr()
    a.n, a.num_heads, a.num_kv_heads, a.head_dim = n, H, H, D
    a.max_seq_len = int(max_seq_len)
    a.k_up, a.k_up_stride, a.k_up_dtype = k_up.data_ptr(), _lib.i64s(k_up.stride()), _lib.dtype_code(k_up)
    a.k_width = row.k_width
    a.v_up_by_q, a.v_up_stride, a.v_up_dtype = v_up_by_q.data_ptr(), _lib.i64s(v_up_by_q.stride()), \
        _lib.dtype_code(v_up_by_q)
    a.v_rank = row.v_rank
    a.cos_sin_cache, a.cs_stride, a.cs_dtype, a.cs_rows = cos_sin_cache.data_ptr(), \
        _lib.i64s(cos_sin_cache.stride()), _lib.dtype_code(cos_sin_cache), cos_sin_cache.shape[0]
    a.scale = float(scale)
    a.out, a.out_stride, a.out_dtype = out.data_ptr(), _lib.i64s(out.stride()), _lib.dtype_code(out)
    a.row_nbytes, a.ks_off, a.vs_off, a.vq_off = row.nbytes, row.ks_off, row.vs_off, row.vq_off
    a.v_nout, a.v_nbo, a.v_bytes = row.v_nout, row.v_nbo, row.v_bytes
    a.head_of_lane = head_of_lane.data_ptr()
    a.tile_head, a.tile_nout, a.tile_last = th.data_ptr(), tn.data_ptr(), tlast.data_ptr()
    if context is not None:
        rank, world = context
        st = _lib.lib().starkv_paged_decode_q32_partial(a, int(rank), int(world), m_out.data_ptr(), l_out.data_ptr(),
                                     ws.data_ptr(), ws.numel(), _lib.stream_ptr(query.device))
        _lib.check(st, "paged_quant_decode")
        return out, m_out, l_out
    st = _lib.lib().starkv_paged_decode_q32(a, ws.data_ptr(), ws.numel(), _lib.stream_ptr(query.device))
    _lib.check(st, "paged_quant_decode")
    return out
