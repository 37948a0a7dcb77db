"""Paged STAR-KV decode attention over bf16 / f16 codes, on the sm_100a library.

Drop-in for ``starkv_serve/kernels/paged_decode.py``: ``paged_starkv_decode`` keeps
the reference signature and result (paged_decode.py:150-226) and is called from
the same place (attention.py:204-207). The work runs in
``starkv_paged_decode_bf16`` (include/starkv_b200.h): fold the query into the K
up-projection, tcgen05 logits over the paged K codes, tcgen05 P.V over the shared
V codes, lift with ``v_up_by_q``. No torch math runs on this path and there is no
fallback: if the native library is missing the call raises.
"""
from __future__ import annotations

import torch

from .. import _lib, context_parallel, workspace

# Kept for call-site compatibility with the reference (paged_decode.py:22-28);
# the tile shapes of this implementation are fixed inside the library.
BLOCK_L = 128
TARGET_V_PROGRAMS = 256


def paged_starkv_decode(
    query: torch.Tensor,          # [n, H_q, head_dim], RoPE already applied
    kv_cache: torch.Tensor,       # [num_blocks, block_size, width] (inner stride 1)
    block_table: torch.Tensor,    # [n, max_blocks] int32
    seq_lens: torch.Tensor,       # [n] int32, including the token just written
    max_seq_len: int,             # host-side bound on seq_lens (max_model_len in a CUDA graph)
    k_up: torch.Tensor,           # [k_width, head_dim]  U^T, heads side by side
    k_ranks: torch.Tensor,        # [H_kv] int32
    k_head_offsets: torch.Tensor, # [H_kv] int32
    k_width: int,
    v_up_by_q: torch.Tensor,      # [H_q, v_rank, head_dim]
    cos_sin_cache: torch.Tensor,  # [max_positions, head_dim] = cat(cos, sin)
    scale: float,
    v_programs: int = TARGET_V_PROGRAMS,  # accepted for compatibility; work split is automatic
    *,
    out: torch.Tensor | None = None,
    ws: torch.Tensor | None = None,
    context: tuple[int, int] | None = None,
    partial: torch.Tensor | None = None,
):
    """Returns the attention output per query head, ``[n, H_q, head_dim]`` in
    ``v_up_by_q.dtype`` (paged_decode.py:166).

    With ``context=(rank, world)`` the call decodes only this rank's share of every
    sequence (context-parallel decode, starkv_b200.context_parallel) and returns
    ``(out, m, l)``: ``out`` f32 ``[n, H, 128]`` unnormalised, ``m`` / ``l`` f32
    ``[n, H]`` the rank's per-head logit max and softmax denominator.
    The three are views of one packed f32 buffer (``partial``, allocated when not
    given; see ``context_parallel.partial_views``)."""
    n, num_heads, head_dim = query.shape
    num_kv_heads = k_ranks.numel()
    v_rank = v_up_by_q.shape[1]
    # the reference's own preconditions (paged_decode.py:172-174)
    assert head_dim % 2 == 0 and num_heads % num_kv_heads == 0
    assert kv_cache.shape[-1] == k_width + v_rank, "cache width != K codes + V codes"
    assert cos_sin_cache.shape[-1] == head_dim and cos_sin_cache.shape[0] >= max_seq_len
    if context is not None:
        out, m_out, l_out = context_parallel.partial_views(query.shape[0], query.shape[1], query.device, partial)
    if out is None:
        out = torch.empty((n, num_heads, head_dim), dtype=v_up_by_q.dtype, device=query.device)
    if n == 0:
        return (out, m_out.fill_(float("-inf")), l_out.zero_()) if context is not None else out
    k_ranks = k_ranks if k_ranks.dtype == torch.int32 else k_ranks.to(torch.int32)
    k_head_offsets = k_head_offsets if k_head_offsets.dtype == torch.int32 else k_head_offsets.to(torch.int32)
    block_table = block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)
    seq_lens = seq_lens if seq_lens.dtype == torch.int32 else seq_lens.to(torch.int32)
    need = workspace.bytes_needed(n, num_heads, num_kv_heads, k_width, v_rank, max_seq_len)
    if ws is None:
        ws = workspace.get(query.device, need)
    a = _lib.DecodeArgs()
    a.query, a.q_stride, a.q_dtype = query.data_ptr(), _lib.i64s(query.stride()), _lib.dtype_code(query)
    a.kv_cache, a.cache_stride, a.cache_dtype = kv_cache.data_ptr(), _lib.i64s(kv_cache.stride()), \
        _lib.dtype_code(kv_cache)
    a.num_blocks, a.block_size = kv_cache.shape[0], kv_cache.shape[1]
    a.block_table, a.bt_stride, a.max_blocks = block_table.data_ptr(), _lib.i64s(block_table.stride()), \
        block_table.shape[1]
    a.seq_lens = seq_lens.data_ptr()
    a.n, a.num_heads, a.num_kv_heads, a.head_dim = n, num_heads, num_kv_heads, head_dim
    a.max_seq_len = int(max_seq_len)
    a.k_up, a.k_up_stride, a.k_up_dtype = k_up.data_ptr(), _lib.i64s(k_up.stride()), _lib.dtype_code(k_up)
    a.k_ranks, a.k_head_offsets, a.k_width = k_ranks.data_ptr(), k_head_offsets.data_ptr(), int(k_width)
    a.v_up_by_q, a.v_up_stride, a.v_up_dtype = v_up_by_q.data_ptr(), _lib.i64s(v_up_by_q.stride()), \
        _lib.dtype_code(v_up_by_q)
    a.v_rank = v_rank
    a.cos_sin_cache, a.cs_stride, a.cs_dtype, a.cs_rows = cos_sin_cache.data_ptr(), \
        _lib.i64s(cos_sin_cache.stride()), _lib.dtype_code(cos_sin_cache), cos_sin_cache.shape[0]
    a.scale = float(scale)
    a.out, a.out_stride, a.out_dtype = out.data_ptr(), _lib.i64s(out.stride()), _lib.dtype_code(out)
    if context is not None:
        rank, world = context
        st = _lib.lib().starkv_paged_decode_bf16_partial(a, int(rank), int(world), m_out.data_ptr(), l_out.data_ptr(),
                                     ws.data_ptr(), ws.numel(), _lib.stream_ptr(query.device))
        _lib.check(st, "paged_starkv_decode")
        return out, m_out, l_out
    st = _lib.lib().starkv_paged_decode_bf16(a, ws.data_ptr(), ws.numel(), _lib.stream_ptr(query.device))
    _lib.check(st, "paged_starkv_decode")
    return out


def write_kv_bf16(key: torch.Tensor, value: torch.Tensor, kv_cache: torch.Tensor, slot_mapping: torch.Tensor,
                  status: torch.Tensor | None = None) -> None:
    """``cache[slot // bs, slot % bs] = cat(key, value)`` with slot -1 sent to the
    null block (attention.py:179-185), on the library's cache-write kernel."""
    n = key.shape[0]
    if n == 0:
        return
    assert key.stride(-1) == 1 and value.stride(-1) == 1
    a = _lib.CacheWriteArgs()
    a.key, a.key_stride0, a.key_dtype = key.data_ptr(), key.stride(0), _lib.dtype_code(key)
    a.value, a.value_stride0, a.value_dtype = value.data_ptr(), value.stride(0), _lib.dtype_code(value)
    a.cache, a.cache_stride, a.cache_dtype = kv_cache.data_ptr(), _lib.i64s(kv_cache.stride()), \
        _lib.dtype_code(kv_cache)
    a.num_blocks, a.block_size = kv_cache.shape[0], kv_cache.shape[1]
    a.slot_mapping, a.slot_dtype = slot_mapping.data_ptr(), _lib.dtype_code(slot_mapping)
    a.n, a.k_width, a.v_rank = n, key.shape[1], value.shape[1]
    a.status = None if status is None else status.data_ptr()
    _lib.check(_lib.lib().starkv_cache_write_bf16(a, _lib.stream_ptr(kv_cache.device)), "write_kv_bf16")


def kv_down_write(hidden: torch.Tensor, kv_down: torch.Tensor, kv_cache: torch.Tensor, slot_mapping: torch.Tensor,
                  status: torch.Tensor | None = None) -> None:
    """The step's codes straight into the cache: ``cache[slot] = hidden . kv_down^T``
    (model.py:70 ``F.linear(hidden, kv_down)`` followed by the cache write of
    attention.py:179-185, slot -1 sent to the null block), in one launch of the
    library's fused GEMM + write kernel. hidden [n, hidden_dim], kv_down [W + rv,
    hidden_dim], both in the cache's dtype (bf16 or f16); hidden_dim a multiple of 512."""
    n = hidden.shape[0]
    if n == 0:
        return
    if hidden.stride(-1) != 1 or kv_down.stride(-1) != 1:
        raise ValueError("kv_down_write: hidden and kv_down need a contiguous last dimension")
    if hidden.dtype != kv_cache.dtype or kv_down.dtype != kv_cache.dtype:
        raise ValueError("kv_down_write: hidden, kv_down and the cache must share one dtype")
    st = _lib.lib().starkv_kv_down_cache_write(
        hidden.data_ptr(), hidden.stride(0), kv_down.data_ptr(), kv_down.stride(0), _lib.dtype_code(hidden), n,
        hidden.shape[1], kv_down.shape[0], kv_cache.data_ptr(), _lib.i64s(kv_cache.stride()[:2]), kv_cache.shape[0],
        kv_cache.shape[1], slot_mapping.data_ptr(), _lib.dtype_code(slot_mapping), _lib.ptr(status),
        _lib.stream_ptr(kv_cache.device))
    _lib.check(st, "kv_down_write")
