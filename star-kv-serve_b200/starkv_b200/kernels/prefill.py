"""Causal attention of whole prompts for the dense prefill, on the sm_100a library.

Replaces the ``flash_attn_varlen_func`` call of the reference's prefill
(attention.py:246-250): each prompt attends causally over its own lifted, rotated
keys and lifted values. The work runs in ``starkv_prefill_attention``
(include/starkv_b200.h): tcgen05 Q.K^T and P.V with the accumulators in tensor
memory and an online softmax between them. There is no fallback: if the native
library is missing the call raises.
"""
from __future__ import annotations

import torch

from .. import _lib

HEAD_DIM = 128
Q_TILE = 128


def cu_seqlens_of(prompt_lens: list[int], device) -> torch.Tensor:
    """int32 prompt offsets [n + 1] (the reference's ``query_start_loc``)."""
    offs = [0]
    for L in prompt_lens:
        offs.append(offs[-1] + int(L))
    return torch.tensor(offs, dtype=torch.int32, device=device)


def prefill_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, prompt_lens: list[int], scale: float,
                      *, cu_seqlens: torch.Tensor | None = None, out: torch.Tensor | None = None,
                      status: torch.Tensor | None = None) -> torch.Tensor:
    """``out[t, h] = softmax_k(scale q[t, h] . k[k, h // (H / H_k)]) v[k, h // (H / H_v)]``
    over the keys of t's own prompt up to t (causal), prompts back to back in the
    token dimension (``prompt_lens``, host ints).

    q [T, H, 128], k [T, H_k, 128], v [T, H_v, 128] (H_v = H: one V per query head,
    as the layer lifts it with ``v_up_by_q``; H_v = H_k: per KV head, as the
    reference does), bf16 or f16, last dimension contiguous. Returns out [T, H, 128]
    in q's dtype."""
    T, H, D = q.shape
    if D != HEAD_DIM or k.shape[-1] != HEAD_DIM or v.shape[-1] != HEAD_DIM:
        raise ValueError("prefill_attention: head_dim must be 128")
    if k.shape[0] != T or v.shape[0] != T:
        raise ValueError("prefill_attention: q, k and v must hold the same tokens")
    if sum(int(L) for L in prompt_lens) != T:
        raise ValueError("prefill_attention: prompt_lens must cover the T tokens")
    if q.dtype not in (torch.bfloat16, torch.float16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("prefill_attention: q, k and v must be bf16 or f16, all the same")
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.stride(-1) != 1:
            raise ValueError(f"prefill_attention: {name} needs a contiguous last dimension")
    if out is None:
        out = torch.empty((T, H, HEAD_DIM), dtype=q.dtype, device=q.device)
    if T == 0:
        return out
    if cu_seqlens is None:
        cu_seqlens = cu_seqlens_of(prompt_lens, q.device)
    q_tiles = sum(-(-int(L) // Q_TILE) for L in prompt_lens)
    st = _lib.lib().starkv_prefill_attention(
        q.data_ptr(), _lib.i64s(q.stride()[:2]), k.data_ptr(), _lib.i64s(k.stride()[:2]),
        v.data_ptr(), _lib.i64s(v.stride()[:2]), _lib.dtype_code(q), T, H, k.shape[1], v.shape[1],
        cu_seqlens.data_ptr(), len(prompt_lens), q_tiles, float(scale), out.data_ptr(),
        _lib.i64s(out.stride()[:2]), _lib.ptr(status), _lib.stream_ptr(q.device))
    _lib.check(st, "prefill_attention")
    return out
