"""Context-parallel decode: each rank decodes, for all heads, its share of every
sequence (its contiguous run of 256-token tiles) with
``paged_starkv_decode(..., context=(rank, world))`` or
``paged_quant_decode(..., context=...)``, and the ranks' partial results are
combined exactly:

    M = max_r m_r,   out = sum_r exp(m_r - M) out_r / sum_r exp(m_r - M) l_r

(out_r is the rank's unnormalised, already lifted output, m_r / l_r its per-head
logit max and softmax denominator). Every rank reads 1/world of the K and V codes,
including the V latent that head sharding has to replicate. The exchange is one
MAX all-reduce of [n, H] and one SUM all-reduce of [n, H, 129] f32 (about 1 MB for
64 sequences x 32 heads).
"""
from __future__ import annotations

import torch


def _normalise(buf: torch.Tensor, dtype) -> torch.Tensor:
    num, den = buf[..., :-1], buf[..., -1:]
    return torch.where(den > 0, num / den.clamp_min(torch.finfo(torch.float32).tiny), torch.zeros_like(num)).to(dtype)


def combine(out: torch.Tensor, m: torch.Tensor, l: torch.Tensor, group=None, dtype=torch.bfloat16) -> torch.Tensor:
    """All ranks of `group` call this with their partial (out, m, l); every rank gets
    the combined [n, H, 128] output in `dtype`."""
    import torch.distributed as dist
    M = m.clone()
    dist.all_reduce(M, op=dist.ReduceOp.MAX, group=group)
    s = torch.exp(m - M)                                   # 0 where this rank has no token
    buf = torch.cat([out * s.unsqueeze(-1), (l * s).unsqueeze(-1)], -1)
    dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)
    return _normalise(buf, dtype)


def combine_local(parts: list[tuple[torch.Tensor, torch.Tensor, torch.Tensor]], dtype=torch.bfloat16) -> torch.Tensor:
    """The same combination for partial results held by one process (tests, one GPU)."""
    M = torch.stack([m for _, m, _ in parts]).amax(0)
    buf = None
    for out, m, l in parts:
        s = torch.exp(m - M)
        t = torch.cat([out * s.unsqueeze(-1), (l * s).unsqueeze(-1)], -1)
        buf = t if buf is None else buf + t
    return _normalise(buf, dtype)
