"""Seeded synthetic STAR-KV layers with the shapes and value distributions of the
benchmark configurations (Llama-2-7B attention geometry: 32 heads, head_dim 128).

No public dataset is involved: the reference benchmarks random-token prompts
(bench_serving.py:235-237), which these seeded tensors stand in for.

* K ranks per head uniform over {16, 32, 48, 64}; V: one latent shared by all
  heads whose width is the sum of 32 per-head draws from {32, 64}.
* Skewed variant (mixed-length batch): K = 16k, k in 1..8 with P ~ 0.5^(k-1);
  per-head V = 32k, k in 1..4 with P ~ 0.25^(k-1), summed.
* Codes and queries ~ N(0, 1); B_k rows of head h ~ N(0, 1/sqrt(rank_h)) (std),
  B_v ~ N(0, 1/sqrt(v_rank)); lanes between a head's rank and its 16-aligned
  width are zero, as the fused checkpoint's zero rows make them.
* Paged cache with 16-token pages; the block table is a seeded permutation of
  the physical pages, page 0 is the reserved null block.
* 3.2-bit layers: codes are rotated by the block Hadamard (per K head and for V,
  a fresh generator seeded 1234 per projection, as the checkpoint loader
  does) and packed with the library's bit-exact packer.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from .kernels import paged_quant as pq

HEAD_DIM = 128
PAGE = 16


def align16(x: int) -> int:
    return -(-int(x) // 16) * 16


def sample_ranks(num_heads: int, seed: int, skewed: bool = False) -> tuple[list[int], int]:
    rng = np.random.default_rng(seed)
    if skewed:
        pk = 0.5 ** np.arange(8)
        k = rng.choice(np.arange(1, 9), size=num_heads, p=pk / pk.sum())
        pv = 0.25 ** np.arange(4)
        v = rng.choice(np.arange(1, 5), size=num_heads, p=pv / pv.sum())
        return [int(16 * x) for x in k], int(32 * v.sum())
    k = rng.choice([16, 32, 48, 64], size=num_heads)
    v = rng.choice([32, 64], size=num_heads)
    return [int(x) for x in k], int(v.sum())


def rope_cos_sin(max_pos: int, device, dtype=torch.bfloat16, base: float = 10000.0) -> torch.Tensor:
    """vLLM-style rotary ``cos_sin_cache`` [max_pos, 128] = cat(cos, sin), Llama frequencies."""
    inv = 1.0 / (base ** (torch.arange(0, HEAD_DIM, 2, dtype=torch.float32, device=device) / HEAD_DIM))
    fr = torch.arange(max_pos, dtype=torch.float32, device=device)[:, None] * inv[None, :]
    return torch.cat([fr.cos(), fr.sin()], 1).to(dtype)


@dataclass
class Layer:
    """One synthetic layer and its decode inputs (device tensors + host metadata)."""
    quant: bool
    ranks: list[int]
    v_rank: int
    k_width: int
    offsets: list[int]
    seq_lens_host: list[int]
    query: torch.Tensor
    kv_cache: torch.Tensor
    block_table: torch.Tensor
    seq_lens: torch.Tensor
    k_up: torch.Tensor
    k_ranks: torch.Tensor
    k_head_offsets: torch.Tensor
    v_up_by_q: torch.Tensor
    cos_sin_cache: torch.Tensor
    scale: float
    max_seq_len: int
    row: pq.QuantRow | None = None
    k_nouts: torch.Tensor | None = None
    head_of_lane: torch.Tensor | None = None
    k_tiles: tuple | None = None
    extra: dict = field(default_factory=dict)

    @property
    def n(self) -> int:
        return len(self.seq_lens_host)

    @property
    def num_heads(self) -> int:
        return self.query.shape[1]

    def kv_tokens(self) -> int:
        return int(sum(self.seq_lens_host))

    def algorithmic_bytes(self) -> int:
        """HBM bytes one decode step must move (per-token payload + weights + tables)."""
        H, n = self.num_heads, self.n
        T = self.kv_tokens()
        if self.quant:
            per_tok = self.k_width // 2 + 4 * len(self.ranks) + 4 + self.row.v_bytes
        else:
            per_tok = 2 * (self.k_width + self.v_rank)
        pages = sum(-(-L // PAGE) for L in self.seq_lens_host)
        return (T * per_tok + 2 * self.k_width * HEAD_DIM + 2 * H * self.v_rank * HEAD_DIM + 4 * pages
                + 2 * n * H * HEAD_DIM * 2)

    def algorithmic_flops(self) -> int:
        T = self.kv_tokens()
        H = self.num_heads
        return T * (2 * self.k_width * HEAD_DIM + 2 * self.k_width + 2 * H * self.v_rank) + \
            2 * self.n * H * self.v_rank * HEAD_DIM


def _paged_table(seq_lens: list[int], gen: torch.Generator, device, max_blocks: int | None = None):
    pages = [-(-L // PAGE) for L in seq_lens]
    total = sum(pages)
    mb = max(max(pages), 1) if max_blocks is None else max_blocks
    perm = torch.randperm(total, generator=gen) + 1          # page 0 = null block
    bt = torch.zeros(len(seq_lens), mb, dtype=torch.int32)
    o = 0
    for b, p in enumerate(pages):
        bt[b, :p] = perm[o:o + p].to(torch.int32)
        o += p
    return bt.to(device), total + 1


def make_layer(seq_lens: list[int], num_heads: int = 32, quant: bool = False, seed: int = 0,
               device="cuda", skewed: bool = False, ranks: list[int] | None = None,
               v_rank: int | None = None, num_kv_heads: int | None = None, max_seq_len: int | None = None,
               dtype=torch.bfloat16, chunk_tokens: int = 1 << 16) -> Layer:
    """Build a layer. ``seq_lens`` per sequence; ranks drawn from the config sampler
    unless given. GQA (num_kv_heads < num_heads) only for bf16 codes."""
    device = torch.device(device)
    hkv = num_kv_heads or num_heads
    if ranks is None:
        ranks, rv = sample_ranks(hkv, seed, skewed)
    else:
        rv = v_rank
    if not quant:
        rv = align16(rv)
    widths = [align16(r) for r in ranks]
    offsets = [sum(widths[:h]) for h in range(hkv)]
    W = sum(widths)
    g_cpu = torch.Generator().manual_seed(seed + 1)
    g = torch.Generator(device=device).manual_seed(seed + 2)
    bt, num_blocks = _paged_table(seq_lens, g_cpu, device)
    max_seq_len = max_seq_len or max(max(seq_lens), 1)
    n = len(seq_lens)

    k_up = torch.zeros(W, HEAD_DIM, device=device, dtype=torch.float32)
    for r, o in zip(ranks, offsets):
        k_up[o:o + r] = torch.randn(r, HEAD_DIM, generator=g, device=device) / r ** 0.5
    v_up_by_q = (torch.randn(num_heads, rv, HEAD_DIM, generator=g, device=device) / rv ** 0.5).to(dtype)
    query = torch.randn(n, num_heads, HEAD_DIM, generator=g, device=device).to(dtype)
    cs = rope_cos_sin(max_seq_len, device, dtype)
    common = dict(ranks=list(ranks), v_rank=rv, k_width=W, offsets=offsets, seq_lens_host=list(seq_lens),
                  query=query, block_table=bt, seq_lens=torch.tensor(seq_lens, dtype=torch.int32, device=device),
                  k_ranks=torch.tensor(ranks, dtype=torch.int32, device=device),
                  k_head_offsets=torch.tensor(offsets, dtype=torch.int32, device=device),
                  v_up_by_q=v_up_by_q, cos_sin_cache=cs, scale=HEAD_DIM ** -0.5, max_seq_len=max_seq_len)
    if not quant:
        cache = torch.randn(num_blocks, PAGE, W + rv, generator=g, device=device, dtype=dtype)
        for r, o, w in zip(ranks, offsets, widths):
            if w > r:
                cache[..., o + r:o + w] = 0
        return Layer(quant=False, kv_cache=cache, k_up=k_up.to(dtype), **common)

    assert hkv == num_heads, "3.2-bit cache: MHA only"
    row = pq.QuantRow(W, hkv, rv)
    # rotate K rows of k_up by each head's block Hadamard, V by the layer's (the
    # loader's fold, checkpoint.py:96-103); codes are drawn already in the rotated basis
    gk = torch.Generator().manual_seed(pq.HADAMARD_SEED)
    Tk = [pq.block_hadamard(r, pq.n_outlier(r), gk).to(device=device, dtype=torch.float32) for r in ranks]
    for T, r, o in zip(Tk, ranks, offsets):
        k_up[o:o + r] = T.t() @ k_up[o:o + r]
    gv = torch.Generator().manual_seed(pq.HADAMARD_SEED)
    Tv = pq.block_hadamard(rv, pq.n_outlier(rv), gv).to(device=device, dtype=torch.float32)
    k_up = k_up.to(dtype)
    nouts, hol, tiles = pq.k_tables(ranks, device)
    cache = torch.zeros(num_blocks, PAGE, row.nbytes, dtype=torch.uint8, device=device)
    total = num_blocks * PAGE
    slots_all = torch.arange(total, device=device, dtype=torch.int64)
    for s0 in range(0, total, chunk_tokens):
        s1 = min(total, s0 + chunk_tokens)
        m = s1 - s0
        kc = torch.randn(m, W, generator=g, device=device)
        for T, r, o, w in zip(Tk, ranks, offsets, widths):
            kc[:, o:o + r] = kc[:, o:o + r] @ T
            if w > r:
                kc[:, o + r:o + w] = 0
        vc = torch.randn(m, rv, generator=g, device=device) @ Tv
        pq.pack_kv(kc.to(dtype), vc.to(dtype), cache, slots_all[s0:s1], row,
                   common["k_ranks"], common["k_head_offsets"], nouts)
    return Layer(quant=True, kv_cache=cache, k_up=k_up, row=row, k_nouts=nouts, head_of_lane=hol,
                 k_tiles=tiles, **common)


def gather_rows(layer: Layer, b: int) -> torch.Tensor:
    """Cache rows of sequence b's tokens, [L, width] on the CPU (for oracle checks)."""
    L = layer.seq_lens_host[b]
    pos = torch.arange(L, device=layer.kv_cache.device)
    blk = layer.block_table[b, pos // PAGE].long()
    return layer.kv_cache[blk, pos % PAGE].cpu()
