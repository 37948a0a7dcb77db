"""One compressed attention layer's decode step: the callers on either side of the
paged low-rank decode, as StarKVLlamaAttention.forward (model.py:68-74) and
StarKVAttentionImpl.forward (attention.py:168-212) run them, on this library's
kernels:

    q      = rope(hidden . Wq^T)              Q rows of qkv_proj, neox rotary from the
                                              [cos | sin] table (vLLM forward_native)
    codes  = hidden . kv_down^T = [k_codes | v_codes]     (checkpoint.py:154 fuse)
    cache <- codes at slot_mapping            bf16 row write, or the 3.2-bit pack
    attn   = paged decode(q, cache, ...)      starkv_b200.kernels
    out    = attn . Wo^T                      o_proj

The GEMMs are plain library GEMMs (torch / cuBLAS). Tensor parallel over heads,
which the reference rejects (model.py:32-33): rank r keeps its KV heads (LPT on K
width, starkv_b200.sharding) - their Q rows, K rows of kv_down, k_up rows,
v_up_by_q rows and o_proj columns - and the whole V part of kv_down (the V latent
is read by every head); the o_proj partial sums are all-reduced over the group.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import context_parallel, sharding
from .collectives import all_reduce_
from .kernels import paged_quant as pq
from .kernels.paged_decode import kv_down_write, paged_starkv_decode, write_kv_bf16
from .kernels.prefill import prefill_attention

HEAD_DIM = 128


@dataclass
class AttnWeights:
    """Full (unsharded) weights of one compressed attention layer."""
    wq: torch.Tensor          # [Hq * Hd, hidden]
    kv_down: torch.Tensor     # [W + rv, hidden]: K code rows (heads at 16-lane widths), then V
    wo: torch.Tensor          # [hidden, Hq * Hd]
    k_up: torch.Tensor        # [W, Hd]
    v_up_by_q: torch.Tensor   # [Hq, rv, Hd]
    k_ranks: list[int]        # per KV head
    v_rank: int
    num_heads: int
    num_kv_heads: int
    rotated: bool = False     # K/V factors already in the 3.2-bit cache's rotated basis

    @classmethod
    def from_checkpoint(cls, lw, wq: torch.Tensor, wo: torch.Tensor, num_heads: int, device=None,
                        dtype=torch.bfloat16) -> "AttnWeights":
        """The layer's weights from a fused checkpoint layer (starkv_b200.checkpoint,
        the serving layout) plus the model's q_proj / o_proj rows, as
        StarKVAttentionImpl.to_device builds them (attention.py:134-166): kv_down =
        [k_down | v_down], k_up as stored, and one V up-projection per KV head,
        repeated over that head's query heads, as v_up_by_q [Hq, rv, Hd]. A checkpoint
        loaded with kv_quant carries the Hadamard rotations already (rotated=True)."""
        H = lw.k_head_ranks.numel()
        if num_heads % H:
            raise ValueError(f"{num_heads} query heads do not group over {H} KV heads")
        dev = device if device is not None else wq.device
        v_up_by_q = (lw.v_up.view(H, HEAD_DIM, lw.v_rank).repeat_interleave(num_heads // H, dim=0)
                     .transpose(-1, -2))
        return cls(wq=wq.to(device=dev, dtype=dtype), kv_down=torch.cat([lw.k_down, lw.v_down]).to(dev, dtype),
                   wo=wo.to(device=dev, dtype=dtype), k_up=lw.k_up.to(dev, dtype).contiguous(),
                   v_up_by_q=v_up_by_q.to(dev, dtype).contiguous(), k_ranks=[int(r) for r in lw.k_head_ranks],
                   v_rank=lw.v_rank, num_heads=num_heads, num_kv_heads=H, rotated=lw.kv_quant)


def random_weights(hidden: int, num_heads: int, ranks: list[int], v_rank: int, seed: int = 0,
                   num_kv_heads: int | None = None, device="cuda", dtype=torch.bfloat16) -> AttnWeights:
    """Seeded random-init weights of the layer's shapes (std 1/sqrt(fan-in), K/V
    factors 1/sqrt(rank); K rows past a head's rank are zero, as the loader pads)."""
    hkv = num_kv_heads or num_heads
    g = torch.Generator(device=device).manual_seed(seed)
    offs = sharding.k_offsets(ranks)
    W = sum(sharding.align16(r) for r in ranks)

    def rnd(*shape, std):
        return (torch.randn(*shape, generator=g, device=device) * std).to(dtype)

    kv_down = rnd(W + v_rank, hidden, std=hidden ** -0.5)
    k_up = torch.zeros(W, HEAD_DIM, device=device, dtype=dtype)
    for r, o in zip(ranks, offs):
        kv_down[o + r:o + sharding.align16(r)] = 0
        k_up[o:o + r] = rnd(r, HEAD_DIM, std=r ** -0.5)
    # one V up-projection per KV head, repeated over its query heads (attention.py:158-160)
    v_up_by_q = rnd(hkv, v_rank, HEAD_DIM, std=v_rank ** -0.5).repeat_interleave(num_heads // hkv, dim=0)
    return AttnWeights(wq=rnd(num_heads * HEAD_DIM, hidden, std=hidden ** -0.5), kv_down=kv_down,
                       wo=rnd(hidden, num_heads * HEAD_DIM, std=(num_heads * HEAD_DIM) ** -0.5), k_up=k_up,
                       v_up_by_q=v_up_by_q.contiguous(), k_ranks=list(ranks), v_rank=v_rank, num_heads=num_heads,
                       num_kv_heads=hkv)


def rope(x: torch.Tensor, positions: torch.Tensor, cos_sin_cache: torch.Tensor) -> torch.Tensor:
    """Neox rotary of x [n, H, 128] at `positions` from the [P, 128] = [cos | sin] table."""
    cos, sin = cos_sin_cache[positions.long()].to(x.dtype).chunk(2, dim=-1)
    cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


class StarKVAttentionLayer:
    """The layer on one rank of a tensor-parallel group of `world` ranks (1: whole)."""

    def __init__(self, w: AttnWeights, cos_sin_cache: torch.Tensor, quant: bool = False, rank: int = 0,
                 world: int = 1, group=None):
        if quant and w.num_kv_heads != w.num_heads:
            raise NotImplementedError("3.2-bit cache: MHA only (paged_quant.py:374-376)")
        self.quant, self.rank, self.world, self.group = quant, rank, world, group
        self.cos_sin_cache = cos_sin_cache
        self.scale = HEAD_DIM ** -0.5
        gsize = w.num_heads // w.num_kv_heads
        heads = (list(range(w.num_kv_heads)) if world == 1 else sharding.lpt_shard(w.k_ranks, world)[rank])
        qh = sharding.query_heads(heads, gsize)
        ranks, offsets, W, lanes = sharding.shard_lanes(w.k_ranks, heads)
        W_full = sum(sharding.align16(r) for r in w.k_ranks)
        dev = w.wq.device
        lanes_t = torch.tensor(lanes, dtype=torch.long, device=dev)
        qh_t = torch.tensor(qh, dtype=torch.long, device=dev)
        hidden = w.wq.shape[1]
        self.heads, self.q_heads = heads, qh
        self.num_heads, self.num_kv_heads = len(qh), len(heads)
        self.k_ranks_host, self.k_width, self.v_rank = ranks, W, w.v_rank
        self.wq = w.wq.view(w.num_heads, HEAD_DIM, hidden)[qh_t].reshape(-1, hidden).contiguous()
        self.kv_down = torch.cat([w.kv_down[lanes_t], w.kv_down[W_full:]]).contiguous()
        self.wo = w.wo.view(hidden, w.num_heads, HEAD_DIM)[:, qh_t].reshape(hidden, -1).contiguous()
        self.k_up = w.k_up[lanes_t].contiguous()
        self.v_up_by_q = w.v_up_by_q[qh_t].contiguous()
        self.k_ranks = torch.tensor(ranks, dtype=torch.int32, device=dev)
        self.k_head_offsets = torch.tensor(offsets, dtype=torch.int32, device=dev)
        if quant:
            self.row = pq.QuantRow(W, len(heads), w.v_rank)
            self.k_nouts, self.head_of_lane, self.k_tiles = pq.k_tables(ranks, dev)
            if not w.rotated:   # a kv_quant checkpoint carries the rotations already
                self._fold_rotations(w.k_ranks, heads, offsets)
        else:
            self.row = None
        # prefill lifts every head in one bmm over a uniform width: codes gathered
        # into [T, Hkv, R] (R = the widest head; indices past a head's width repeat
        # its first lane and meet zero k_up rows), k_up padded to [Hkv, R, Hd]
        # (attention.py:146-156)
        R = max(sharding.align16(r) for r in ranks)
        idx = torch.empty(len(heads) * R, dtype=torch.long)
        kup = self.k_up.new_zeros(len(heads), R, HEAD_DIM)
        for i, (r, o) in enumerate(zip(ranks, offsets)):
            wdt = sharding.align16(r)
            idx[i * R:i * R + wdt] = torch.arange(o, o + wdt)
            idx[i * R + wdt:(i + 1) * R] = o
            kup[i, :wdt] = self.k_up[o:o + wdt]
        self.k_prefill_gather, self.k_up_T, self.k_max_width = idx.to(dev), kup.contiguous(), R

    def _fold_rotations(self, all_ranks: list[int], heads: list[int], offsets: list[int]) -> None:
        """3.2-bit codes are stored in a rotated basis (block Hadamard per K head and
        for the V latent, seeded, paged_quant.py:50-68); the rotations fold into the
        factors once, as the loader does (checkpoint.py:96-103, 140-153): code rows
        of kv_down and k_up rows become T^T x (so codes come out rotated and
        codes . k_up is unchanged), the V rows of kv_down and v_up_by_q likewise. The
        K rotations are drawn for every head in order, so a shard uses its heads'
        rotations of the whole layer."""
        dev, dt = self.kv_down.device, self.kv_down.dtype
        kd = self.kv_down.float()
        ku = self.k_up.float()
        gk = torch.Generator().manual_seed(pq.HADAMARD_SEED)
        rot = [pq.block_hadamard(r, pq.n_outlier(r), gk) for r in all_ranks]
        for h, o in zip(heads, offsets):
            r = all_ranks[h]
            T = rot[h].to(device=dev, dtype=torch.float32)
            kd[o:o + r] = T.t() @ kd[o:o + r]
            ku[o:o + r] = T.t() @ ku[o:o + r]
        gv = torch.Generator().manual_seed(pq.HADAMARD_SEED)
        Tv = pq.block_hadamard(self.v_rank, pq.n_outlier(self.v_rank), gv).to(device=dev, dtype=torch.float32)
        kd[self.k_width:] = Tv.t() @ kd[self.k_width:]
        self.kv_down = kd.to(dt).contiguous()
        self.k_up = ku.to(dt).contiguous()
        self.v_up_by_q = torch.einsum("vu,huc->hvc", Tv.t(), self.v_up_by_q.float()).to(dt).contiguous()

    def cache_row(self) -> tuple[int, torch.dtype]:
        """Width and dtype of one cache row on this rank."""
        return (self.row.nbytes, torch.uint8) if self.quant else (self.k_width + self.v_rank, self.kv_down.dtype)

    def codes(self, hidden: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """This step's K and V codes [n, W] / [n, rv] (3.2-bit: already in the stored
        rotated basis, the rotations being folded into kv_down)."""
        return F.linear(hidden, self.kv_down).split([self.k_width, self.v_rank], dim=-1)

    def forward(self, hidden: torch.Tensor, positions: torch.Tensor, cache: torch.Tensor,
                block_table: torch.Tensor, seq_lens: torch.Tensor, max_seq_len: int,
                slot_mapping: torch.Tensor, ws=None, reduce: bool = True) -> torch.Tensor:
        """Decode step of n sequences, one new token each (hidden [n, hidden] at
        `positions`, written at `slot_mapping`, sequences `seq_lens` long including
        it); returns the o_proj output [n, hidden], all-reduced over the group
        unless `reduce` is False (then this rank's partial sum)."""
        n = hidden.shape[0]
        q = rope(F.linear(hidden, self.wq).view(n, self.num_heads, HEAD_DIM), positions, self.cos_sin_cache)
        # CUDA-graph padding rows carry slot -1 (written to the reserved null block)
        # and length 0; as attention.py:199 does, they attend to one null-block position
        seq_lens = seq_lens.clamp(min=1)
        if self.quant:
            k, v = self.codes(hidden)
            pq.pack_kv(k, v, cache, slot_mapping, self.row, self.k_ranks, self.k_head_offsets, self.k_nouts)
            attn = pq.paged_quant_decode(q, cache, block_table, seq_lens, max_seq_len, self.row, self.k_up,
                                         self.head_of_lane, self.k_tiles, self.v_up_by_q, self.cos_sin_cache,
                                         self.scale, ws=ws)
        else:
            self._write_codes(hidden, cache, slot_mapping)
            attn = paged_starkv_decode(q, cache, block_table, seq_lens, max_seq_len, self.k_up, self.k_ranks,
                                       self.k_head_offsets, self.k_width, self.v_up_by_q, self.cos_sin_cache,
                                       self.scale, ws=ws)
        return self._o_proj(attn.reshape(n, -1), reduce)

    def _write_codes(self, hidden: torch.Tensor, cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
        """bf16 / f16 cache: the step's codes go straight from the down-projection into
        their cache rows (one fused launch) at decode batch sizes, where the weight read
        is the cost (64 tokens, config-2 widths: 13.0 against 14.1 us for F.linear and
        the cache-write kernel; 24 tokens 9.3 against 13.7 us); larger batches, where
        the split-K reduction dominates (256 tokens: 33 against 15 us), and shapes the
        kernel does not take go through F.linear and the cache-write kernel."""
        if (hidden.shape[0] <= 128 and hidden.dtype == cache.dtype == self.kv_down.dtype
                and hidden.shape[1] % 512 == 0 and hidden.stride(-1) == 1 and hidden.stride(0) % 8 == 0):
            kv_down_write(hidden, self.kv_down, cache, slot_mapping)
        else:
            k, v = self.codes(hidden)
            write_kv_bf16(k, v, cache, slot_mapping)

    def _o_proj(self, attn: torch.Tensor, reduce: bool) -> torch.Tensor:
        out = F.linear(attn.to(self.wo.dtype), self.wo)
        if self.world > 1 and reduce:
            all_reduce_(out, group=self.group)
        return out

    def prefill(self, hidden: torch.Tensor, positions: torch.Tensor, prompt_lens: list[int], cache: torch.Tensor,
                slot_mapping: torch.Tensor, reduce: bool = True) -> torch.Tensor:
        """Dense prefill of whole prompts with nothing cached before them
        (attention.py:219-251): every prompt token's codes are written / packed at
        `slot_mapping`, K is lifted per head from this step's own codes with one
        bmm and rotated, V lifted by v_up, and each prompt attends causally over
        itself (the library's prefill attention kernel, in place of the reference's
        flash_attn_varlen_func). hidden [T, hidden] holds the prompts back to back
        (`prompt_lens`), `positions` their positions; returns o_proj [T, hidden]."""
        T = hidden.shape[0]
        if sum(prompt_lens) != T:
            raise ValueError("prompt_lens must cover the T tokens of hidden")
        H = self.num_kv_heads
        q = rope(F.linear(hidden, self.wq).view(T, self.num_heads, HEAD_DIM), positions, self.cos_sin_cache)
        kc, vc = self.codes(hidden)
        if self.quant:
            pq.pack_kv(kc, vc, cache, slot_mapping, self.row, self.k_ranks, self.k_head_offsets, self.k_nouts)
        else:
            write_kv_bf16(kc, vc, cache, slot_mapping)
        kp = kc[:, self.k_prefill_gather].view(T, H, self.k_max_width)
        k = rope(torch.bmm(kp.transpose(0, 1), self.k_up_T).transpose(0, 1), positions, self.cos_sin_cache)
        # V per query head: v_codes . v_up_by_q[hq] (the heads of a KV group share one
        # v_up in a checkpoint, attention.py:158-160, but nothing here relies on it)
        v = torch.einsum("tr,hrd->thd", vc, self.v_up_by_q)
        dt = q.dtype if q.dtype in (torch.bfloat16, torch.float16) else torch.bfloat16
        out = prefill_attention(q.to(dt).contiguous(), k.to(dt).contiguous(), v.to(dt).contiguous(), prompt_lens,
                                self.scale)
        return self._o_proj(out.to(q.dtype).reshape(T, -1), reduce)


class StarKVContextLayer(StarKVAttentionLayer):
    """The layer's decode step with the KV cache split by pages over `world` ranks
    (context parallel, starkv_b200.context_parallel): page p of every sequence lives on
    rank p % world. Every rank keeps the whole layer (all heads, the whole o_proj),
    so K and V codes are both divided by `world`, where head sharding must keep the V
    latent whole on every rank (checkpoint.py:140-153). Per step each rank writes the
    codes of the tokens whose page it owns, decodes all heads over its own pages into
    a partial (out, max, denominator), and the partials are all-gathered and combined
    exactly; o_proj then runs on every rank with no all-reduce."""

    def __init__(self, w: AttnWeights, cos_sin_cache: torch.Tensor, quant: bool = False, rank: int = 0,
                 world: int = 1, group=None, block_size: int = 16):
        super().__init__(w, cos_sin_cache, quant=quant)
        self.cp_rank, self.cp_world, self.cp_group, self.block_size = rank, world, group, block_size
        self.local_cos_sin = context_parallel.local_rotary_table(cos_sin_cache, rank, world, block_size)

    def forward_partial(self, hidden: torch.Tensor, positions: torch.Tensor, cache: torch.Tensor,
                        block_table: torch.Tensor, seq_lens: torch.Tensor, max_seq_len: int,
                        slot_mapping: torch.Tensor, ws=None):
        """This rank's part of a decode step. `positions` are global (the query's
        rotary); `block_table`, `seq_lens` (including the new token where this rank
        owns its page), `max_seq_len` and `slot_mapping` (-1 where another rank owns
        the page) describe this rank's local sequences. Returns (out f32 [n, H, 128]
        unnormalised, m [n, H], l [n, H])."""
        n = hidden.shape[0]
        q = rope(F.linear(hidden, self.wq).view(n, self.num_heads, HEAD_DIM), positions, self.cos_sin_cache)
        if self.quant:
            k, v = self.codes(hidden)
            pq.pack_kv(k, v, cache, slot_mapping, self.row, self.k_ranks, self.k_head_offsets, self.k_nouts)
            return pq.paged_quant_decode(q, cache, block_table, seq_lens, max_seq_len, self.row, self.k_up,
                                         self.head_of_lane, self.k_tiles, self.v_up_by_q, self.local_cos_sin,
                                         self.scale, ws=ws, context=(0, 1))
        self._write_codes(hidden, cache, slot_mapping)
        return paged_starkv_decode(q, cache, block_table, seq_lens, max_seq_len, self.k_up, self.k_ranks,
                                   self.k_head_offsets, self.k_width, self.v_up_by_q, self.local_cos_sin,
                                   self.scale, ws=ws, context=(0, 1))

    def forward(self, hidden, positions, cache, block_table, seq_lens, max_seq_len, slot_mapping, ws=None,
                reduce: bool = True) -> torch.Tensor:
        """Decode step over this rank's pages, the exchange and combination of the
        partials, and o_proj: [n, hidden], the same on every rank (`reduce` is
        accepted for the signature of StarKVAttentionLayer.forward; there is no
        partial sum to reduce)."""
        n = hidden.shape[0]
        out, m, l = self.forward_partial(hidden, positions, cache, block_table, seq_lens, max_seq_len,
                                         slot_mapping, ws)
        if self.cp_world > 1:
            attn = context_parallel.combine(out, m, l, self.cp_group, dtype=self.wo.dtype)
        else:
            attn = context_parallel.combine_local([(out, m, l)], dtype=self.wo.dtype)
        return F.linear(attn.reshape(n, -1), self.wo)
