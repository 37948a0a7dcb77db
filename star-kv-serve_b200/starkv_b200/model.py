"""Decode step of a whole STAR-KV Llama (StarKVLlamaForCausalLM, model.py:78-106):
embedding, per layer RMSNorm -> attention -> residual -> RMSNorm -> SiLU MLP ->
residual, final RMSNorm, LM head logits.

Compressed layers run starkv_b200.layer.StarKVAttentionLayer (this library's paged
low-rank decode); the layers the checkpoint left full-rank run stock attention
over a paged bf16 K/V cache (vLLM's paged-attention and cache-write ops, as the
reference's stock LlamaAttention does). Tensor parallel over `world` ranks in the
Megatron layout the reference leaves at TP=1 (model.py:32-33): attention heads and
the MLP's intermediate columns are split, o_proj and down_proj are row-parallel
and all-reduced; embedding, norms and LM head are replicated. Weights are
seeded random-init of the configured geometry; the compressed layers' K/V factors
can come from a fused_weights.pt instead (starkv_b200.checkpoint), which then
also decides which layers are compressed.

With attn_parallel="context" the compressed layers split their KV cache by pages
instead of heads (starkv_b200.layer.StarKVContextLayer): every rank holds all heads
and 1/world of every sequence's pages, so the V latent, which head sharding keeps
whole on every rank, is divided too. The full-rank layers and the MLP stay
tensor parallel.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch
import torch.nn.functional as F

from . import sharding
from .collectives import all_reduce_
from .layer import HEAD_DIM, AttnWeights, StarKVAttentionLayer, StarKVContextLayer, rope
from .workload import rope_cos_sin


@dataclass
class ModelConfig:
    hidden: int = 4096
    heads: int = 32
    ffn: int = 11008
    vocab: int = 32000
    layers: int = 32
    full_layers: tuple = (0, 1, 2, 31)   # left full-rank by the checkpoint
    rms_eps: float = 1e-5
    max_pos: int = 32768
    seed: int = 0
    k_rank_choices: tuple = (16, 32, 48)         # comp-ratio 0.75: W ~ 1000 for 32 heads
    k_rank_probs: tuple = (0.35, 0.45, 0.20)
    v_rank_choices: tuple = (32, 64)             # rv ~ 1280
    v_rank_probs: tuple = (0.75, 0.25)
    ranks: dict = field(default_factory=dict)    # layer -> (k ranks, v rank), filled on first use

    def layer_ranks(self, i: int) -> tuple[list[int], int]:
        if i not in self.ranks:
            rng = np.random.default_rng(self.seed * 1000 + i)
            k = rng.choice(self.k_rank_choices, size=self.heads, p=self.k_rank_probs)
            v = rng.choice(self.v_rank_choices, size=self.heads, p=self.v_rank_probs)
            self.ranks[i] = ([int(x) for x in k], int(v.sum()))
        return self.ranks[i]


def checkpoint_layer_ranks(cfg: ModelConfig) -> dict:
    """(K ranks, V rank) of every compressed layer of `cfg`, for
    starkv_b200.checkpoint.write_synthetic_checkpoint."""
    return {i: cfg.layer_ranks(i) for i in range(cfg.layers) if i not in cfg.full_layers}


def _rnd(shape, std, g, device, dtype=torch.bfloat16):
    return (torch.randn(*shape, generator=g, device=device) * std).to(dtype)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype) * w


class StockAttentionLayer:
    """Full-rank attention over a paged bf16 K/V cache in vLLM's layout
    (key [blocks, heads, 128 / 8, 16, 8], value [blocks, heads, 128, 16]); heads
    split evenly over the group."""

    def __init__(self, wq, wk, wv, wo, cos_sin_cache, rank=0, world=1, group=None):
        H = wq.shape[0] // HEAD_DIM
        hidden = wq.shape[1]
        if H % world:
            raise ValueError(f"{H} heads do not split over {world} ranks")
        hl = H // world
        sl = slice(rank * hl * HEAD_DIM, (rank + 1) * hl * HEAD_DIM)
        self.wqkv = torch.cat([wq[sl], wk[sl], wv[sl]]).contiguous()
        self.wo = wo[:, sl].contiguous()
        self.heads, self.hidden, self.world, self.group = hl, hidden, world, group
        self.cos_sin_cache = cos_sin_cache
        self.scale = HEAD_DIM ** -0.5
        self.one = torch.ones((), dtype=torch.float32, device=wq.device)

    def cache_shapes(self, num_blocks: int):
        return (num_blocks, self.heads, HEAD_DIM // 8, 16, 8), (num_blocks, self.heads, HEAD_DIM, 16)

    def forward(self, hidden, positions, kcache, vcache, block_table, seq_lens, max_seq_len, slot_mapping,
                reduce=True):
        """Decode step: q / k / v projections, rotary, cache write, paged attention,
        o_proj (all-reduced over the group unless `reduce` is False)."""
        from vllm import _custom_ops as ops
        n = hidden.shape[0]
        q, k, v = F.linear(hidden, self.wqkv).view(n, 3, self.heads, HEAD_DIM).unbind(1)
        q = rope(q, positions, self.cos_sin_cache).contiguous()
        k = rope(k, positions, self.cos_sin_cache).contiguous()
        ops.reshape_and_cache(k, v.contiguous(), kcache, vcache, slot_mapping, "auto", self.one, self.one)
        out = torch.empty_like(q)
        parts = -(-max_seq_len // 512)
        exp_sums = torch.empty(n, self.heads, parts, dtype=torch.float32, device=q.device)
        max_logits = torch.empty_like(exp_sums)
        tmp = torch.empty(n, self.heads, parts, HEAD_DIM, dtype=q.dtype, device=q.device)
        ops.paged_attention_v2(out, exp_sums, max_logits, tmp, q, kcache, vcache, self.heads, self.scale,
                               block_table, seq_lens, 16, max_seq_len, None, "auto", self.one, self.one)
        o = F.linear(out.view(n, -1), self.wo)
        if self.world > 1 and reduce:
            all_reduce_(o, group=self.group)
        return o


class StarKVModel:
    """The model on one rank of a tensor-parallel group (world 1: whole)."""

    def __init__(self, cfg: ModelConfig, device, quant: bool = False, rank: int = 0, world: int = 1, group=None,
                 dtype=torch.bfloat16, attn_parallel: str = "heads", checkpoint=None):
        """`checkpoint`: a fused_weights.pt (path, state dict or loaded
        starkv_b200.checkpoint.StarKVCheckpoint) whose compressed layers' K/V factors
        the model serves; the layers it leaves out are full-rank. Without one, every
        layer outside cfg.full_layers gets seeded random factors. The other weights
        (embedding, q/o projections, MLP, norms, LM head) are seeded random-init
        either way: the checkpoint holds only the K/V factors."""
        if attn_parallel not in ("heads", "context"):
            raise ValueError(f"attn_parallel must be 'heads' or 'context', not {attn_parallel!r}")
        ckpt = None
        if checkpoint is not None:
            import dataclasses
            from .checkpoint import StarKVCheckpoint, load_fused_checkpoint
            ckpt = checkpoint if isinstance(checkpoint, StarKVCheckpoint) else load_fused_checkpoint(
                checkpoint, cfg.layers, cfg.heads, HEAD_DIM, dtype=torch.float32, kv_quant=quant)
            if any(lw.kv_quant != quant for lw in ckpt.layers.values()):
                raise ValueError("checkpoint loaded with kv_quant != the model's quant")
            cfg = dataclasses.replace(cfg, full_layers=tuple(ckpt.skip_layers))
        self.cfg, self.quant, self.rank, self.world, self.group = cfg, quant, rank, world, group
        self.attn_parallel = attn_parallel
        self.device = torch.device(device)
        d, H = cfg.hidden, cfg.heads
        g = torch.Generator(device=self.device).manual_seed(cfg.seed)
        self.embed = _rnd((cfg.vocab, d), 1.0, g, self.device, dtype)
        self.lm_head = _rnd((cfg.vocab, d), d ** -0.5, g, self.device, dtype)
        self.final_norm = torch.ones(d, device=self.device, dtype=dtype)
        self.cos_sin_cache = rope_cos_sin(cfg.max_pos, self.device)
        if cfg.ffn % world:
            raise ValueError(f"ffn {cfg.ffn} does not split over {world} ranks")
        fl = cfg.ffn // world
        self.layers = []
        for i in range(cfg.layers):
            gl = torch.Generator(device=self.device).manual_seed(cfg.seed * 1000 + i + 1)
            norms = (torch.ones(d, device=self.device, dtype=dtype), torch.ones(d, device=self.device, dtype=dtype))
            wq = _rnd((H * HEAD_DIM, d), d ** -0.5, gl, self.device, dtype)
            wo = _rnd((d, H * HEAD_DIM), (H * HEAD_DIM) ** -0.5, gl, self.device, dtype)
            if i in cfg.full_layers:
                wk = _rnd((H * HEAD_DIM, d), d ** -0.5, gl, self.device, dtype)
                wv = _rnd((H * HEAD_DIM, d), d ** -0.5, gl, self.device, dtype)
                attn = StockAttentionLayer(wq, wk, wv, wo, self.cos_sin_cache, rank, world, group)
                del wk, wv
            elif ckpt is not None:
                w = AttnWeights.from_checkpoint(ckpt.layers[i], wq, wo, H, device=self.device, dtype=dtype)
                attn = (StarKVContextLayer if attn_parallel == "context" else StarKVAttentionLayer)(
                    w, self.cos_sin_cache, quant=quant, rank=rank, world=world, group=group)
                del w
            else:
                ranks, rv = cfg.layer_ranks(i)
                offs = sharding.k_offsets(ranks)
                W = sum(sharding.align16(r) for r in ranks)
                kv_down = _rnd((W + rv, d), d ** -0.5, gl, self.device, dtype)
                k_up = torch.zeros(W, HEAD_DIM, device=self.device, dtype=dtype)
                for r, o in zip(ranks, offs):
                    kv_down[o + r:o + sharding.align16(r)] = 0
                    k_up[o:o + r] = _rnd((r, HEAD_DIM), r ** -0.5, gl, self.device, dtype)
                v_up_by_q = _rnd((H, rv, HEAD_DIM), rv ** -0.5, gl, self.device, dtype)
                w = AttnWeights(wq=wq, kv_down=kv_down, wo=wo, k_up=k_up, v_up_by_q=v_up_by_q, k_ranks=ranks,
                                v_rank=rv, num_heads=H, num_kv_heads=H)
                if attn_parallel == "context":
                    attn = StarKVContextLayer(w, self.cos_sin_cache, quant=quant, rank=rank, world=world,
                                              group=group)
                else:
                    attn = StarKVAttentionLayer(w, self.cos_sin_cache, quant=quant, rank=rank, world=world,
                                                group=group)
                del w, kv_down, k_up, v_up_by_q
            gate_up = _rnd((2 * cfg.ffn, d), d ** -0.5, gl, self.device, dtype)
            down = _rnd((d, cfg.ffn), cfg.ffn ** -0.5, gl, self.device, dtype)
            # column-parallel gate / up rows and row-parallel down columns of this rank
            cols = slice(rank * fl, (rank + 1) * fl)
            gu = torch.cat([gate_up[:cfg.ffn][cols], gate_up[cfg.ffn:][cols]]).contiguous()
            self.layers.append(dict(norms=norms, attn=attn, gate_up=gu, down=down[:, cols].contiguous(),
                                    full=i in cfg.full_layers))
            del wq, wo, gate_up, down
        torch.cuda.empty_cache()

    def allocate_caches(self, num_blocks: int, compressed_blocks: int | None = None) -> list:
        """One paged cache per layer (16-token blocks): STAR-KV code rows
        (`compressed_blocks` of them, default `num_blocks`: with attn_parallel
        "context" a rank holds only its pages of every sequence), or the stock
        (key, value) pair."""
        caches = []
        for ly in self.layers:
            a = ly["attn"]
            if ly["full"]:
                ks, vs = a.cache_shapes(num_blocks)
                caches.append((torch.zeros(ks, dtype=torch.bfloat16, device=self.device),
                               torch.zeros(vs, dtype=torch.bfloat16, device=self.device)))
            else:
                width, dt = a.cache_row()
                nb = num_blocks if compressed_blocks is None else compressed_blocks
                caches.append(torch.zeros(nb, 16, width, dtype=dt, device=self.device))
        return caches

    def kv_bytes_per_token(self) -> int:
        """Cache bytes this rank holds per token of context, over all layers."""
        tot = 0.0
        for ly in self.layers:
            a = ly["attn"]
            if ly["full"]:
                tot += 2 * a.heads * HEAD_DIM * 2
            else:
                width, dt = a.cache_row()
                share = 1.0 / self.world if self.attn_parallel == "context" else 1.0
                tot += width * torch.empty((), dtype=dt).element_size() * share
        return int(tot)

    def _all_reduce(self, x):
        if self.world > 1:
            all_reduce_(x, group=self.group)
        return x

    def decode_step(self, tokens, positions, caches, block_table, seq_lens, max_seq_len, slot_mapping, ws=None,
                    local=None):
        """One decode step of n sequences: token ids [n] at `positions` (written at
        `slot_mapping`, sequences `seq_lens` long including them); returns the
        logits [n, vocab] (f32), the same on every rank. With attn_parallel
        "context", `local` = (block_table, seq_lens, max_seq_len, slot_mapping) of
        this rank's pages (starkv_b200.context_parallel.local_len / local_index) for
        the compressed layers; the other arguments serve the full-rank layers."""
        if self.attn_parallel == "context" and local is None:
            raise ValueError("attn_parallel='context' needs the local page metadata (`local`)")
        cmeta = local if local is not None else (block_table, seq_lens, max_seq_len, slot_mapping)
        eps = self.cfg.rms_eps
        x = self.embed[tokens]
        for ly, cache in zip(self.layers, caches):
            h = rms_norm(x, ly["norms"][0], eps)
            if ly["full"]:
                a = ly["attn"].forward(h, positions, cache[0], cache[1], block_table, seq_lens, max_seq_len,
                                       slot_mapping)
            else:
                a = ly["attn"].forward(h, positions, cache, *cmeta, ws=ws)
            x = x + a
            h = rms_norm(x, ly["norms"][1], eps)
            g, u = F.linear(h, ly["gate_up"]).chunk(2, dim=-1)
            x = x + self._all_reduce(F.linear(F.silu(g) * u, ly["down"]))
        return F.linear(rms_norm(x, self.final_norm, eps), self.lm_head).float()
