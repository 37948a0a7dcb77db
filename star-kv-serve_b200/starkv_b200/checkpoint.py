"""The fused STAR-KV checkpoint (``fused_weights.pt``) and its serving layout.

Restates the reference loader (starkv_serve/checkpoint.py:74-169) so this
library's layer and model run from the same file the reference serves. The
format is an interface and is kept as the reference writes it (train.py's
fuse_and_prune), per compressed layer ``li`` under
``model.layers.{li}.self_attn.``::

    k_proj.head_ranks  [H] int32            real K rank of each KV head
    k_proj.VS.weight   [sum(ranks), hidden] K down rows, head after head
    k_proj.U.weight    [H*Hd, sum(ranks)]   K up, block-diagonal by head
    v_proj.VS.weight   [rv, hidden]         V down (one latent for all heads)
    v_proj.U.weight    [H*Hd, rv]           V up

Serving layout (checkpoint.py:106-169): each head's K codes at its own width,
the rank rounded up to K_ALIGN, heads side by side (``k_head_offsets``), rows
between a head's rank and its width zero; ``k_up`` rank-major [k_width, Hd]. V
padded with zero rows / columns to a multiple of V_ALIGN for bf16 caches. With
``kv_quant`` the K and V factors are first rotated by the block Hadamard of
paged_quant.py:50-68 (seed HADAMARD_SEED, a fresh generator per projection),
``VS <- T^T VS`` and ``U <- U T`` in float64 (checkpoint.py:96-103), so the codes
come out in the rotated basis the 3.2-bit cache stores and ``U VS`` is unchanged;
V is then not padded. A layer without ``k_proj.head_ranks`` is left full-rank.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .kernels.paged_quant import HADAMARD_SEED, QuantRow, block_hadamard, n_outlier

K_ALIGN = 16      # K code width per head: rank rounded up to this (checkpoint.py:30)
V_ALIGN = 16      # V code width of bf16 caches rounded up to this (checkpoint.py:26)


def _ceil_to(n: int, m: int) -> int:
    return (int(n) + m - 1) // m * m


@dataclass
class StarKVLayerWeights:
    """One compressed layer in the serving layout (checkpoint.py:37-63)."""
    layer_idx: int
    k_head_ranks: torch.Tensor     # [H] int32
    k_head_widths: torch.Tensor    # [H] int32, rank rounded up to K_ALIGN
    k_head_offsets: torch.Tensor   # [H] int32, first K lane of each head
    k_width: int                   # sum of the widths
    k_max_rank: int                # widest head width (prefill padding)
    k_down: torch.Tensor           # [k_width, hidden]
    k_up: torch.Tensor             # [k_width, Hd]
    v_rank: int                    # stored V width (padded for bf16 caches)
    v_rank_real: int               # V rank in the checkpoint
    v_down: torch.Tensor           # [v_rank, hidden]
    v_up: torch.Tensor             # [H*Hd, v_rank]
    kv_quant: bool = False         # factors rotated for the 3.2-bit cache

    @property
    def cache_width(self) -> int:
        return self.k_width + self.v_rank

    def cache_bytes(self, elem_size: int) -> int:
        """Cache bytes per token of this layer (3.2-bit: one QuantRow)."""
        if self.kv_quant:
            return QuantRow(self.k_width, self.k_head_ranks.numel(), self.v_rank).nbytes
        return self.cache_width * elem_size


@dataclass
class StarKVCheckpoint:
    layers: dict            # layer index -> StarKVLayerWeights
    skip_layers: tuple      # layers left full-rank

    def is_compressed(self, layer_idx: int) -> bool:
        return layer_idx in self.layers


def load_fused_checkpoint(path, num_layers: int, num_kv_heads: int, head_dim: int,
                          dtype: torch.dtype = torch.float16, kv_quant: bool = False) -> StarKVCheckpoint:
    """Read ``fused_weights.pt`` (checkpoint.py:74-93): every layer holding
    ``k_proj.head_ranks`` is loaded into the serving layout, the others are
    full-rank. ``path`` may also be an already-loaded state dict."""
    sd = path if isinstance(path, dict) else torch.load(path, map_location="cpu", mmap=True, weights_only=True)
    layers = {}
    for li in range(num_layers):
        pre = f"model.layers.{li}.self_attn."
        if f"{pre}k_proj.head_ranks" in sd:
            layers[li] = load_layer(sd, pre, li, num_kv_heads, head_dim, dtype, kv_quant)
        elif f"{pre}k_proj.Sigma_blocks.0.diag" in sd:
            raise ValueError(f"{path if not isinstance(path, dict) else 'state dict'}: layer {li} holds the "
                             "unfused U/Sigma/V factors; serving needs the fused format (fuse_and_prune)")
    if not layers:
        raise ValueError("no fused STAR-KV layer in the checkpoint")
    return StarKVCheckpoint(layers=layers, skip_layers=tuple(i for i in range(num_layers) if i not in layers))


def rotate_blocks(vs: torch.Tensor, u: torch.Tensor, ranks: list[int], generator: torch.Generator) -> None:
    """In place, per block of `ranks` rows: VS <- T^T VS, U <- U T with T the block
    Hadamard of that rank (drawn from `generator` in block order), in float64 and
    rounded back to float32 (checkpoint.py:96-103)."""
    c = 0
    for r in ranks:
        T = block_hadamard(r, n_outlier(r), generator)
        vs[c:c + r] = (T.T @ vs[c:c + r].double()).float()
        u[:, c:c + r] = (u[:, c:c + r].double() @ T).float()
        c += r


def load_layer(sd: dict, pre: str, li: int, H: int, Hd: int, dtype: torch.dtype,
               kv_quant: bool) -> StarKVLayerWeights:
    """One layer of the state dict in the serving layout (checkpoint.py:106-169)."""
    ranks = [int(x) for x in sd[f"{pre}k_proj.head_ranks"].tolist()]
    if len(ranks) != H:
        raise ValueError(f"layer {li}: {len(ranks)} K head ranks for {H} KV heads")
    R = sum(ranks)
    kvs = sd[f"{pre}k_proj.VS.weight"].float()
    ku = sd[f"{pre}k_proj.U.weight"].float()
    if tuple(kvs.shape[:1]) != (R,) or tuple(ku.shape) != (H * Hd, R):
        raise ValueError(f"layer {li}: k_proj VS {tuple(kvs.shape)} / U {tuple(ku.shape)} do not fit ranks "
                         f"summing to {R} with H={H}, Hd={Hd}")
    if kv_quant:   # the loaded tensors may be memory-mapped: rotate copies
        kvs, ku = kvs.clone(), ku.clone()
        rotate_blocks(kvs, ku, ranks, torch.Generator().manual_seed(HADAMARD_SEED))
    hidden = kvs.shape[1]
    widths = [_ceil_to(r, K_ALIGN) for r in ranks]
    offsets = [sum(widths[:h]) for h in range(H)]
    W = sum(widths)
    k_down = kvs.new_zeros(W, hidden)
    k_up = kvs.new_zeros(W, Hd)
    src = 0
    for h, (r, o) in enumerate(zip(ranks, offsets)):
        k_down[o:o + r] = kvs[src:src + r]
        k_up[o:o + r] = ku[h * Hd:(h + 1) * Hd, src:src + r].T   # head h's diagonal block, rank-major
        src += r

    vvs = sd[f"{pre}v_proj.VS.weight"].float()
    vu = sd[f"{pre}v_proj.U.weight"].float()
    rv = vvs.shape[0]
    if tuple(vu.shape) != (H * Hd, rv):
        raise ValueError(f"layer {li}: v_proj VS {tuple(vvs.shape)} / U {tuple(vu.shape)}")
    if kv_quant:
        vvs, vu = vvs.clone(), vu.clone()
        rotate_blocks(vvs, vu, [rv], torch.Generator().manual_seed(HADAMARD_SEED))
    rv_store = rv if kv_quant else _ceil_to(rv, V_ALIGN)
    v_down = vvs.new_zeros(rv_store, hidden)
    v_down[:rv] = vvs
    v_up = vu.new_zeros(H * Hd, rv_store)
    v_up[:, :rv] = vu
    return StarKVLayerWeights(
        layer_idx=li, k_head_ranks=torch.tensor(ranks, dtype=torch.int32),
        k_head_widths=torch.tensor(widths, dtype=torch.int32), k_head_offsets=torch.tensor(offsets, dtype=torch.int32),
        k_width=W, k_max_rank=max(widths), k_down=k_down.to(dtype), k_up=k_up.to(dtype), v_rank=rv_store,
        v_rank_real=rv, v_down=v_down.to(dtype), v_up=v_up.to(dtype), kv_quant=kv_quant)


def synthetic_state_dict(layer_ranks: dict, hidden: int, num_kv_heads: int, head_dim: int = 128, seed: int = 0,
                         dtype: torch.dtype = torch.bfloat16) -> dict:
    """A random-init fused state dict in the format above: ``layer_ranks`` maps each
    compressed layer to (K ranks per head, V rank). Factors ~ N(0, 1/fan-in): VS
    rows std hidden^-1/2, U columns std rank^-1/2 (per head for K, block-diagonal)."""
    g = torch.Generator().manual_seed(seed)
    H, Hd = num_kv_heads, head_dim
    sd = {}
    for li in sorted(layer_ranks):
        ranks, rv = layer_ranks[li]
        pre = f"model.layers.{li}.self_attn."
        R = sum(ranks)
        ku = torch.zeros(H * Hd, R)
        c = 0
        for h, r in enumerate(ranks):
            ku[h * Hd:(h + 1) * Hd, c:c + r] = torch.randn(Hd, r, generator=g) * r ** -0.5
            c += r
        sd[f"{pre}k_proj.head_ranks"] = torch.tensor(ranks, dtype=torch.int32)
        sd[f"{pre}k_proj.VS.weight"] = (torch.randn(R, hidden, generator=g) * hidden ** -0.5).to(dtype)
        sd[f"{pre}k_proj.U.weight"] = ku.to(dtype)
        sd[f"{pre}v_proj.VS.weight"] = (torch.randn(rv, hidden, generator=g) * hidden ** -0.5).to(dtype)
        sd[f"{pre}v_proj.U.weight"] = (torch.randn(H * Hd, rv, generator=g) * rv ** -0.5).to(dtype)
    return sd


def write_synthetic_checkpoint(path, layer_ranks: dict, hidden: int, num_kv_heads: int, head_dim: int = 128,
                               seed: int = 0, dtype: torch.dtype = torch.bfloat16) -> None:
    """Write synthetic_state_dict(...) as a ``fused_weights.pt``."""
    torch.save(synthetic_state_dict(layer_ranks, hidden, num_kv_heads, head_dim, seed, dtype), path)
