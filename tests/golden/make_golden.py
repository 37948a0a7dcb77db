"""Generate the golden fixtures in this directory from the REFERENCE implementation.

Run from the repository root, in a container where the reference project is
importable (its path in ``$STARKV_REF``):

    STARKV_REF=/path/to/STAR-KV-Serve python tests/golden/make_golden.py

Every expected value below is produced by the reference's own code:

* packing: ``kv_quant.pack_k_ref`` / ``pack_v_ref`` (kv_quant.py:140-179), placed
  into the paged row layout with ``starkv_serve.kernels.paged_quant.QuantRow``
  (paged_quant.py:71-111), plus ``k_tables`` (paged_quant.py:114-131) and
  ``block_hadamard`` (paged_quant.py:50-68);
* bf16 decode: the PyTorch reference math of ``model.py`` (``_expand_ragged_k``
  1204-1220, ``_rope_tables`` 127-137, the no-Triton decode branch 1333-1386),
  in fp32, plus the reference paged Triton kernel ``paged_starkv_decode``
  (paged_decode.py:150-226) run by Triton's CPU interpreter in fp16;
* 3.2-bit decode: ``kv_quant.unpack_k_ref`` / ``unpack_v_ref`` followed by the same
  math, plus ``paged_quant_decode`` (paged_quant.py:357-411) under the interpreter;
* weights layout: ``starkv_serve.checkpoint._load_layer`` (checkpoint.py:106-169)
  for a small synthetic fused state dict, with and without ``kv_quant``, and
  ``load_fused_checkpoint`` (checkpoint.py:74-93) on a small fused_weights.pt
  with compressed and uncompressed layers;
* query fold: ``starkv_serve.kernels.paged_quant.fold_q`` (paged_quant.py:223-255)
  under Triton's CPU interpreter.

The fixtures are small .npz files; bf16 tensors are stored as uint16 bits.
"""

import os
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np
import torch

REF = os.environ.get("STARKV_REF", "/root/reference")
sys.path.insert(0, REF)

import kv_quant  # noqa: E402
import model as ref_model  # noqa: E402
from starkv_serve import checkpoint as ref_ckpt  # noqa: E402
from starkv_serve.kernels import paged_decode as ref_pd  # noqa: E402
from starkv_serve.kernels import paged_quant as ref_pq  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def align16(n):
    return -(-n // 16) * 16


# ---------------------------------------------------------------------------
# 1. packing known-answer vectors
# ---------------------------------------------------------------------------

def quant_rows_ref(k_codes, v_codes, ranks):
    """Reference packers -> one QuantRow per token (row padding zero)."""
    widths = [align16(r) for r in ranks]
    offsets = [sum(widths[:h]) for h in range(len(ranks))]
    W = sum(widths)
    nouts = [ref_pq.n_outlier(r) for r in ranks]
    rv = v_codes.shape[-1]
    row = ref_pq.QuantRow(W, len(ranks), rv)
    T = k_codes.shape[0]
    kq, ks = kv_quant.pack_k_ref(k_codes[None], offsets, widths, nouts)     # [1,T,W/2], [1,T,H,2]
    vq, vs = kv_quant.pack_v_ref(v_codes[None], row.v_nout)                 # [1,T,v_row], [1,T,2]
    rows = np.zeros((T, row.nbytes), np.uint8)
    rows[:, :W // 2] = kq[0].numpy()
    rows[:, row.ks_off:row.ks_off + 4 * len(ranks)] = bits(ks[0]).reshape(T, -1).view(np.uint8)
    rows[:, row.vs_off:row.vs_off + 4] = bits(vs[0]).view(np.uint8).reshape(T, 4)
    rows[:, row.vq_off:row.vq_off + row.v_bytes] = vq[0, :, :row.v_bytes].numpy()
    kd = kv_quant.unpack_k_ref(kq, ks, offsets, widths, nouts)[0].numpy()
    vd = kv_quant.unpack_v_ref(vq[..., :row.v_bytes], vs, row.v_nout, rv)[0].numpy()
    return rows, kd, vd, row


def make_pack_cases():
    g = torch.Generator().manual_seed(7)
    cases = {}
    specs = [
        ("plain", [16, 20, 37, 64], 45, False),
        ("small_ranks", [3, 4, 5, 9], 33, False),      # nout 0,0,1,1; V odd blocks
        ("wide", [128, 64, 80, 16], 160, False),
        ("pad_lanes_nonzero", [17, 33, 2, 50], 64, True),
        ("ties", [16, 32, 48, 64], 64, False),
    ]
    for name, ranks, rv, pad_nonzero in specs:
        widths = [align16(r) for r in ranks]
        W = sum(widths)
        T = 24
        k = torch.randn(T, W, generator=g) * 2.0
        v = torch.randn(T, rv, generator=g) * 3.0
        if not pad_nonzero:
            off = 0
            for r, w in zip(ranks, widths):
                k[:, off + r:off + w] = 0
                off += w
        # token 0: all zeros (EPS clamp); token 1: one huge outlier
        k[0] = 0
        v[0] = 0
        k[1, 0] = 40.0
        v[1, 0] = -55.0
        if name == "ties":
            # exact rounding ties: block amax = qmax * 2^e, x = (c + 0.5) * 2^e
            off = 0
            for r, w in zip(ranks, widths):
                no = ref_pq.n_outlier(r)
                for t in range(2, T):
                    e = 2.0 ** (t % 5 - 2)
                    if no:
                        k[t, off:off + no] = (torch.randint(-8, 7, (no,), generator=g) + 0.5) * e
                        k[t, off] = 7 * e
                    k[t, off + no:off + r] = (torch.randint(-4, 3, (r - no,), generator=g) + 0.5) * e
                    k[t, off + no] = 3 * e
                off += w
            nv = ref_pq.n_outlier(rv)
            for t in range(2, T):
                e = 2.0 ** (t % 3 - 1)
                v[t, :nv] = (torch.randint(-8, 7, (nv,), generator=g) + 0.5) * e
                v[t, 0] = 7 * e
                v[t, nv:] = (torch.randint(-4, 3, (rv - nv,), generator=g) + 0.5) * e
                v[t, nv] = -4 * e
        kb, vb = k.to(torch.bfloat16), v.to(torch.bfloat16)
        rows, kd, vd, row = quant_rows_ref(kb.float(), vb.float(), ranks)
        cases[name] = dict(ranks=np.asarray(ranks, np.int32), v_rank=np.int32(rv),
                           k_codes=bits(kb), v_codes=bits(vb), rows=rows,
                           k_deq=kd.astype(np.float32), v_deq=vd.astype(np.float32),
                           nbytes=np.int32(row.nbytes))
    return cases


# ---------------------------------------------------------------------------
# 2/3. decode cases
# ---------------------------------------------------------------------------

def rope_table(P, Hd=128):
    inv = 1.0 / (10000.0 ** (torch.arange(0, Hd, 2, dtype=torch.float32) / Hd))
    cos, sin = ref_model._rope_tables(inv, P, "cpu", torch.float32)
    return inv, torch.cat([cos[:, :Hd // 2], sin[:, :Hd // 2]], 1)


def paged_setup(g, n, seq_lens, width, bs, dtype):
    max_blocks = max(-(-s // bs) for s in seq_lens)
    nb = 1 + n * max_blocks + 3
    cache = torch.randn(nb, bs, width, generator=g).to(dtype)
    perm = torch.randperm(nb - 1, generator=g) + 1
    bt = perm[:n * max_blocks].view(n, max_blocks).to(torch.int32)
    return cache, bt


def make_bf16_case(name, H_q, H_kv, ranks, rv, seq_lens, seed):
    g = torch.Generator().manual_seed(seed)
    Hd, bs = 128, 16
    n = len(seq_lens)
    widths = [align16(r) for r in ranks]
    offsets = [sum(widths[:h]) for h in range(H_kv)]
    W = sum(widths)
    cache, bt = paged_setup(g, n, seq_lens, W + rv, bs, torch.bfloat16)
    # lanes past each head's rank hold zero codes, as the k_down rows there are zero
    for r, o, w in zip(ranks, offsets, widths):
        cache[..., o + r:o + w] = 0
    k_up = torch.zeros(W, Hd)
    for r, o in zip(ranks, offsets):
        k_up[o:o + r] = torch.randn(r, Hd, generator=g) / r ** 0.5
    k_up = k_up.to(torch.bfloat16)
    v_up_by_q = (torch.randn(H_q, rv, Hd, generator=g) / rv ** 0.5).to(torch.bfloat16)
    q = torch.randn(n, H_q, Hd, generator=g).to(torch.bfloat16)
    inv, cs = rope_table(max(seq_lens) + 5)
    cs_b = cs.to(torch.bfloat16)
    scale = Hd ** -0.5
    sl = torch.tensor(seq_lens, dtype=torch.int32)
    outs = []
    for b in range(n):
        L = seq_lens[b]
        pos = torch.arange(L)
        rows = cache[bt[b, pos // bs].long(), pos % bs].float()
        # the reference serving kernel reads cos/sin from the (bf16) rotary cache;
        # feed the math the same rounded table through inv-free tables
        o = reference_math_table(q[b].float(), rows[:, :W], rows[:, W:], k_up.float(), ranks, offsets,
                                 H_q // H_kv, v_up_by_q.float(), cs_b.float(), scale)
        outs.append(o)
    ref_out = torch.stack(outs)
    # the reference paged Triton kernel, CPU interpreter, fp16
    tri = ref_pd.paged_starkv_decode(q.half(), cache.half(), bt, sl, max(seq_lens), k_up.half(),
                                     torch.tensor(ranks, dtype=torch.int32),
                                     torch.tensor(offsets, dtype=torch.int32), W,
                                     v_up_by_q.half(), cs_b.half(), scale).float()
    return dict(query=bits(q), cache=bits(cache), block_table=bt.numpy(), seq_lens=sl.numpy(),
                k_up=bits(k_up), k_ranks=np.asarray(ranks, np.int32),
                k_head_offsets=np.asarray(offsets, np.int32), k_width=np.int32(W),
                v_up_by_q=bits(v_up_by_q), cos_sin=bits(cs_b), scale=np.float32(scale),
                out_ref_fp32=ref_out.numpy().astype(np.float32),
                out_triton_fp16=tri.numpy().astype(np.float32))


def reference_math_table(q, k_rows, v_rows, k_up, ranks, offsets, group, v_up_by_q, cs, scale):
    """model.py's decode math with the RoPE tables taken from a [cos | sin] table
    (what the serving kernels read, paged_decode.py:89-95) instead of recomputed."""
    L = k_rows.shape[0]
    half = cs.shape[1] // 2
    cos = torch.cat([cs[:L, :half], cs[:L, :half]], 1)
    sin = torch.cat([cs[:L, half:], cs[:L, half:]], 1)
    key_states = k_rows.t()[None]
    kf = ref_model._expand_ragged_k(key_states, k_up, list(zip(offsets, ranks)))
    from transformers.models.llama.modeling_llama import rotate_half
    kf = kf * cos + rotate_half(kf) * sin
    kf = kf.repeat_interleave(group, dim=1)
    w = torch.matmul(q[None, :, None, :], kf.transpose(2, 3)) * scale
    p = torch.softmax(w, dim=-1)
    pv = p.squeeze(2) @ v_rows[None]
    return torch.bmm(pv.transpose(0, 1), v_up_by_q).transpose(0, 1)[0]


def make_quant_case(name, ranks, rv, seq_lens, seed):
    g = torch.Generator().manual_seed(seed)
    Hd, bs = 128, 16
    H = len(ranks)
    n = len(seq_lens)
    widths = [align16(r) for r in ranks]
    offsets = [sum(widths[:h]) for h in range(H)]
    W = sum(widths)
    row = ref_pq.QuantRow(W, H, rv)
    max_blocks = max(-(-s // bs) for s in seq_lens)
    nb = 1 + n * max_blocks + 2
    T = nb * bs
    k = torch.randn(T, W, generator=g)
    for r, o, w in zip(ranks, offsets, widths):
        k[:, o + r:o + w] = 0
    v = torch.randn(T, rv, generator=g)
    kb, vb = k.to(torch.bfloat16), v.to(torch.bfloat16)
    rows, kd, vd, _ = quant_rows_ref(kb.float(), vb.float(), ranks)
    cache = torch.from_numpy(rows).view(nb, bs, row.nbytes)
    perm = torch.randperm(nb - 1, generator=g) + 1
    bt = perm[:n * max_blocks].view(n, max_blocks).to(torch.int32)
    k_up = torch.zeros(W, Hd)
    for r, o in zip(ranks, offsets):
        k_up[o:o + r] = torch.randn(r, Hd, generator=g) / r ** 0.5
    k_up = k_up.to(torch.bfloat16)
    v_up_by_q = (torch.randn(H, rv, Hd, generator=g) / rv ** 0.5).to(torch.bfloat16)
    q = torch.randn(n, H, Hd, generator=g).to(torch.bfloat16)
    _, cs = rope_table(max(seq_lens) + 5)
    cs_b = cs.to(torch.bfloat16)
    scale = Hd ** -0.5
    sl = torch.tensor(seq_lens, dtype=torch.int32)
    kd_t, vd_t = torch.from_numpy(kd).view(nb, bs, W), torch.from_numpy(vd).view(nb, bs, rv)
    outs = []
    for b in range(n):
        L = seq_lens[b]
        pos = torch.arange(L)
        blk = bt[b, pos // bs].long()
        outs.append(reference_math_table(q[b].float(), kd_t[blk, pos % bs], vd_t[blk, pos % bs],
                                         k_up.float(), ranks, offsets, 1, v_up_by_q.float(),
                                         cs_b.float(), scale))
    ref_out = torch.stack(outs)
    nouts, hol, tiles = ref_pq.k_tables(ranks, "cpu")
    tri = ref_pq.paged_quant_decode(q.half(), cache, bt, sl, max(seq_lens), row, k_up.half(), hol,
                                    tiles, v_up_by_q.half(), cs_b.half(), scale).float()
    return dict(query=bits(q), cache=rows.reshape(nb, bs, row.nbytes), block_table=bt.numpy(),
                seq_lens=sl.numpy(), k_up=bits(k_up), k_ranks=np.asarray(ranks, np.int32),
                v_rank=np.int32(rv), v_up_by_q=bits(v_up_by_q), cos_sin=bits(cs_b),
                scale=np.float32(scale), out_ref_fp32=ref_out.numpy().astype(np.float32),
                out_triton_fp16=tri.numpy().astype(np.float32),
                k_nouts=nouts.numpy(), head_of_lane=hol.numpy(),
                tile_head=tiles[0].numpy(), tile_nout=tiles[1].numpy(), tile_last=tiles[2].numpy())


# ---------------------------------------------------------------------------
# 4. weights layout (checkpoint._load_layer) and the block Hadamard
# ---------------------------------------------------------------------------

def make_ckpt_case():
    g = torch.Generator().manual_seed(11)
    H, Hd, hidden = 4, 128, 64
    ranks = [13, 32, 7, 40]
    rv = 50
    pre = "model.layers.0.self_attn."
    sd = {
        f"{pre}k_proj.head_ranks": torch.tensor(ranks, dtype=torch.int32),
        f"{pre}k_proj.VS.weight": torch.randn(sum(ranks), hidden, generator=g),
        f"{pre}v_proj.VS.weight": torch.randn(rv, hidden, generator=g),
        f"{pre}v_proj.U.weight": torch.randn(H * Hd, rv, generator=g),
    }
    u = torch.zeros(H * Hd, sum(ranks))
    col = 0
    for h, r in enumerate(ranks):
        u[h * Hd:(h + 1) * Hd, col:col + r] = torch.randn(Hd, r, generator=g)
        col += r
    sd[f"{pre}k_proj.U.weight"] = u
    out = {f"in_{k.split('self_attn.')[1]}": v.numpy() for k, v in sd.items()}
    for quant in (False, True):
        lw = ref_ckpt._load_layer(sd, pre, 0, H, Hd, torch.float32, quant)
        tag = "q" if quant else "b"
        out[f"{tag}_k_down"] = lw.k_down.numpy()
        out[f"{tag}_k_up"] = lw.k_up.numpy()
        out[f"{tag}_v_down"] = lw.v_down.numpy()
        out[f"{tag}_v_up"] = lw.v_up.numpy()
        out[f"{tag}_k_head_offsets"] = lw.k_head_offsets.numpy()
        out[f"{tag}_k_head_widths"] = lw.k_head_widths.numpy()
        out[f"{tag}_meta"] = np.asarray([lw.k_width, lw.k_max_rank, lw.v_rank, lw.v_rank_real,
                                         lw.cache_bytes(2)], np.int64)
    hs = {}
    for r in (1, 2, 5, 16, 37, 64, 100):
        gen = torch.Generator().manual_seed(ref_pq.HADAMARD_SEED)
        hs[f"T{r}"] = ref_pq.block_hadamard(r, ref_pq.n_outlier(r), gen).numpy()
    out.update(hs)
    return out


def make_fold_case():
    g = torch.Generator().manual_seed(13)
    ranks = [16, 20, 37, 64, 5]
    widths = [align16(r) for r in ranks]
    offsets = [sum(widths[:h]) for h in range(len(ranks))]
    W = sum(widths)
    H, n = len(ranks), 3
    _, hol, _ = ref_pq.k_tables(ranks, "cpu")
    q = torch.randn(n, H, 128, generator=g).to(torch.bfloat16)
    k_up = torch.zeros(W, 128)
    for r, o in zip(ranks, offsets):
        k_up[o:o + r] = torch.randn(r, 128, generator=g) / r ** 0.5
    k_up = k_up.to(torch.bfloat16)
    scale = 128 ** -0.5
    ab = ref_pq.fold_q(q.float(), k_up.float(), hol, scale)        # fp32 inputs (bf16 values)
    return dict(query=bits(q), k_up=bits(k_up), head_of_lane=hol.numpy(), scale=np.float32(scale),
                ab_f16=ab.numpy())


def main():
    for name, case in make_pack_cases().items():
        np.savez_compressed(os.path.join(OUT, f"pack_{name}.npz"), **case)
    np.savez_compressed(os.path.join(OUT, "decode_bf16_mha.npz"),
                        **make_bf16_case("mha", 4, 4, [16, 32, 48, 64], 96, [1, 17, 40], 1))
    np.savez_compressed(os.path.join(OUT, "decode_bf16_ragged.npz"),
                        **make_bf16_case("ragged", 4, 4, [5, 16, 33, 64], 48, [15, 16, 64, 70], 2))
    np.savez_compressed(os.path.join(OUT, "decode_bf16_gqa.npz"),
                        **make_bf16_case("gqa", 8, 4, [16, 20, 64, 40], 64, [3, 33], 3))
    np.savez_compressed(os.path.join(OUT, "decode_quant.npz"),
                        **make_quant_case("quant", [16, 20, 37, 64], 45, [1, 17, 40], 4))
    np.savez_compressed(os.path.join(OUT, "decode_quant_b.npz"),
                        **make_quant_case("quant_b", [64, 48, 5, 128], 160, [16, 31, 130], 5))
    np.savez_compressed(os.path.join(OUT, "checkpoint_layer.npz"), **make_ckpt_case())
    np.savez_compressed(os.path.join(OUT, "fold_q.npz"), **make_fold_case())
    print("golden fixtures written to", OUT)


if __name__ == "__main__":
    main()
