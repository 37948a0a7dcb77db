"""CPU oracle for STAR-KV paged low-rank decode attention.

TEST INFRASTRUCTURE ONLY. This module is the checker for the CUDA path: only
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / reference arm
of ``bench.py`` may import it. The product path (``starkv_b200``) never calls it
and fails loudly when its CUDA library is missing.

It restates, in numpy, the reference's algorithm for the decode hot path. Every
function cites the reference file:line it follows (paths relative to the
STAR-KV-Serve project root).

Pinning: ``tests/golden/make_golden.py`` imports the reference itself
(``kv_quant.pack_k_ref`` / ``pack_v_ref`` / ``unpack_*_ref``, ``model._expand_ragged_k``,
``model._rope_tables``, ``paged_quant.QuantRow`` / ``k_tables`` / ``block_hadamard``,
``checkpoint._load_layer``) and commits its outputs under ``tests/golden/``;
``tests/test_oracle_golden.py`` checks this module against those fixtures
byte-for-byte (packing) and to fp32 rounding (decode).

The only third-party arithmetic is torch's CPU random generator, used by
``block_hadamard`` exactly as the reference does (paged_quant.py:66): the sign
flips are defined by that generator's stream, so the oracle draws them the
same way.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

OUTLIER_RATIO = 0.2          # paged_quant.py:39
HADAMARD_SEED = 1234         # paged_quant.py:40
EPS = np.float32(1e-5)       # paged_quant.py:41
HEAD_DIM = 128               # paged_quant.py:43
K_ALIGN = 16                 # checkpoint.py:30
V_ALIGN = 16                 # checkpoint.py:26


# ---------------------------------------------------------------------------
# bf16 helpers (numpy has no bfloat16): values travel as uint16 bit patterns.
# ---------------------------------------------------------------------------

def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16, as torch's ``.to(torch.bfloat16)``."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FC0
    return r


def round_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


# ---------------------------------------------------------------------------
# Format: quantizer, row layout, tile tables (kv_quant.py, paged_quant.py)
# ---------------------------------------------------------------------------

def n_outlier(rank: int) -> int:
    """paged_quant.py:46-47 / kv_quant.py:76-77."""
    return int(OUTLIER_RATIO * rank)


def align_up(n: int, m: int) -> int:
    return -(-int(n) // m) * m


def block_hadamard(rank: int, n_out: int, generator) -> np.ndarray:
    """paged_quant.py:50-68 (== kv_quant.py:84-103): rank x rank orthonormal,
    diag(H_outlier, H_inlier); each block a Sylvester Hadamard on its largest
    power-of-two leading part with random row signs, identity on the rest."""
    import torch  # RNG stream only

    T = np.eye(rank, dtype=np.float64)
    for a, n in ((0, n_out), (n_out, rank - n_out)):
        if n <= 1:
            continue
        m = 1 << (n.bit_length() - 1)
        H = np.ones((1, 1))
        while H.shape[0] < m:
            H = np.block([[H, H], [H, -H]])
        draws = torch.rand(m, generator=generator).numpy()
        signs = np.where(draws < 0.5, -1.0, 1.0)
        T[a:a + m, a:a + m] = signs[:, None] * H / math.sqrt(m)
    return T


def quantize_block(x: np.ndarray, bits: int) -> tuple[np.ndarray, np.ndarray]:
    """kv_quant.py:111-121 (`_q`), the definition of the format.

    x [..., c] float32. Returns (codes + 8 as uint8, fp32 scale [...]).
    amax clamped to EPS; scale = amax / qmax by IEEE division; codes =
    round-half-even(x / scale) by IEEE division, clamped to [-(qmax+1), qmax].
    """
    x = np.asarray(x, dtype=np.float32)
    qmax = np.float32(2 ** (bits - 1) - 1)
    amax = np.maximum(np.abs(x).max(axis=-1), EPS).astype(np.float32)
    s = (amax / qmax).astype(np.float32)              # numpy fp32 '/' is IEEE div_rn
    q = np.rint(x / s[..., None]).astype(np.float32)  # np.rint: half to even
    q = np.clip(q, -(qmax + 1), qmax)
    return (q + 8).astype(np.uint8), s


@dataclass(frozen=True)
class QuantRow:
    """paged_quant.py:71-111: byte layout of one token of a 4-bit layer."""
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
        return align_up(self.vq_off + self.v_bytes, 16)


def k_layout(ranks):
    """checkpoint.py:125-127: per-head width align16(rank), offsets, total width."""
    widths = [align_up(r, K_ALIGN) for r in ranks]
    offsets = [sum(widths[:h]) for h in range(len(ranks))]
    return widths, offsets, sum(widths)


def k_tables(ranks):
    """paged_quant.py:114-131: (outlier lanes per head, head of every lane,
    per-16-lane-tile (head, outlier lanes in tile, is-last-tile-of-head))."""
    nouts = [n_outlier(r) for r in ranks]
    lanes, head, t_out, last = [], [], [], []
    for h, (r, no) in enumerate(zip(ranks, nouts)):
        tiles = -(-r // 16)
        lanes += [h] * (16 * tiles)
        for j in range(tiles):
            head.append(h)
            t_out.append(max(0, min(16, no - 16 * j)))
            last.append(int(j == tiles - 1))
    i32 = lambda v: np.asarray(v, dtype=np.int32)  # noqa: E731
    return i32(nouts), i32(lanes), (i32(head), i32(t_out), i32(last))


def pack_rows(k_codes: np.ndarray, v_codes: np.ndarray, row: QuantRow, ranks) -> np.ndarray:
    """Quantize tokens into QuantRow bytes.

    k_codes [T, W], v_codes [T, rv] float32 (the model-dtype codes upcast).
    Follows paged_quant.py:146-202 (`_pack_k`, `_pack_v`) whose bytes equal
    kv_quant.pack_k_ref / pack_v_ref (kv_quant.py:140-179):
      K: per head, lanes [0, nout) 4-bit, [nout, align16(rank)) 3-bit; nibble
         of lane 2k in the low half of byte k; scales (s_out or 1.0 when nout
         == 0, s_in) as bf16 at ks_off + 4h.
      V: outlier channels packed first (bytes [0, nbo)), then inliers, an odd
         block ending in pad nibble 8; scales at vs_off.
    Bytes past vq_off + v_bytes (row padding) are left zero.
    """
    T = k_codes.shape[0]
    widths, offsets, W = k_layout(ranks)
    assert k_codes.shape[1] == W == row.k_width
    out = np.zeros((T, row.nbytes), dtype=np.uint8)
    nib = np.full((T, W), 8, dtype=np.uint8)
    for h, (r, off, w) in enumerate(zip(ranks, offsets, widths)):
        no = n_outlier(r)
        s_out = np.ones(T, dtype=np.float32)
        if no:
            nib[:, off:off + no], s_out = quantize_block(k_codes[:, off:off + no], 4)
        nib[:, off + no:off + w], s_in = quantize_block(k_codes[:, off + no:off + w], 3)
        sc = np.stack([f32_to_bf16_bits(s_out), f32_to_bf16_bits(s_in)], -1)   # [T, 2]
        out[:, row.ks_off + 4 * h:row.ks_off + 4 * h + 4] = sc.view(np.uint8).reshape(T, 4)
    out[:, :W // 2] = nib[:, 0::2] | (nib[:, 1::2] << 4)

    R, no = row.v_rank, row.v_nout
    s_out = np.ones(T, dtype=np.float32)
    n_o = np.zeros((T, 0), dtype=np.uint8)
    if no:
        n_o, s_out = quantize_block(v_codes[:, :no], 4)
    n_i, s_in = quantize_block(v_codes[:, no:R], 3)

    def nibble_pack(n):
        if n.shape[1] % 2:
            n = np.concatenate([n, np.full((T, 1), 8, np.uint8)], 1)
        return n[:, 0::2] | (n[:, 1::2] << 4)

    vq = np.concatenate([nibble_pack(n_o), nibble_pack(n_i)], 1)
    assert vq.shape[1] == row.v_bytes
    out[:, row.vq_off:row.vq_off + row.v_bytes] = vq
    sc = np.stack([f32_to_bf16_bits(s_out), f32_to_bf16_bits(s_in)], -1)
    out[:, row.vs_off:row.vs_off + 4] = sc.view(np.uint8).reshape(T, 4)
    return out


def unpack_rows(rows: np.ndarray, row: QuantRow, ranks) -> tuple[np.ndarray, np.ndarray]:
    """Dequantize QuantRow bytes -> (K [T, W], V [T, rv]) float32.

    kv_quant.py:154-161 (unpack_k_ref) and :182-188 (unpack_v_ref):
    value = (nibble - 8) * float(bf16 scale). Lanes past a head's rank keep
    their stored (zero) codes, as unpack_k_ref does.
    """
    T = rows.shape[0]
    widths, offsets, W = k_layout(ranks)
    kb = rows[:, :W // 2]
    n = np.stack([kb & 15, kb >> 4], -1).reshape(T, W).astype(np.float32) - 8
    k = np.zeros((T, W), dtype=np.float32)
    for h, (r, off, w) in enumerate(zip(ranks, offsets, widths)):
        no = n_outlier(r)
        sc = bf16_bits_to_f32(rows[:, row.ks_off + 4 * h:row.ks_off + 4 * h + 4].copy().view(np.uint16))
        k[:, off:off + no] = n[:, off:off + no] * sc[:, :1]
        k[:, off + no:off + w] = n[:, off + no:off + w] * sc[:, 1:2]
    R, no, nbo = row.v_rank, row.v_nout, row.v_nbo
    vb = rows[:, row.vq_off:row.vq_off + row.v_bytes]
    vs = bf16_bits_to_f32(rows[:, row.vs_off:row.vs_off + 4].copy().view(np.uint16))

    def un(b, cnt):
        return (np.stack([b & 15, b >> 4], -1).reshape(T, -1).astype(np.float32) - 8)[:, :cnt]

    v = np.concatenate([un(vb[:, :nbo], no) * vs[:, :1], un(vb[:, nbo:], R - no) * vs[:, 1:2]], 1)
    return k, v


# ---------------------------------------------------------------------------
# Decode math (model.py:1204-1220, 127-137, 1333-1386)
# ---------------------------------------------------------------------------

def gather_tokens(cache: np.ndarray, block_table: np.ndarray, b: int, L: int) -> np.ndarray:
    """Rows of sequence b's first L tokens from a paged cache [nb, bs, width]
    (paged_decode.py:63-67: block = table[b, l // bs], slot = l % bs)."""
    bs = cache.shape[1]
    pos = np.arange(L)
    return cache[block_table[b, pos // bs].astype(np.int64), pos % bs]


def attend_one(q: np.ndarray, k_rows: np.ndarray, v_rows: np.ndarray, k_up: np.ndarray,
               ranks, offsets, group: int, v_up_by_q: np.ndarray, cos_sin: np.ndarray,
               scale: float, dtype=np.float64) -> np.ndarray:
    """One sequence: q [Hq, Hd], K codes [L, W], V codes [L, rv] -> out [Hq, Hd].

    model.py:1204-1220 (`_expand_ragged_k`: K_h = x[:, off:off+rank] @ U[off:off+rank]),
    RoPE with the table rows 0..L-1 in vLLM's [cos | sin] form
    (paged_decode.py:89-95, == `k*cos + rotate_half(k)*sin` of model.py:1358),
    logits = q.K^T * scale, softmax, P @ V codes, then the per-query-head lift
    with v_up_by_q (model.py:1360-1386; paged_decode.py:199-226).
    """
    L = k_rows.shape[0]
    Hq, Hd = q.shape
    half = Hd // 2
    cs = cos_sin[:L].astype(dtype)
    cos, sin = cs[:, :half], cs[:, half:]
    kc = k_rows.astype(dtype)
    u = k_up.astype(dtype)
    out = np.empty((Hq, Hd), dtype=dtype)
    logits = np.empty((Hq, L), dtype=dtype)
    for h in range(Hq):
        g = h // group
        off, r = offsets[g], ranks[g]
        k = kc[:, off:off + r] @ u[off:off + r]                     # [L, Hd]
        k0, k1 = k[:, :half], k[:, half:]
        kr = np.concatenate([k0 * cos - k1 * sin, k1 * cos + k0 * sin], 1)
        logits[h] = (kr @ q[h].astype(dtype)) * scale
    m = logits.max(1, keepdims=True)
    p = np.exp(logits - m)
    p /= p.sum(1, keepdims=True)
    pv = p @ v_rows.astype(dtype)                                   # [Hq, rv]
    for h in range(Hq):
        out[h] = pv[h] @ v_up_by_q[h].astype(dtype)
    return out


def decode_paged_bf16(query, kv_cache, block_table, seq_lens, k_up, k_ranks, k_head_offsets,
                      k_width, v_up_by_q, cos_sin_cache, scale, seqs=None, dtype=np.float64):
    """Oracle for `paged_starkv_decode` (paged_decode.py:150-226).

    All arrays float32 (bf16 inputs already upcast) / int32. Returns [len(seqs), Hq, Hd].
    """
    n, Hq, Hd = query.shape
    Hkv = len(k_ranks)
    group = Hq // Hkv
    seqs = range(n) if seqs is None else seqs
    outs = []
    for b in seqs:
        L = max(int(seq_lens[b]), 1)
        rows = gather_tokens(kv_cache, block_table, b, L)
        outs.append(attend_one(query[b], rows[:, :k_width], rows[:, k_width:], k_up,
                               list(k_ranks), list(k_head_offsets), group, v_up_by_q,
                               cos_sin_cache, scale, dtype))
    return np.stack(outs)


def decode_paged_quant(query, kv_cache_u8, block_table, seq_lens, row: QuantRow, k_ranks,
                       k_up, v_up_by_q, cos_sin_cache, scale, seqs=None, dtype=np.float64):
    """Oracle for `paged_quant_decode` (paged_quant.py:357-411): dequantize the
    gathered rows bit-exactly (unpack_rows), then the same math as the bf16 path
    (model.py:1696-1733 is algebraically this: fold_q/abx_z/pv_fold)."""
    n, H, Hd = query.shape
    _, offsets, _ = k_layout(k_ranks)
    seqs = range(n) if seqs is None else seqs
    outs = []
    for b in seqs:
        L = max(int(seq_lens[b]), 1)
        rows = gather_tokens(kv_cache_u8, block_table, b, L)
        kd, vd = unpack_rows(rows, row, k_ranks)
        outs.append(attend_one(query[b], kd, vd, k_up, list(k_ranks), offsets, 1, v_up_by_q,
                               cos_sin_cache, scale, dtype))
    return np.stack(outs)


def fold_q(q: np.ndarray, k_up: np.ndarray, head_of_lane: np.ndarray, scale: float) -> np.ndarray:
    """Oracle for `fold_q` / `_fold_q` (paged_quant.py:223-255): the query folded
    into the K up-projection, A|B [n, W, 128] rounded to float16, with

        A[r, i] = (q_i U[r, i] + q_{i+64} U[r, i+64]) * scale
        B[r, i] = (q_{i+64} U[r, i] - q_i U[r, i+64]) * scale

    q [n, H, 128] and k_up [W, 128] as float32 (bf16 inputs upcast); head_of_lane
    [W] picks each lane's query head. Products and sums in float32 as the Triton
    kernel does (it may fuse one multiply-add, so results can differ from a fused
    implementation by one float16 ulp)."""
    q = np.asarray(q, np.float32)
    u = np.asarray(k_up, np.float32)
    qh = q[:, np.asarray(head_of_lane, np.int64), :]           # [n, W, 128]
    a0, a1 = qh[..., :64], qh[..., 64:]
    u0, u1 = u[None, :, :64], u[None, :, 64:]
    sc = np.float32(scale)
    A = ((a0 * u0 + a1 * u1) * sc).astype(np.float16)
    B = ((a1 * u0 - a0 * u1) * sc).astype(np.float16)
    return np.concatenate([A, B], axis=-1)


def rope_cos_sin(max_pos: int, head_dim: int = HEAD_DIM, base: float = 10000.0,
                 linear_factor: float = 1.0) -> np.ndarray:
    """vLLM-style rotary `cos_sin_cache` [max_pos, head_dim] = cat(cos, sin) for
    Llama's default inverse frequencies (the same angles as model.py:127-137
    `_rope_tables`, stored once per half)."""
    inv = 1.0 / (base ** (np.arange(0, head_dim, 2, dtype=np.float64) / head_dim))
    pos = np.arange(max_pos, dtype=np.float64) / linear_factor
    fr = np.outer(pos, inv)
    return np.concatenate([np.cos(fr), np.sin(fr)], 1).astype(np.float32)


def causal_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, prompt_lens, scale: float) -> np.ndarray:
    """The attention of the reference's dense prefill (attention.py:246-250,
    flash_attn_varlen_func with causal=True): prompts back to back in the token
    dimension; query t of a prompt attends to the prompt's keys up to itself.
    q [T, H, D], k [T, H_k, D], v [T, H_v, D] (query head h reads K head
    h // (H / H_k) and V head h // (H / H_v)); returns [T, H, D] in float64."""
    T, H, _ = q.shape
    gk, gv = H // k.shape[1], H // v.shape[1]
    out = np.zeros(q.shape, dtype=np.float64)
    s0 = 0
    for L in prompt_lens:
        for h in range(H):
            qs = q[s0:s0 + L, h].astype(np.float64)
            ks = k[s0:s0 + L, h // gk].astype(np.float64)
            vs = v[s0:s0 + L, h // gv].astype(np.float64)
            s = scale * qs @ ks.T
            s[np.triu_indices(L, 1)] = -np.inf
            p = np.exp(s - s.max(axis=1, keepdims=True))
            out[s0:s0 + L, h] = (p / p.sum(axis=1, keepdims=True)) @ vs
        s0 += L
    return out


def code_rows(hidden: np.ndarray, kv_down: np.ndarray) -> np.ndarray:
    """The step's cache rows before rounding: codes = F.linear(hidden, kv_down)
    (model.py:70), which attention.py:181-185 stores as cat(k_codes, v_codes) at the
    token's slot. float64 [n, W + rv]."""
    return hidden.astype(np.float64) @ kv_down.astype(np.float64).T
