// K side of the paged decode: logits of every (sequence, head, token).
//
// Replaces paged_decode.py:31-102 (_paged_abx_fwd, bf16 codes) and
// paged_quant.py:258-304 (_paged_abx_z, 3.2-bit codes).
//
// Both formats use the z-formulation of kv_quant.py:43-50: with the query and
// the logit scale folded into the K up-projection (AB = fold_q(q, U), f16,
// [W, 128] per sequence),
//     logit[t, h] = sum_{r in head h} x[t, r] * z[t, r],   z = CS[t, :] . AB[r, :]
// where CS[t] = [cos_t | sin_t] is row t of the rotary table. z is a dense
// [tokens x 128 lanes] x K=128 contraction per chunk of lanes; the codes x are
// only used elementwise in the epilogue, so the 4-bit cache is dequantized in
// registers ((n - 8) * bf16 scale, bit-exact) and never has to be laid out as an
// MMA operand.
//
// CTA pairs. Every tile of 128 tokens needs the whole AB of its sequence (W x 256 B,
// ~350 KB), which makes AB, re-read from L2, as large as the codes themselves. Two
// CTAs on neighbouring SMs therefore form a cluster and run one tcgen05.mma with
// cta_group::2 (M = 256 tokens, N = 128 lanes, K = 128): each CTA stages the rotary
// rows of its own 128 tokens (A) and HALF of every AB chunk (B, 64 lanes), so AB is
// read once per 256 tokens. CTA 0 issues the MMAs; the peer's TMA completions and
// its epilogue's buffer releases are counted on CTA 0's barriers, and each MMA
// completion is multicast to the barriers of both CTAs.
//
// Code staging. A tile's codes are read window by window (512 B of each row for
// bf16 codes, 384 B for 3.2-bit codes), one TMA box of 16 rows per page. Boxes of
// 128-byte rows cap the copy engine well below the HBM peak when every page is
// visited once per window; rows of 384-512 B stream near it. The boxes are cut from
// an 8-byte-element view of the cache without swizzling, 16 bytes wider than the
// window when needed so that the row pitch in shared memory is an odd multiple of
// 16 bytes: the epilogue's 16-byte reads of 8 consecutive token rows then fall in
// 8 different bank groups.
//
// Per tile the epilogue reduces each head's logits to the tile max m and stores
// exp(logit - m) as f16 ("e16"); the P.V kernel rescales by exp(m - M) with M the
// sequence max.
//
// Persistent CTA pairs, warp roles in each CTA:
//   warp 0      TMA producer: rotary rows and AB halves (into this CTA, counted on
//               CTA 0's barriers), code windows and 3.2-bit scales (2-slot rings,
//               from HBM) gathered through the block table;
//   warp 1      TMEM owner (pair allocation, all 512 columns); in CTA 0 also the MMA issuer;
//   warps 2-17  epilogue: thread = token row (TMEM lane) x 32-lane group of the
//               chunk. Each 16-lane tile's partial logit goes to its own f16 slot
//               (one writer per tile and token); the tile pass adds a head's tiles.
//               Layers too wide for those slots merge per-head sums with
//               shared-memory atomics instead.
#include "starkv_common.cuh"
#include "starkv_kernels.h"

namespace starkv {

namespace {

constexpr int kTile = 128;       // tokens per CTA and tile (MMA M / 2)
constexpr int kPairTokens = 2 * kTile;
constexpr int kChunk = 128;      // lanes per MMA (N)
constexpr int kHalfLanes = kChunk / 2;   // AB lanes staged by each CTA of the pair
constexpr int kCodeSlots = 2;
constexpr int kCsBytes = kTile * 128 * 2;       // f16 [128 tokens][128]
constexpr int kAbBytes = kHalfLanes * 128 * 2;  // f16 [64 lanes][128] per CTA
constexpr int kTmemCols = 512;
constexpr int kTmemBufs = kTmemCols / kChunk;
constexpr int kGroups = kChunk / 32;            // 32-lane groups per chunk
constexpr int kEpiWarps = 4 * kGroups;          // 4 TMEM lane quarters x groups
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kMaxAbSlots = 3;

template <bool QUANT>
struct Cfg {
  static constexpr int kAbSlots = QUANT ? 3 : 2;
  static constexpr int kWinLanes = QUANT ? 768 : 256;        // lanes per code window
  static constexpr int kWinBytes = QUANT ? kWinLanes / 2 : kWinLanes * 2;
  static constexpr int kChunksPerWin = kWinLanes / kChunk;
};

struct SharedCtl {
  uint64_t ab_full[kMaxAbSlots], ab_empty[kMaxAbSlots];
  uint64_t code_full[kCodeSlots], code_empty[kCodeSlots];
  uint64_t cs_full, cs_empty, sc_full, sc_empty;
  uint64_t tfull[kTmemBufs], tempty[kTmemBufs];
  uint64_t epi;            // bounded barrier among the epilogue warps
  uint32_t tmem_base;
  int abort_flag;
};

// Shared memory carve-up (byte offsets from the 1024-aligned base).
struct SmemLayout {
  int cs, ab, codes, code_slot, sc, logits, tiles, hspan, prefix, sbeg, ctl, total;
};

// parts: the epilogue stores one f16 partial per (16-lane tile, token) [NC * 8][128]
// instead of adding per-head f32 sums [H][129] with shared-memory atomics.
__host__ __device__ inline SmemLayout smem_layout(bool quant, bool parts, int H, int n, int k_width,
                                                  int code_pitch, int sc_pitch) {
  SmemLayout L;
  const int ab_slots = quant ? Cfg<true>::kAbSlots : Cfg<false>::kAbSlots;
  const int nc = (k_width + kChunk - 1) / kChunk;
  L.cs = 0;
  L.ab = L.cs + kCsBytes;
  L.codes = L.ab + ab_slots * kAbBytes;
  L.code_slot = (kTile * code_pitch + 127) & ~127;
  L.sc = L.codes + kCodeSlots * L.code_slot;
  L.logits = L.sc + (quant ? (kTile * sc_pitch + 127) & ~127 : 0);
  L.tiles = (L.logits + (parts ? nc * (kChunk / 16) * kTile * 2 : H * (kTile + 1) * 4) + 15) & ~15;
  L.hspan = L.tiles + nc * (kChunk / 16) * 4;   // [H] first tile | tile count << 16
  L.prefix = L.hspan + H * 4;
  L.sbeg = L.prefix + (n + 1) * 4;
  L.ctl = (L.sbeg + n * 4 + 15) & ~15;
  L.total = L.ctl + (int)sizeof(SharedCtl);
  return L;
}

__device__ __forceinline__ int find_seq(const int* prefix, int n, int item) {
  int lo = 0, hi = n;  // prefix[lo] <= item < prefix[hi]
  while (hi - lo > 1) {
    int mid = (lo + hi) >> 1;
    if (prefix[mid] <= item) lo = mid; else hi = mid;
  }
  return lo;
}

}  // namespace

// Row pitch (bytes) of a staged code window of `bytes` bytes: rounded up to 16 and,
// if needed, one more 16 so that pitch / 16 is odd.
int code_pitch_bytes(int bytes) {
  int p = (bytes + 15) & ~15;
  if (((p >> 4) & 1) == 0) p += 16;
  return p;
}

int scores_window_bytes(bool quant) { return quant ? Cfg<true>::kWinBytes : Cfg<false>::kWinBytes; }

size_t scores_smem_bytes(bool quant, int num_kv_heads, int n, int k_width, int code_pitch, int sc_pitch,
                         bool parts) {
  return (size_t)smem_layout(quant, parts, num_kv_heads, n, k_width, code_pitch, sc_pitch).total + 1024;
}

template <bool QUANT, bool F16, bool PARTS>
__global__ void __launch_bounds__(kThreads, 1)
scores_kernel(const __grid_constant__ CUtensorMap tm_cs, const __grid_constant__ CUtensorMap tm_ab,
              const __grid_constant__ CUtensorMap tm_code, const __grid_constant__ CUtensorMap tm_tail,
              const __grid_constant__ CUtensorMap tm_sc, const ScoresParams p) {
  using C = Cfg<QUANT>;
  constexpr int kAbSlots = C::kAbSlots;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int H = p.num_kv_heads;
  const int NT = p.k_width / 16;
  const int NC = (p.k_width + kChunk - 1) / kChunk;
  const SmemLayout SL = smem_layout(QUANT, PARTS, H, p.n, p.k_width, p.code_pitch, p.sc_pitch);
  float* logits = reinterpret_cast<float*>(smem + SL.logits);    // !PARTS: [H][129] per-head sums
  __half* parts = reinterpret_cast<__half*>(smem + SL.logits);   // PARTS: [NC * 8][128] per-tile partials
  int* tiles = reinterpret_cast<int*>(smem + SL.tiles);           // [NC * 8], -1 past NT
  int* hspan = reinterpret_cast<int*>(smem + SL.hspan);           // [H] first tile | count << 16
  int* prefix = reinterpret_cast<int*>(smem + SL.prefix);         // [n+1] item prefix over sequences
  int* sbeg = reinterpret_cast<int*>(smem + SL.sbeg);             // [n] first 256-token tile of this rank
  SharedCtl* ctl = reinterpret_cast<SharedCtl*>(smem + SL.ctl);
  volatile int* abort_flag = &ctl->abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();           // 0: issues the pair's MMAs
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;

  // ---- prologue: tables, zeroed logits, barriers, TMEM ----
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int b = 0; b < p.n; ++b) {
      prefix[b] = acc;
      const int L = min(max(p.seq_lens[b], 0), p.max_seq_len);
      const int T = (L + kPairTokens - 1) / kPairTokens;     // 256-token tiles of the sequence
      const int s0 = (int)((int64_t)T * p.cp_rank / p.cp_world), s1 = (int)((int64_t)T * (p.cp_rank + 1) / p.cp_world);
      sbeg[b] = s0;
      acc += (s1 - s0) * p.group;
    }
    prefix[p.n] = acc;
  }
  for (int t = threadIdx.x; t < NC * (kChunk / 16); t += blockDim.x) {
    int entry = -1;   // head | outlier lanes << 16 (3.2-bit)
    if (t >= NT) {
    } else if (QUANT) {
      const int h = p.tile_head[t];
      if (h >= 0 && h < H) entry = h | (min(max(p.tile_nout[t], 0), 16) << 16);
      else record_status(p.status, STARKV_EBOUNDS);
    } else {
      for (int h = 0; h < H; ++h) {
        const int off = p.k_head_offsets[h], w = (p.k_ranks[h] + 15) & ~15;
        if (16 * t >= off && 16 * t < off + w) {
          entry = h;
          break;
        }
      }
    }
    tiles[t] = entry;
  }
  if (!PARTS)
    for (int i = threadIdx.x; i < H * (kTile + 1); i += blockDim.x) logits[i] = 0.f;
  // each head's range of 16-lane tiles, first | span << 16 (the tile pass adds the
  // partials of the range's tiles that belong to the head)
  if (PARTS)
    for (int h = threadIdx.x; h < H; h += blockDim.x) {
      int first = 0, span = 0;
      if (QUANT) {
        for (int t = 0; t < NT; ++t)
          if (p.tile_head[t] == h) {
            if (span == 0) first = t;
            span = t - first + 1;
          }
      } else {
        first = min(max(p.k_head_offsets[h], 0), NT * 16) / 16;
        span = min((max(p.k_ranks[h], 0) + 15) / 16 + 1, NT - first);
      }
      hspan[h] = first | (span << 16);
    }
  if (threadIdx.x == 0) {
    // In CTA 0, ab_full / cs_full count the TMA bytes of BOTH CTAs and tempty the
    // epilogue warps of both; the peer's own copies of those barriers stay unused.
    for (int s = 0; s < kAbSlots; ++s) {
      mbar_init(&ctl->ab_full[s], 1);
      mbar_init(&ctl->ab_empty[s], 1);
    }
    for (int s = 0; s < kCodeSlots; ++s) {
      mbar_init(&ctl->code_full[s], 1);
      mbar_init(&ctl->code_empty[s], kEpiWarps);
    }
    mbar_init(&ctl->cs_full, 1);
    mbar_init(&ctl->cs_empty, 1);
    mbar_init(&ctl->sc_full, 1);
    mbar_init(&ctl->sc_empty, kEpiWarps);
    for (int i = 0; i < kTmemBufs; ++i) {
      mbar_init(&ctl->tfull[i], 1);
      mbar_init(&ctl->tempty[i], 2 * kEpiWarps);
    }
    mbar_init(&ctl->epi, kEpiWarps);   // one arrival per epilogue warp
    ctl->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc_pair(&ctl->tmem_base, kTmemCols);
  tc_fence_before();
  cluster_sync_all();   // both CTAs' barriers and TMEM exist before any remote use
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const int total_items = prefix[p.n];

  if (warp == 0) {
    // ================= TMA producer (both CTAs) =================
    // Lanes 0-7 fetch the 8 block ids of this CTA's half of the NEXT item while
    // lane 0 issues the current copies, so the block table's latency stays off the
    // issue path.
    if (lane == 0) {
      tma_prefetch(&tm_cs);
      tma_prefetch(&tm_ab);
      tma_prefetch(&tm_code);
      tma_prefetch(&tm_tail);
      if (QUANT) tma_prefetch(&tm_sc);
    }
    auto block_of = [&](int item) -> int {   // block id of page `lane` of an item (lanes 0-7)
      if (item >= total_items || lane >= 8) return 0;
      const int b = find_seq(prefix, p.n, item);
      const int sup = sbeg[b] + (item - prefix[b]) / p.group;
      const int L = min(max(p.seq_lens[b], 0), p.max_seq_len);
      const int t = sup * kPairTokens + kTile * (int)rank + 16 * lane;
      if (t >= L) return 0;
      const int col = t / p.block_size;
      int id = -1;
      if (col < p.max_blocks) id = p.block_table[(int64_t)b * p.bt_s0 + (int64_t)col * p.bt_s1];
      if (id < 0 || id >= p.num_blocks) {
        record_status(p.status, STARKV_EBOUNDS);
        id = 0;
      }
      return id;
    };
    const int win_u64 = C::kWinBytes / 8;
    const uint32_t cs_full_l = leader_addr(&ctl->cs_full);
    uint32_t ab_it = 0, code_it = 0, item_cnt = 0;
    int ids_next = block_of(pair);
    for (int item = pair; item < total_items; item += n_pairs, ++item_cnt) {
      const int ids = ids_next;
      ids_next = block_of(item + n_pairs);
      int blk[8], slot[8];
#pragma unroll
      for (int pg = 0; pg < 8; ++pg) blk[pg] = __shfl_sync(0xffffffffu, ids, pg);
      int ok = 1;
      if (lane == 0) {
        const int b = find_seq(prefix, p.n, item);
        const int rem = item - prefix[b];
        const int j = rem % p.group;
        const int t0 = (sbeg[b] + rem / p.group) * kPairTokens + kTile * (int)rank;   // this CTA's first token
#pragma unroll
        for (int pg = 0; pg < 8; ++pg) slot[pg] = (t0 + 16 * pg) % p.block_size;
        // rotary rows of this CTA's tokens: the pair MMA's A half
        ok = !*abort_flag && mbar_wait(&ctl->cs_empty, (item_cnt & 1) ^ 1, abort_flag, p.status);
        if (ok) {
          if (rank == 0) mbar_arrive_expect_tx(&ctl->cs_full, 2 * kCsBytes);
          tma_load_2d_pair(smem + SL.cs, &tm_cs, cs_full_l, 0, (t0 / kTile) * 16);   // one 32 KB tile image
        }
        if (ok && QUANT) {
          ok = mbar_wait(&ctl->sc_empty, (item_cnt & 1) ^ 1, abort_flag, p.status);
          if (ok) {
            mbar_arrive_expect_tx(&ctl->sc_full, kTile * p.sc_pitch);
            for (int pg = 0; pg < 8; ++pg)
              tma_load_3d(smem + SL.sc + pg * 16 * p.sc_pitch, &tm_sc, &ctl->sc_full, p.sc_x0 / 8, slot[pg], blk[pg]);
          }
        }
        // this CTA's half of each AB chunk (lanes [64 rank, 64 rank + 64) of the chunk):
        // 16 KB image blocks, 8 rows of 2 KB each
        const int ab_row0 = ((b * p.group + j) * NC * 2 + (int)rank) * 8;
        for (int c = 0; ok && c < NC; ++c, ++ab_it) {
          if (c % C::kChunksPerWin == 0) {
            // next code window of this CTA's tokens: one box of 16 rows per page
            const int w = c / C::kChunksPerWin;
            const bool tail = w == p.n_wins - 1;
            const int pitch = tail ? p.tail_pitch : p.code_pitch;
            const int sc = code_it % kCodeSlots;
            if (!mbar_wait(&ctl->code_empty[sc], ((code_it / kCodeSlots) & 1) ^ 1, abort_flag, p.status)) {
              ok = 0;
              break;
            }
            uint8_t* cds = smem + SL.codes + sc * SL.code_slot;
            mbar_arrive_expect_tx(&ctl->code_full[sc], kTile * pitch);
#pragma unroll
            for (int pg = 0; pg < 8; ++pg)
              tma_load_3d(cds + pg * 16 * pitch, tail ? &tm_tail : &tm_code, &ctl->code_full[sc], w * win_u64,
                          slot[pg], blk[pg]);
            ++code_it;
          }
          const int sa = ab_it % kAbSlots;
          if (!mbar_wait(&ctl->ab_empty[sa], ((ab_it / kAbSlots) & 1) ^ 1, abort_flag, p.status)) {
            ok = 0;
            break;
          }
          uint8_t* abs = smem + SL.ab + sa * kAbBytes;
          const uint32_t full_l = leader_addr(&ctl->ab_full[sa]);
          if (rank == 0) mbar_arrive_expect_tx(&ctl->ab_full[sa], 2 * kAbBytes);
          tma_load_2d_pair(abs, &tm_ab, full_l, 0, ab_row0 + c * 16);
        }
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
    }
    // Drain: wait for the MMA completions still to be multicast into this CTA's
    // empty barriers (the last AB slots and the last rotary rows), so none lands
    // after the CTA has left.
    if (lane == 0 && !*abort_flag) {
      for (int k = 0; k < kAbSlots; ++k) {
        const uint32_t it = ab_it + k;
        if (!mbar_wait(&ctl->ab_empty[it % kAbSlots], ((it / kAbSlots) & 1) ^ 1, abort_flag, p.status)) break;
      }
      mbar_wait(&ctl->cs_empty, (item_cnt & 1) ^ 1, abort_flag, p.status);
    }
  } else if (warp == 1) {
    // ================= MMA issuer (CTA 0 of the pair) =================
    if (rank == 0 && lane == 0) {
      const uint32_t idesc = instr_desc_f16(/*f16*/ 0, 0, 0, kPairTokens, kChunk);
      uint32_t ab_it = 0, tb = 0, item_cnt = 0;
      const uint32_t cs_addr = smem_u32(smem + SL.cs);
      for (int item = pair; item < total_items && !*abort_flag; item += n_pairs, ++item_cnt) {
        if (!mbar_wait(&ctl->cs_full, item_cnt & 1, abort_flag, p.status)) break;
        tc_fence_after();
        for (int c = 0; c < NC; ++c, ++ab_it, ++tb) {
          const int sa = ab_it % kAbSlots;
          const int buf = tb % kTmemBufs;
          if (!mbar_wait(&ctl->ab_full[sa], (ab_it / kAbSlots) & 1, abort_flag, p.status)) break;
          if (!mbar_wait(&ctl->tempty[buf], ((tb / kTmemBufs) & 1) ^ 1, abort_flag, p.status)) break;
          tc_fence_after();
          const uint32_t ab_addr = smem_u32(smem + SL.ab + sa * kAbBytes);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t da = smem_desc(cs_addr + (kk >> 2) * (kCsBytes / 2) + (kk & 3) * 32, 16, 1024,
                                          kSwizzle128B);
            const uint64_t db = smem_desc(ab_addr + (kk >> 2) * (kAbBytes / 2) + (kk & 3) * 32, 16, 1024,
                                          kSwizzle128B);
            umma_f16_pair(tmem + buf * kChunk, da, db, idesc, kk > 0);
          }
          umma_commit_pair(&ctl->ab_empty[sa]);
          umma_commit_pair(&ctl->tfull[buf]);
        }
        umma_commit_pair(&ctl->cs_empty);
      }
    }
  } else {
    // ================= epilogue (warps 2-17, both CTAs) =================
    // Thread = (token row of this CTA's tile, 32-lane group g of the chunk): warp w
    // may only read TMEM lanes 32 (w % 4) .. +32, so the 16 warps cover the 4 lane
    // quarters x 4 groups.
    const int ew = warp - 2;              // 0..15
    const int q = warp & 3;               // TMEM lane quarter this warp may access
    const int g = ew >> 2;                // 32-lane group: chunk columns [32 g, 32 g + 32)
    const int row = q * 32 + lane;        // token within the tile
    uint32_t code_it = 0, tb = 0, item_cnt = 0, epi_phase = 0;
    // Bounded barrier among the epilogue threads (a plain bar.sync could wait
    // forever if another epilogue warp left on a timed-out pipeline wait).
    // One arrival per warp, after __syncwarp (which orders the lanes' shared-memory
    // writes before lane 0's release): an arrival per thread, 512 on one barrier
    // word, serialised in the shared-memory unit.
    auto epi_sync = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->epi);
      return mbar_wait(&ctl->epi, (epi_phase++) & 1, abort_flag, p.status);
    };
    const uint32_t tempty_l = leader_addr(&ctl->tempty[0]);
    for (int item = pair; item < total_items; item += n_pairs, ++item_cnt) {
      if (*abort_flag) break;
      const int b = find_seq(prefix, p.n, item);
      const int rem = item - prefix[b];
      const int j = rem % p.group;
      const int tile = (sbeg[b] + rem / p.group) * 2 + (int)rank;   // this CTA's 128-token tile
      const int L = min(max(p.seq_lens[b], 0), p.max_seq_len);
      const int t0 = tile * kTile;
      if (QUANT && !mbar_wait(&ctl->sc_full, item_cnt & 1, abort_flag, p.status)) break;
      // running sums of the current head: 4 independent chains over all of its
      // lanes (ai); 3.2-bit codes also sum the outlier lanes apart (ao), so the
      // flush applies logit = s_in * ai + (s_out - s_in) * ao.
      float2 ai[4], ao[2];
#pragma unroll
      for (int i = 0; i < 4; ++i) ai[i] = make_float2(0.f, 0.f);
      ao[0] = ao[1] = make_float2(0.f, 0.f);
      int cur_h = -1;
      int sc_h = -1;            // PARTS, 3.2-bit: head whose scales so_c / si_c hold
      float so_c = 0.f, si_c = 0.f;
      auto flush = [&]() {
        const float all = ((ai[0].x + ai[0].y) + (ai[1].x + ai[1].y)) + ((ai[2].x + ai[2].y) + (ai[3].x + ai[3].y));
        float v;
        if (QUANT) {
          // (outlier, inlier) bf16 scales of head cur_h for this token
          const uint32_t sw = *reinterpret_cast<const uint32_t*>(smem + SL.sc + row * p.sc_pitch + p.ks_off +
                                                                 4 * cur_h - p.sc_x0);
          const float so = __uint_as_float(sw << 16), si = __uint_as_float(sw & 0xFFFF0000u);
          const float out = (ao[0].x + ao[0].y) + (ao[1].x + ao[1].y);
          v = si * all + (so - si) * out;
        } else {
          v = all;
        }
        atomicAdd(&logits[cur_h * (kTile + 1) + row], v);
#pragma unroll
        for (int i = 0; i < 4; ++i) ai[i] = make_float2(0.f, 0.f);
        ao[0] = ao[1] = make_float2(0.f, 0.f);
      };
      bool ok = true;
      int sc = 0;
      const uint8_t* crow = nullptr;   // this token's row of the current code window
      for (int c = 0; c < NC; ++c, ++tb) {
        const int buf = tb % kTmemBufs;
        const int cw = c % C::kChunksPerWin;
        if (cw == 0) {
          sc = code_it % kCodeSlots;
          const int pitch = (c / C::kChunksPerWin == p.n_wins - 1) ? p.tail_pitch : p.code_pitch;
          crow = smem + SL.codes + sc * SL.code_slot + row * pitch;
          if (!mbar_wait(&ctl->code_full[sc], (code_it / kCodeSlots) & 1, abort_flag, p.status)) {
            ok = false;
            break;
          }
        }
        if (!mbar_wait(&ctl->tfull[buf], (tb / kTmemBufs) & 1, abort_flag, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (NT * 16 > c * kChunk + 32 * g) {   // this group holds real lanes (warp-uniform)
          uint32_t z[32];
          tmem_ld32_issue(tmem + ((uint32_t)(q * 32) << 16) + buf * kChunk + 32 * g, z);
          // this token's codes of the group's 32 lanes, read while the TMEM load is in flight
          const int lane_in_win = cw * kChunk + 32 * g;
          constexpr int kWords = QUANT ? 4 : 16;
          uint32_t w[kWords];
          if (QUANT) {
            const uint4 u = *reinterpret_cast<const uint4*>(crow + lane_in_win / 2);
            w[0] = u.x; w[1] = u.y; w[2] = u.z; w[3] = u.w;
          } else {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const uint4 u = *reinterpret_cast<const uint4*>(crow + lane_in_win * 2 + 16 * v);
              w[4 * v] = u.x; w[4 * v + 1] = u.y; w[4 * v + 2] = u.z; w[4 * v + 3] = u.w;
            }
          }
          const int2 m2 = reinterpret_cast<const int2*>(tiles)[c * kGroups + g];   // the 2 lane tiles
          tmem_wait(z);
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int meta = hh == 0 ? m2.x : m2.y;
            if (meta < 0) continue;
            const int h = meta & 0xFFFF;
            if (PARTS) {   // the sums below are this tile's alone
#pragma unroll
              for (int i = 0; i < 4; ++i) ai[i] = make_float2(0.f, 0.f);
              ao[0] = ao[1] = make_float2(0.f, 0.f);
            } else if (h != cur_h) {
              if (cur_h >= 0) flush();
              cur_h = h;
            }
            float2 x2[8];   // codes of lanes (2i, 2i+1) of this 16-lane tile
            if (QUANT) {
              const float2 off8 = make_float2(-8388616.f, -8388616.f);
#pragma unroll
              for (int k = 0; k < 2; ++k) {
                const uint32_t wd = w[2 * hh + k];
                const uint32_t lo = wd & 0x0F0F0F0Fu, hi = (wd >> 4) & 0x0F0F0F0Fu;
#pragma unroll
                for (int bb = 0; bb < 4; ++bb) {
                  // bytes 0x4B0000nn are the float 2^23 + n; minus 2^23 + 8 gives n - 8
                  const float2 raw = make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7650u | bb)),
                                                 __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7650u | bb)));
                  x2[4 * k + bb] = __fadd2_rn(raw, off8);
                }
              }
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const uint32_t wd = w[8 * hh + i];
                if (F16)
                  x2[i] = __half22float2(*reinterpret_cast<const __half2*>(&wd));
                else
                  x2[i] = make_float2(__uint_as_float(wd << 16), __uint_as_float(wd & 0xFFFF0000u));
              }
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float2 zz = make_float2(__uint_as_float(z[16 * hh + 2 * i]), __uint_as_float(z[16 * hh + 2 * i + 1]));
              ai[i & 3] = __ffma2_rn(x2[i], zz, ai[i & 3]);
            }
            if (QUANT) {
              const int nout = (meta >> 16) & 0xFF;   // outlier lanes lead the head's first tile
              if (nout > 0) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  const float2 zz =
                      make_float2(__uint_as_float(z[16 * hh + 2 * i]), __uint_as_float(z[16 * hh + 2 * i + 1]));
                  if (2 * i + 1 < nout)
                    ao[i & 1] = __ffma2_rn(x2[i], zz, ao[i & 1]);
                  else if (2 * i < nout)
                    ao[0].x = fmaf(x2[i].x, zz.x, ao[0].x);
                }
              }
            }
            if (PARTS) {
              // this tile's partial logit (scales of its head applied) -> its own slot:
              // one writer per (tile, token), no atomics
              const float2 s01 = __fadd2_rn(__fadd2_rn(ai[0], ai[1]), __fadd2_rn(ai[2], ai[3]));
              float v = s01.x + s01.y;
              if (QUANT) {
                if (h != sc_h) {
                  const uint32_t sw = *reinterpret_cast<const uint32_t*>(smem + SL.sc + row * p.sc_pitch + p.ks_off +
                                                                         4 * h - p.sc_x0);
                  so_c = __uint_as_float(sw << 16);
                  si_c = __uint_as_float(sw & 0xFFFF0000u);
                  sc_h = h;
                }
                const float out = (ao[0].x + ao[0].y) + (ao[1].x + ao[1].y);
                v = si_c * v + (so_c - si_c) * out;
              }
              parts[(c * kGroups * 2 + 2 * g + hh) * kTile + row] = __float2half_rn(v);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive_cluster(tempty_l + 8u * buf);   // the MMA issuer's barrier, in CTA 0
          if (cw == C::kChunksPerWin - 1 || c == NC - 1) mbar_arrive(&ctl->code_empty[sc]);
        }
        if (cw == C::kChunksPerWin - 1 || c == NC - 1) ++code_it;
      }
      if (!PARTS && cur_h >= 0) flush();
      if (QUANT) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->sc_empty);
      }
      if (!ok || !epi_sync()) break;
      // ---- per-head tile max, e16 = exp(logit - max), and the logits cleared for the
      // next tile's atomic flushes: warp ew owns heads ew, ew + 16, ...; lane l tokens
      // l, l + 32, l + 64, l + 96 (consecutive words: conflict-free) ----
      for (int h = ew; h < H; h += kEpiWarps) {
        float v[4];
        float m = -INFINITY;
        if (PARTS) {
          // the head's logit is the sum of its tiles' partials
          const int sp = hspan[h], tf = sp & 0xFFFF, cnt = sp >> 16;
#pragma unroll
          for (int i = 0; i < 4; ++i) v[i] = 0.f;
          for (int k = 0; k < cnt; ++k) {
            if ((tiles[tf + k] & 0xFFFF) != h) continue;   // -1 (past the lanes) or another head
            const __half* pr = parts + (tf + k) * kTile;
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] += __half2float(pr[lane + 32 * i]);
          }
        } else {
          float* lrow = logits + h * (kTile + 1);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            v[i] = lrow[lane + 32 * i];
            lrow[lane + 32 * i] = 0.f;
          }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (t0 + lane + 32 * i < L) m = fmaxf(m, v[i]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (t0 < L) {
          const int hq = h * p.group + j;
          __half* dst = p.e16 + ((int64_t)b * p.num_heads + hq) * p.l_pad + t0;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int t = lane + 32 * i;
            dst[t] = __float2half_rn(t0 + t < L ? __expf(v[i] - m) : 0.f);
          }
          if (lane == 0) {
            p.m_tile[((int64_t)b * p.num_heads + hq) * p.n_tiles + tile] = m;
            atomic_max_f32(p.m_seq + (int64_t)b * p.num_heads + hq, m);
          }
        }
      }
      if (!epi_sync()) break;
    }
  }

  // ---- teardown: no pair MMA, remote arrive or commit may target a CTA that left ----
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

namespace {

template <bool QUANT, bool F16, bool PARTS>
int launch_pairs(const CUtensorMap& tm_cs, const CUtensorMap& tm_ab, const CUtensorMap& tm_code,
                 const CUtensorMap& tm_tail, const CUtensorMap& tm_sc, const ScoresParams& p, int num_sms,
                 size_t smem, cudaStream_t stream) {
  auto fn = scores_kernel<QUANT, F16, PARTS>;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return STARKV_ECUDA;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // persistent: as many pairs as can be resident at once (SMs that cannot be
  // paired inside a GPC stay idle rather than run a second wave)
  int dev = 0;
  cudaGetDevice(&dev);
  static int max_pairs[64][2][2] = {};
  int& mp = max_pairs[dev & 63][QUANT ? 1 : 0][PARTS ? 1 : 0];
  if (mp == 0) {
    cfg.gridDim = dim3(num_sms & ~1);
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, (const void*)fn, &cfg) != cudaSuccess || clusters <= 0)
      clusters = num_sms / 2;
    mp = clusters < num_sms / 2 ? clusters : num_sms / 2;
  }
  cfg.gridDim = dim3(2 * mp);
  if (cudaLaunchKernelEx(&cfg, fn, tm_cs, tm_ab, tm_code, tm_tail, tm_sc, p) != cudaSuccess) return STARKV_ECUDA;
  return STARKV_OK;
}

}  // namespace

int launch_scores(bool quant, const CUtensorMap& tm_cs, const CUtensorMap& tm_ab, const CUtensorMap& tm_code,
                  const CUtensorMap& tm_tail, const CUtensorMap& tm_sc, const ScoresParams& p, int num_sms,
                  cudaStream_t stream) {
  // per-tile partials when their shared memory fits (wide layers fall back to the
  // per-head sums merged with shared-memory atomics)
  const size_t smem_p = scores_smem_bytes(quant, p.num_kv_heads, p.n, p.k_width, p.code_pitch, p.sc_pitch, true);
  const size_t smem_a = scores_smem_bytes(quant, p.num_kv_heads, p.n, p.k_width, p.code_pitch, p.sc_pitch, false);
  const bool parts = smem_p <= 227 * 1024;
  const size_t smem = parts ? smem_p : smem_a;
  if (smem > 227 * 1024) return STARKV_EINVAL;
  if (quant)
    return parts ? launch_pairs<true, false, true>(tm_cs, tm_ab, tm_code, tm_tail, tm_sc, p, num_sms, smem, stream)
                 : launch_pairs<true, false, false>(tm_cs, tm_ab, tm_code, tm_tail, tm_sc, p, num_sms, smem, stream);
  if (p.cache_dtype == STARKV_F16)
    return parts ? launch_pairs<false, true, true>(tm_cs, tm_ab, tm_code, tm_tail, tm_sc, p, num_sms, smem, stream)
                 : launch_pairs<false, true, false>(tm_cs, tm_ab, tm_code, tm_tail, tm_sc, p, num_sms, smem, stream);
  return parts ? launch_pairs<false, false, true>(tm_cs, tm_ab, tm_code, tm_tail, tm_sc, p, num_sms, smem, stream)
               : launch_pairs<false, false, false>(tm_cs, tm_ab, tm_code, tm_tail, tm_sc, p, num_sms, smem, stream);
}

}  // namespace starkv
