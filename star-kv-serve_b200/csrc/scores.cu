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
// [128 tokens x 128 lanes] x K=128 contraction per chunk: it runs on the
// tcgen05 tensor core (M=128 tokens, N=128 lanes, K=128, f16 in, f32 in TMEM).
// The codes x are only used elementwise in the epilogue, so the 4-bit cache is
// dequantized in registers ((n - 8) * bf16 scale, bit-exact) and never has to
// be laid out as an MMA operand.
//
// Per tile (one sequence, 128 tokens) the epilogue reduces each head's logits
// to (tile max m, tile sum l = sum exp(logit - m)) and stores exp(logit - m) as
// f16 ("e16"); the P.V kernel rescales by exp(m - M) with M the sequence max.
//
// Warp roles (persistent CTAs, one per SM): warp 0 TMA producer, warp 1 MMA
// issuer (also owns the TMEM allocation), warps 2-5 epilogue (one token row per
// thread, TMEM lanes 0-127).
#include "starkv_common.cuh"
#include "starkv_kernels.h"

namespace starkv {

namespace {

constexpr int kTile = 128;       // tokens per tile (MMA M)
constexpr int kChunk = 128;      // lanes per chunk (MMA N)
constexpr int kTmemBufs = 2;
constexpr int kCsBytes = kTile * 128 * 2;       // f16 [128 tokens][128]
constexpr int kAbBytes = kChunk * 128 * 2;      // f16 [128 lanes][128]
constexpr int kMaxStages = 3;

template <bool QUANT>
struct Layout {
  // bf16 codes: 2 boxes of 64 lanes (128 B) per page; 3.2-bit codes: one box of
  // 64 bytes (128 lanes) per page.
  static constexpr int kStages = QUANT ? 3 : 2;
  static constexpr int kCodeBoxes = QUANT ? 1 : 2;
  static constexpr int kCodeBoxBytes = QUANT ? 16 * 64 : 16 * 128;
  static constexpr int kCodeBytes = 8 * kCodeBoxes * kCodeBoxBytes;   // per stage (8 pages)
  static constexpr int kStageBytes = kAbBytes + kCodeBytes;
  static constexpr int kOffCs = 0;
  static constexpr int kOffStages = kOffCs + kCsBytes;
  static constexpr int kOffScales = kOffStages + kStages * kStageBytes;   // 3.2-bit scale boxes
  // logits and tables follow the scale boxes (8 pages x ks_boxes x 2 KB)
  static __host__ __device__ int off_logits(int ks_boxes) { return kOffScales + ks_boxes * 8 * 2048; }
};

struct SharedCtl {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t epi;            // bounded barrier among the 4 epilogue warps
  uint64_t cs_full, cs_empty, sc_full, sc_empty;
  uint64_t tfull[kTmemBufs];
  uint64_t tempty[kTmemBufs];
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ int find_seq(const int* prefix, int n, int item) {
  int lo = 0, hi = n;  // prefix[lo] <= item < prefix[hi]
  while (hi - lo > 1) {
    int mid = (lo + hi) >> 1;
    if (prefix[mid] <= item) lo = mid; else hi = mid;
  }
  return lo;
}

}  // namespace

size_t scores_smem_bytes(bool quant, int num_kv_heads, int n, int k_width, int ks_boxes) {
  const int nt = k_width / 16;
  size_t bytes = quant ? Layout<true>::off_logits(ks_boxes) : Layout<false>::off_logits(0);
  bytes += (size_t)num_kv_heads * (kTile + 1) * 4;    // logits [H][129]
  bytes += (size_t)2 * 4 * num_kv_heads * 4;          // cross-warp max / sum
  bytes += (size_t)nt * 4;                            // lane-tile table
  bytes += (size_t)(n + 1) * 4;                       // tile prefix over sequences
  bytes = (bytes + 15) & ~size_t(15);
  bytes += sizeof(SharedCtl) + 1024;                  // control + alignment slack
  return bytes;
}

template <bool QUANT>
__global__ void __launch_bounds__(192, 1)
scores_kernel(const __grid_constant__ CUtensorMap tm_cs, const __grid_constant__ CUtensorMap tm_ab,
              const __grid_constant__ CUtensorMap tm_codes, const __grid_constant__ CUtensorMap tm_scales,
              const ScoresParams p) {
  using LY = Layout<QUANT>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int H = p.num_kv_heads;
  const int NT = p.k_width / 16;
  const int NC = (p.k_width + kChunk - 1) / kChunk;
  const int ks_boxes = QUANT ? p.ks_boxes : 0;
  float* logits = reinterpret_cast<float*>(smem + LY::off_logits(ks_boxes));   // [H][129]
  float* red_m = logits + H * (kTile + 1);                            // [4][H]
  float* red_l = red_m + 4 * H;                                       // [4][H]
  int* tiles = reinterpret_cast<int*>(red_l + 4 * H);                 // [NT]
  int* prefix = tiles + NT;                                           // [n+1]
  SharedCtl* ctl = reinterpret_cast<SharedCtl*>((reinterpret_cast<uintptr_t>(prefix + p.n + 1) + 15) & ~uintptr_t(15));
  volatile int* abort_flag = &ctl->abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---- prologue: tables, barriers, TMEM ----
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int b = 0; b < p.n; ++b) {
      prefix[b] = acc;
      int L = p.seq_lens[b];
      L = L < 0 ? 0 : (L > p.max_seq_len ? p.max_seq_len : L);
      acc += (L + kTile - 1) / kTile * p.group;
    }
    prefix[p.n] = acc;
  }
  for (int t = threadIdx.x; t < NT; t += blockDim.x) {
    int entry = -1;
    if (QUANT) {
      int h = p.tile_head[t];
      if (h >= 0 && h < H) entry = h | (min(max(p.tile_nout[t], 0), 16) << 16) | ((p.tile_last[t] != 0) << 24);
      else record_status(p.status, STARKV_EBOUNDS);
    } else {
      for (int h = 0; h < H; ++h) {
        int off = p.k_head_offsets[h], r = p.k_ranks[h];
        int w = (r + 15) & ~15;
        if (16 * t >= off && 16 * t < off + w) {
          entry = h | ((16 * t + 16 >= off + w) << 24);
          break;
        }
      }
    }
    tiles[t] = entry;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < LY::kStages; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1 + 4);
    }
    mbar_init(&ctl->epi, 128);
    mbar_init(&ctl->cs_full, 1);
    mbar_init(&ctl->cs_empty, 1);
    mbar_init(&ctl->sc_full, 1);
    mbar_init(&ctl->sc_empty, 4);
    for (int i = 0; i < kTmemBufs; ++i) {
      mbar_init(&ctl->tfull[i], 1);
      mbar_init(&ctl->tempty[i], 4);
    }
    ctl->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&ctl->tmem_base, kTmemBufs * kChunk);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const int total_items = prefix[p.n];

  if (warp == 0) {
    // ================= TMA producer =================
    if (lane == 0) {
      tma_prefetch(&tm_cs);
      tma_prefetch(&tm_ab);
      tma_prefetch(&tm_codes);
      if (QUANT) tma_prefetch(&tm_scales);
      uint32_t it = 0, item_cnt = 0;
      for (int item = blockIdx.x; item < total_items && !*abort_flag; item += gridDim.x, ++item_cnt) {
        const int b = find_seq(prefix, p.n, item);
        const int rem = item - prefix[b];
        const int j = rem % p.group;
        const int tile = rem / p.group;
        int L = min(max(p.seq_lens[b], 0), p.max_seq_len);
        const int t0 = tile * kTile;
        int blk[8], slot[8];
        for (int pg = 0; pg < 8; ++pg) {
          const int t = t0 + 16 * pg;
          blk[pg] = 0;
          slot[pg] = 0;
          if (t < L) {
            const int col = t / p.block_size;
            int id = -1;
            if (col < p.max_blocks) id = p.block_table[(int64_t)b * p.bt_s0 + (int64_t)col * p.bt_s1];
            if (id < 0 || id >= p.num_blocks) {
              record_status(p.status, STARKV_EBOUNDS);
              id = 0;
            }
            blk[pg] = id;
            slot[pg] = t % p.block_size;
          }
        }
        // rotary table rows of this tile (+ the 3.2-bit scales of its tokens)
        if (!mbar_wait(&ctl->cs_empty, (item_cnt & 1) ^ 1, abort_flag, p.status)) break;
        mbar_arrive_expect_tx(&ctl->cs_full, kCsBytes);
        tma_load_2d(smem + LY::kOffCs, &tm_cs, &ctl->cs_full, 0, t0);
        tma_load_2d(smem + LY::kOffCs + kCsBytes / 2, &tm_cs, &ctl->cs_full, 64, t0);
        if (QUANT) {
          if (!mbar_wait(&ctl->sc_empty, (item_cnt & 1) ^ 1, abort_flag, p.status)) break;
          mbar_arrive_expect_tx(&ctl->sc_full, 8 * p.ks_boxes * 2048);
          for (int pg = 0; pg < 8; ++pg)
            for (int jb = 0; jb < p.ks_boxes; ++jb)
              tma_load_3d(smem + LY::kOffScales + (jb * 8 + pg) * 2048, &tm_scales, &ctl->sc_full,
                          p.ks_x0 + 128 * jb, slot[pg], blk[pg]);
        }
        const int ab_row0 = (b * p.group + j) * p.k_width;
        for (int c = 0; c < NC; ++c, ++it) {
          const int s = it % LY::kStages;
          if (!mbar_wait(&ctl->empty[s], ((it / LY::kStages) & 1) ^ 1, abort_flag, p.status)) break;
          uint8_t* st = smem + LY::kOffStages + s * LY::kStageBytes;
          mbar_arrive_expect_tx(&ctl->full[s], LY::kStageBytes);
          tma_load_2d(st, &tm_ab, &ctl->full[s], 0, ab_row0 + c * kChunk);
          tma_load_2d(st + kAbBytes / 2, &tm_ab, &ctl->full[s], 64, ab_row0 + c * kChunk);
          for (int pg = 0; pg < 8; ++pg)
            for (int i = 0; i < LY::kCodeBoxes; ++i) {
              const int x = QUANT ? c * 64 : c * kChunk + 64 * i;
              tma_load_3d(st + kAbBytes + (i * 8 + pg) * LY::kCodeBoxBytes, &tm_codes, &ctl->full[s], x,
                          slot[pg], blk[pg]);
            }
        }
      }
    }
  } else if (warp == 1) {
    // ================= MMA issuer =================
    if (lane == 0) {
      const uint32_t idesc = instr_desc_f16(/*f16*/ 0, 0, 0, kTile, kChunk);
      uint32_t it = 0, tb = 0, item_cnt = 0;
      const uint32_t cs_addr = smem_u32(smem + LY::kOffCs);
      for (int item = blockIdx.x; item < total_items && !*abort_flag; item += gridDim.x, ++item_cnt) {
        if (!mbar_wait(&ctl->cs_full, item_cnt & 1, abort_flag, p.status)) break;
        tc_fence_after();
        for (int c = 0; c < NC; ++c, ++it, ++tb) {
          const int s = it % LY::kStages;
          const int buf = tb % kTmemBufs;
          if (!mbar_wait(&ctl->full[s], (it / LY::kStages) & 1, abort_flag, p.status)) break;
          if (!mbar_wait(&ctl->tempty[buf], ((tb / kTmemBufs) & 1) ^ 1, abort_flag, p.status)) break;
          tc_fence_after();
          const uint32_t ab_addr = smem_u32(smem + LY::kOffStages + s * LY::kStageBytes);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t koff = (kk >> 2) * (kCsBytes / 2) + (kk & 3) * 32;
            const uint64_t da = smem_desc(cs_addr + koff, 16, 1024, kSwizzle128B);
            const uint64_t db = smem_desc(ab_addr + (kk >> 2) * (kAbBytes / 2) + (kk & 3) * 32, 16, 1024,
                                          kSwizzle128B);
            umma_f16(tmem + buf * kChunk, da, db, idesc, kk > 0);
          }
          umma_commit(&ctl->empty[s]);
          umma_commit(&ctl->tfull[buf]);
        }
        umma_commit(&ctl->cs_empty);
      }
    }
  } else {
    // ================= epilogue (warps 2..5) =================
    const int q = warp & 3;               // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;        // token within the tile
    const int e = warp - 2;               // 0..3, for the cross-warp reductions
    uint32_t it = 0, tb = 0, item_cnt = 0, epi_phase = 0;
    // Bounded barrier among the 128 epilogue threads (a plain bar.sync could
    // wait forever if another epilogue warp left on a timed-out pipeline wait).
    auto epi_sync = [&]() -> bool {
      mbar_arrive(&ctl->epi);
      return mbar_wait(&ctl->epi, (epi_phase++) & 1, abort_flag, p.status);
    };
    for (int item = blockIdx.x; item < total_items; item += gridDim.x, ++item_cnt) {
      if (*abort_flag) break;
      const int b = find_seq(prefix, p.n, item);
      const int rem = item - prefix[b];
      const int j = rem % p.group;
      const int tile = rem / p.group;
      const int L = min(max(p.seq_lens[b], 0), p.max_seq_len);
      const int t0 = tile * kTile;
      const int pg = row >> 4, sl = row & 15;
      if (QUANT && !mbar_wait(&ctl->sc_full, item_cnt & 1, abort_flag, p.status)) break;
      float acc = 0.f;
      bool ok = true;
      for (int c = 0; c < NC; ++c, ++it, ++tb) {
        const int s = it % LY::kStages;
        const int buf = tb % kTmemBufs;
        if (!mbar_wait(&ctl->tfull[buf], (tb / kTmemBufs) & 1, abort_flag, p.status) ||
            !mbar_wait(&ctl->full[s], (it / LY::kStages) & 1, abort_flag, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint8_t* codes = smem + LY::kOffStages + s * LY::kStageBytes + kAbBytes;
#pragma unroll 1
        for (int g = 0; g < kChunk / 32; ++g) {
          const int tau0 = (c * kChunk + 32 * g) >> 4;
          if (tau0 >= NT) break;
          float z[32];
          tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + buf * kChunk + 32 * g, z);
          float x[32];
          if (QUANT) {
            // 16 bytes = 32 nibbles of this token's lanes [32g, 32g+32) of the chunk
            const uint8_t* box = codes + pg * LY::kCodeBoxBytes;
            const int phys = g ^ ((sl >> 1) & 3);     // 64-byte swizzle
            uint4 u = *reinterpret_cast<const uint4*>(box + sl * 64 + phys * 16);
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int i = 0; i < 32; ++i) x[i] = (float)(int)((w[i >> 3] >> (4 * (i & 7))) & 15u) - 8.f;
          } else {
            const uint8_t* box = codes + ((g >> 1) * 8 + pg) * LY::kCodeBoxBytes;
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const int chunk16 = (g & 1) * 4 + v;
              const int phys = chunk16 ^ (sl & 7);      // 128-byte swizzle
              uint4 u = *reinterpret_cast<const uint4*>(box + sl * 128 + phys * 16);
              float f[8];
              if (p.cache_dtype == STARKV_BF16) bf16x8_to_f32(u, f); else f16x8_to_f32(u, f);
#pragma unroll
              for (int i = 0; i < 8; ++i) x[8 * v + i] = f[i];
            }
          }
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int tau = tau0 + hh;
            if (tau >= NT) break;
            const int meta = tiles[tau];
            if (meta < 0) continue;
            const int h = meta & 0xFFFF;
            float part = 0.f;
            if (QUANT) {
              // (outlier, inlier) bf16 scales of head h for this token
              const int off = p.ks_off + 4 * h - p.ks_x0;
              const int jb = off >> 7, within = off & 127;
              const uint8_t* sb = smem + LY::kOffScales + (jb * 8 + pg) * 2048 + sl * 128;
              const uint32_t sw = *reinterpret_cast<const uint32_t*>(
                  sb + ((((within >> 4) ^ (sl & 7)) << 4) | (within & 15)));
              const float so = __uint_as_float(sw << 16), si = __uint_as_float(sw & 0xFFFF0000u);
              const int nout = (meta >> 16) & 0xFF;
#pragma unroll
              for (int i = 0; i < 16; ++i) part += x[16 * hh + i] * (i < nout ? so : si) * z[16 * hh + i];
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i) part += x[16 * hh + i] * z[16 * hh + i];
            }
            acc += part;
            if (meta & (1 << 24)) {
              logits[h * (kTile + 1) + row] = acc;
              acc = 0.f;
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&ctl->tempty[buf]);
          mbar_arrive(&ctl->empty[s]);
        }
      }
      if (QUANT) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->sc_empty);
      }
      if (!ok || !epi_sync()) break;
      // ---- per-head tile softmax statistics ----
      for (int h = lane; h < H; h += 32) {
        float m = -INFINITY;
        for (int i = 0; i < 32; ++i) {
          const int t = 32 * e + i;
          if (t0 + t < L) m = fmaxf(m, logits[h * (kTile + 1) + t]);
        }
        red_m[e * H + h] = m;
      }
      if (!epi_sync()) break;
      for (int h = lane; h < H; h += 32) {
        const float m = fmaxf(fmaxf(red_m[h], red_m[H + h]), fmaxf(red_m[2 * H + h], red_m[3 * H + h]));
        const int hq = h * p.group + j;
        float ssum = 0.f;
        __align__(16) __half ev[32];
        for (int i = 0; i < 32; ++i) {
          const int t = 32 * e + i;
          float v = 0.f;
          if (t0 + t < L) v = __expf(logits[h * (kTile + 1) + t] - m);
          ssum += v;
          ev[i] = __float2half_rn(v);
        }
        uint4* dst = reinterpret_cast<uint4*>(p.e16 + ((int64_t)b * p.num_heads + hq) * p.l_pad + t0 + 32 * e);
#pragma unroll
        for (int v = 0; v < 4; ++v) dst[v] = reinterpret_cast<const uint4*>(ev)[v];
        red_l[e * H + h] = ssum;
      }
      if (!epi_sync()) break;
      if (e == 0) {
        for (int h = lane; h < H; h += 32) {
          const float m = fmaxf(fmaxf(red_m[h], red_m[H + h]), fmaxf(red_m[2 * H + h], red_m[3 * H + h]));
          const float l = red_l[h] + red_l[H + h] + red_l[2 * H + h] + red_l[3 * H + h];
          const int hq = h * p.group + j;
          const int64_t mi = ((int64_t)b * p.num_heads + hq) * p.n_tiles + tile;
          p.m_tile[mi] = m;
          p.l_tile[mi] = l;
          atomic_max_f32(p.m_seq + (int64_t)b * p.num_heads + hq, m);
        }
      }
      if (!epi_sync()) break;
    }
  }

  // ---- teardown ----
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemBufs * kChunk);
  }
}

int launch_scores(bool quant, const CUtensorMap& tm_cs, const CUtensorMap& tm_ab, const CUtensorMap& tm_codes,
                  const CUtensorMap& tm_scales, const ScoresParams& p, int num_sms, cudaStream_t stream) {
  const size_t smem = scores_smem_bytes(quant, p.num_kv_heads, p.n, p.k_width, quant ? p.ks_boxes : 0);
  if (smem > 227 * 1024) return STARKV_EINVAL;
  const void* fn = quant ? (const void*)scores_kernel<true> : (const void*)scores_kernel<false>;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return STARKV_ECUDA;
  const int grid = num_sms;
  if (quant)
    scores_kernel<true><<<grid, 192, smem, stream>>>(tm_cs, tm_ab, tm_codes, tm_scales, p);
  else
    scores_kernel<false><<<grid, 192, smem, stream>>>(tm_cs, tm_ab, tm_codes, tm_scales, p);
  return cudaGetLastError() == cudaSuccess ? STARKV_OK : STARKV_ECUDA;
}

}  // namespace starkv
