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
// [128 tokens x 128 lanes] x K=128 contraction per chunk of lanes: it runs on
// the tcgen05 tensor core (M=128 tokens, N=128 lanes, K=128, f16 in, f32 out in
// TMEM). The codes x are only used elementwise in the epilogue, so the 4-bit
// cache is dequantized in registers ((n - 8) * bf16 scale, bit-exact) and never
// has to be laid out as an MMA operand.
//
// Per tile (one sequence, 128 tokens) the epilogue reduces each head's logits
// to (tile max m, tile sum l = sum exp(logit - m)) and stores exp(logit - m) as
// f16 ("e16"); the P.V kernel rescales by exp(m - M) with M the sequence max.
//
// Persistent CTAs (one per SM), warp roles:
//   warp 0      TMA producer: rotary rows, AB chunks (2-slot ring, from L2),
//               code pages (3-4 slot ring, from HBM) gathered through the block table;
//   warp 1      MMA issuer, owns the TMEM allocation (4 z buffers x 128 columns);
//   warps 2-17  epilogue: thread = token row (TMEM lane) x 32-column group of the
//               chunk; per-head partial sums are merged with shared-memory atomics.
#include "starkv_common.cuh"
#include "starkv_kernels.h"

namespace starkv {

namespace {

constexpr int kTile = 128;       // tokens per tile (MMA M)
constexpr int kChunk = 128;      // lanes per chunk (MMA N)
constexpr int kTmemBufs = 4;
constexpr int kAbSlots = 2;
// Epilogue shape. 3.2-bit codes cost more ALU work per lane (nibble decode and a
// separate outlier sum) and need more warps to hide latency; bf16 codes are
// limited by the copy pipeline and do best with fewer, wider threads.
template <bool QUANT>
struct Epi {
  static constexpr int kWarps = QUANT ? 16 : 8;
  static constexpr int kGroups = kWarps / 4;            // column groups per chunk
  static constexpr int kSub = kChunk / kGroups / 32;     // 32-column TMEM loads per thread and chunk
  static constexpr int kThreads = 64 + 32 * kWarps;
  static constexpr int kTokPerWarp = kTile / kWarps;     // tokens per warp in the statistics phase
  static_assert(kTokPerWarp % 8 == 0, "statistics phase stores whole 16-byte groups of f16");
};
constexpr int kMaxEpiWarps = 16;
constexpr int kCsBytes = kTile * 128 * 2;       // f16 [128 tokens][128]
constexpr int kAbBytes = kChunk * 128 * 2;      // f16 [128 lanes][128]
constexpr int kMaxCodeSlots = 4;

template <bool QUANT>
struct Layout {
  // bf16 codes: 2 boxes of 64 lanes (128 B) per page; 3.2-bit codes: one box of
  // 64 bytes (128 lanes) per page.
  static constexpr int kCodeSlots = QUANT ? 4 : 3;
  static constexpr int kCodeBoxes = QUANT ? 1 : 2;
  static constexpr int kCodeBoxBytes = QUANT ? 16 * 64 : 16 * 128;
  static constexpr int kCodeBytes = 8 * kCodeBoxes * kCodeBoxBytes;   // per slot (8 pages)
  static constexpr int kOffCs = 0;
  static constexpr int kOffAb = kOffCs + kCsBytes;
  static constexpr int kOffCodes = kOffAb + kAbSlots * kAbBytes;
  static constexpr int kOffScales = kOffCodes + kCodeSlots * kCodeBytes;   // 3.2-bit scale boxes
  static __host__ __device__ int off_logits(int ks_boxes) { return kOffScales + ks_boxes * 8 * 2048; }
};

struct SharedCtl {
  uint64_t ab_full[kAbSlots], ab_empty[kAbSlots];
  uint64_t code_full[kMaxCodeSlots], code_empty[kMaxCodeSlots];
  uint64_t cs_full, cs_empty, sc_full, sc_empty;
  uint64_t tfull[kTmemBufs], tempty[kTmemBufs];
  uint64_t epi;            // bounded barrier among the epilogue warps
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
  bytes += (size_t)num_kv_heads * (kTile + 1) * 4;            // logits [H][129]
  bytes += (size_t)2 * kMaxEpiWarps * num_kv_heads * 4;       // cross-warp max / sum
  bytes += 16 + (size_t)(nt + 7) / 8 * 8 * 4;                // lane-tile table, padded to whole chunks
  bytes += (size_t)(n + 1) * 4;                               // tile prefix over sequences
  bytes = (bytes + 15) & ~size_t(15);
  bytes += sizeof(SharedCtl) + 1024;                          // control + alignment slack
  return bytes;
}

template <bool QUANT, bool F16>
__global__ void __launch_bounds__(Epi<QUANT>::kThreads, 1)
scores_kernel(const __grid_constant__ CUtensorMap tm_cs, const __grid_constant__ CUtensorMap tm_ab,
              const __grid_constant__ CUtensorMap tm_codes, const __grid_constant__ CUtensorMap tm_scales,
              const ScoresParams p) {
  using LY = Layout<QUANT>;
  using EP = Epi<QUANT>;
  constexpr int kEpiWarps = EP::kWarps;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int H = p.num_kv_heads;
  const int NT = p.k_width / 16;
  const int NC = (p.k_width + kChunk - 1) / kChunk;
  const int ks_boxes = QUANT ? p.ks_boxes : 0;
  float* logits = reinterpret_cast<float*>(smem + LY::off_logits(ks_boxes));   // [H][129]
  float* red_m = logits + H * (kTile + 1);                                      // [8][H]
  float* red_l = red_m + kEpiWarps * H;                                         // [8][H]
  int* tiles = reinterpret_cast<int*>((reinterpret_cast<uintptr_t>(red_l + kEpiWarps * H) + 15) &
                                      ~uintptr_t(15));                          // [NC * 8], -1 past NT
  int* prefix = tiles + NC * 8;                                                 // [n+1]
  SharedCtl* ctl =
      reinterpret_cast<SharedCtl*>((reinterpret_cast<uintptr_t>(prefix + p.n + 1) + 15) & ~uintptr_t(15));
  volatile int* abort_flag = &ctl->abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---- prologue: tables, zeroed logits, barriers, TMEM ----
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int b = 0; b < p.n; ++b) {
      prefix[b] = acc;
      const int L = min(max(p.seq_lens[b], 0), p.max_seq_len);
      acc += (L + kTile - 1) / kTile * p.group;
    }
    prefix[p.n] = acc;
  }
  for (int t = threadIdx.x; t < NC * 8; t += blockDim.x) {
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
  for (int i = threadIdx.x; i < H * (kTile + 1); i += blockDim.x) logits[i] = 0.f;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kAbSlots; ++s) {
      mbar_init(&ctl->ab_full[s], 1);
      mbar_init(&ctl->ab_empty[s], 1);
    }
    for (int s = 0; s < LY::kCodeSlots; ++s) {
      mbar_init(&ctl->code_full[s], 1);
      mbar_init(&ctl->code_empty[s], kEpiWarps);
    }
    mbar_init(&ctl->cs_full, 1);
    mbar_init(&ctl->cs_empty, 1);
    mbar_init(&ctl->sc_full, 1);
    mbar_init(&ctl->sc_empty, kEpiWarps);
    for (int i = 0; i < kTmemBufs; ++i) {
      mbar_init(&ctl->tfull[i], 1);
      mbar_init(&ctl->tempty[i], kEpiWarps);
    }
    mbar_init(&ctl->epi, 32 * kEpiWarps);
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
    // Lanes 0-7 fetch the 8 block ids of the NEXT tile while lane 0 issues the
    // current tile's copies, so the block table's latency stays off the issue path.
    if (lane == 0) {
      tma_prefetch(&tm_cs);
      tma_prefetch(&tm_ab);
      tma_prefetch(&tm_codes);
      if (QUANT) tma_prefetch(&tm_scales);
    }
    auto block_of = [&](int item) -> int {   // block id of page `lane` of an item (lanes 0-7)
      if (item >= total_items || lane >= 8) return 0;
      const int b = find_seq(prefix, p.n, item);
      const int tile = (item - prefix[b]) / p.group;
      const int L = min(max(p.seq_lens[b], 0), p.max_seq_len);
      const int t = tile * kTile + 16 * lane;
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
    uint32_t ab_it = 0, code_it = 0, item_cnt = 0;
    int ids_next = block_of(blockIdx.x);
    for (int item = blockIdx.x; item < total_items; item += gridDim.x, ++item_cnt) {
      const int ids = ids_next;
      ids_next = block_of(item + gridDim.x);
      int blk[8], slot[8];
#pragma unroll
      for (int pg = 0; pg < 8; ++pg) blk[pg] = __shfl_sync(0xffffffffu, ids, pg);
      int ok = 1;
      if (lane == 0) {
        const int b = find_seq(prefix, p.n, item);
        const int rem = item - prefix[b];
        const int j = rem % p.group;
        const int tile = rem / p.group;
        const int t0 = tile * kTile;
#pragma unroll
        for (int pg = 0; pg < 8; ++pg) slot[pg] = (t0 + 16 * pg) % p.block_size;
        // rotary table rows of this tile (+ the 3.2-bit scales of its tokens)
        ok = !*abort_flag && mbar_wait(&ctl->cs_empty, (item_cnt & 1) ^ 1, abort_flag, p.status);
        if (ok) {
          mbar_arrive_expect_tx(&ctl->cs_full, kCsBytes);
          tma_load_2d(smem + LY::kOffCs, &tm_cs, &ctl->cs_full, 0, t0);
          tma_load_2d(smem + LY::kOffCs + kCsBytes / 2, &tm_cs, &ctl->cs_full, 64, t0);
        }
        if (ok && QUANT) {
          ok = mbar_wait(&ctl->sc_empty, (item_cnt & 1) ^ 1, abort_flag, p.status);
          if (ok) {
            mbar_arrive_expect_tx(&ctl->sc_full, 8 * p.ks_boxes * 2048);
            for (int pg = 0; pg < 8; ++pg)
              for (int jb = 0; jb < p.ks_boxes; ++jb)
                tma_load_3d(smem + LY::kOffScales + (jb * 8 + pg) * 2048, &tm_scales, &ctl->sc_full,
                            p.ks_x0 + 128 * jb, slot[pg], blk[pg]);
          }
        }
        const int ab_row0 = (b * p.group + j) * p.k_width;
        for (int c = 0; ok && c < NC; ++c, ++ab_it, ++code_it) {
          const int sa = ab_it % kAbSlots;
          if (!mbar_wait(&ctl->ab_empty[sa], ((ab_it / kAbSlots) & 1) ^ 1, abort_flag, p.status)) {
            ok = 0;
            break;
          }
          uint8_t* abs = smem + LY::kOffAb + sa * kAbBytes;
          mbar_arrive_expect_tx(&ctl->ab_full[sa], kAbBytes);
          tma_load_2d(abs, &tm_ab, &ctl->ab_full[sa], 0, ab_row0 + c * kChunk);
          tma_load_2d(abs + kAbBytes / 2, &tm_ab, &ctl->ab_full[sa], 64, ab_row0 + c * kChunk);
          const int sc = code_it % LY::kCodeSlots;
          if (!mbar_wait(&ctl->code_empty[sc], ((code_it / LY::kCodeSlots) & 1) ^ 1, abort_flag, p.status)) {
            ok = 0;
            break;
          }
          uint8_t* cds = smem + LY::kOffCodes + sc * LY::kCodeBytes;
          mbar_arrive_expect_tx(&ctl->code_full[sc], LY::kCodeBytes);
#pragma unroll
          for (int pg = 0; pg < 8; ++pg)
#pragma unroll
            for (int i = 0; i < LY::kCodeBoxes; ++i) {
              const int x = QUANT ? c * 64 : c * kChunk + 64 * i;
              tma_load_3d(cds + (i * 8 + pg) * LY::kCodeBoxBytes, &tm_codes, &ctl->code_full[sc], x, slot[pg],
                          blk[pg]);
            }
        }
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
    }
  } else if (warp == 1) {
    // ================= MMA issuer =================
    if (lane == 0) {
      const uint32_t idesc = instr_desc_f16(/*f16*/ 0, 0, 0, kTile, kChunk);
      uint32_t ab_it = 0, tb = 0, item_cnt = 0;
      const uint32_t cs_addr = smem_u32(smem + LY::kOffCs);
      for (int item = blockIdx.x; item < total_items && !*abort_flag; item += gridDim.x, ++item_cnt) {
        if (!mbar_wait(&ctl->cs_full, item_cnt & 1, abort_flag, p.status)) break;
        tc_fence_after();
        for (int c = 0; c < NC; ++c, ++ab_it, ++tb) {
          const int sa = ab_it % kAbSlots;
          const int buf = tb % kTmemBufs;
          if (!mbar_wait(&ctl->ab_full[sa], (ab_it / kAbSlots) & 1, abort_flag, p.status)) break;
          if (!mbar_wait(&ctl->tempty[buf], ((tb / kTmemBufs) & 1) ^ 1, abort_flag, p.status)) break;
          tc_fence_after();
          const uint32_t ab_addr = smem_u32(smem + LY::kOffAb + sa * kAbBytes);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t da = smem_desc(cs_addr + (kk >> 2) * (kCsBytes / 2) + (kk & 3) * 32, 16, 1024,
                                          kSwizzle128B);
            const uint64_t db = smem_desc(ab_addr + (kk >> 2) * (kAbBytes / 2) + (kk & 3) * 32, 16, 1024,
                                          kSwizzle128B);
            umma_f16(tmem + buf * kChunk, da, db, idesc, kk > 0);
          }
          umma_commit(&ctl->ab_empty[sa]);
          umma_commit(&ctl->tfull[buf]);
        }
        umma_commit(&ctl->cs_empty);
      }
    }
  } else {
    // ================= epilogue (warps 2 .. 2 + kEpiWarps) =================
    // Thread = (token row of the tile, column group of the chunk): warp w may only
    // read TMEM lanes 32 (w % 4) .. +32, so the warps cover the 4 lane quarters x
    // kGroups column groups of kSub x 32 columns.
    const int ew = warp - 2;              // 0..kEpiWarps-1
    const int q = warp & 3;               // TMEM lane quarter this warp may access
    const int gq = ew >> 2;               // column group: chunk columns [32 kSub gq, 32 kSub (gq + 1))
    const int row = q * 32 + lane;        // token within the tile
    const int pg = row >> 4, sl = row & 15;
    uint32_t code_it = 0, tb = 0, item_cnt = 0, epi_phase = 0;
    // Bounded barrier among the epilogue threads (a plain bar.sync could wait
    // forever if another epilogue warp left on a timed-out pipeline wait).
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
      if (QUANT && !mbar_wait(&ctl->sc_full, item_cnt & 1, abort_flag, p.status)) break;
      // running sums of the current head: 4 independent chains over all of its
      // lanes (ai); 3.2-bit codes also sum the outlier lanes apart (ao), so the
      // flush applies logit = s_in * ai + (s_out - s_in) * ao.
      float2 ai[4], ao[2];
#pragma unroll
      for (int i = 0; i < 4; ++i) ai[i] = make_float2(0.f, 0.f);
      ao[0] = ao[1] = make_float2(0.f, 0.f);
      int cur_h = -1;
      auto flush = [&]() {
        const float all = ((ai[0].x + ai[0].y) + (ai[1].x + ai[1].y)) + ((ai[2].x + ai[2].y) + (ai[3].x + ai[3].y));
        float v;
        if (QUANT) {
          // (outlier, inlier) bf16 scales of head cur_h for this token
          const int off = p.ks_off + 4 * cur_h - p.ks_x0;
          const int jb = off >> 7, within = off & 127;
          const uint8_t* sb = smem + LY::kOffScales + (jb * 8 + pg) * 2048 + sl * 128;
          const uint32_t sw =
              *reinterpret_cast<const uint32_t*>(sb + ((((within >> 4) ^ (sl & 7)) << 4) | (within & 15)));
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
      for (int c = 0; c < NC; ++c, ++code_it, ++tb) {
        const int sc = code_it % LY::kCodeSlots;
        const int buf = tb % kTmemBufs;
        if (!mbar_wait(&ctl->tfull[buf], (tb / kTmemBufs) & 1, abort_flag, p.status) ||
            !mbar_wait(&ctl->code_full[sc], (code_it / LY::kCodeSlots) & 1, abort_flag, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t zr[EP::kSub][32];
        const int nsub = min(EP::kSub, max(0, (NT * 16 - c * kChunk - 32 * EP::kSub * gq + 31) / 32));   // warp-uniform
#pragma unroll
        for (int sb = 0; sb < EP::kSub; ++sb)
          if (sb < nsub)
            tmem_ld32_issue(tmem + ((uint32_t)(q * 32) << 16) + buf * kChunk + 32 * (EP::kSub * gq + sb), zr[sb]);
#pragma unroll
        for (int sb = 0; sb < EP::kSub; ++sb) {
          if (sb >= nsub) break;
          const int g = EP::kSub * gq + sb;     // 32-lane group of the chunk
          const uint8_t* codes = smem + LY::kOffCodes + sc * LY::kCodeBytes;
          // this token's codes of the group's 32 lanes
          constexpr int kWords = QUANT ? 4 : 16;
          uint32_t w[kWords];
          if (QUANT) {
            const uint8_t* box = codes + pg * LY::kCodeBoxBytes;
            const int phys = g ^ ((sl >> 1) & 3);     // 64-byte swizzle
            const uint4 u = *reinterpret_cast<const uint4*>(box + sl * 64 + phys * 16);
            w[0] = u.x; w[1] = u.y; w[2] = u.z; w[3] = u.w;
          } else {
            const uint8_t* box = codes + ((g >> 1) * 8 + pg) * LY::kCodeBoxBytes;
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const int phys = ((g & 1) * 4 + v) ^ (sl & 7);   // 128-byte swizzle
              const uint4 u = *reinterpret_cast<const uint4*>(box + sl * 128 + phys * 16);
              w[4 * v] = u.x; w[4 * v + 1] = u.y; w[4 * v + 2] = u.z; w[4 * v + 3] = u.w;
            }
          }
          const int2 m2 = reinterpret_cast<const int2*>(tiles)[c * 4 + g];   // metadata of the 2 lane tiles
          tmem_wait(zr[sb]);   // the first waits for all loads; each names its own registers
          const uint32_t* z = zr[sb];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int meta = hh == 0 ? m2.x : m2.y;
            if (meta < 0) continue;
            const int h = meta & 0xFFFF;
            if (h != cur_h) {
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
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&ctl->tempty[buf]);
          mbar_arrive(&ctl->code_empty[sc]);
        }
      }
      if (cur_h >= 0) flush();
      if (QUANT) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->sc_empty);
      }
      if (!ok || !epi_sync()) break;
      // ---- per-head tile softmax statistics: warp ew owns kTokPerWarp tokens ----
      constexpr int kTokPerWarp = EP::kTokPerWarp;
      for (int h = lane; h < H; h += 32) {
        float m = -INFINITY;
#pragma unroll
        for (int i = 0; i < kTokPerWarp; ++i) {
          const int t = kTokPerWarp * ew + i;
          if (t0 + t < L) m = fmaxf(m, logits[h * (kTile + 1) + t]);
        }
        red_m[ew * H + h] = m;
      }
      if (!epi_sync()) break;
      for (int h = lane; h < H; h += 32) {
        float m = red_m[h];
        for (int w2 = 1; w2 < kEpiWarps; ++w2) m = fmaxf(m, red_m[w2 * H + h]);
        const int hq = h * p.group + j;
        float ssum = 0.f;
        __align__(16) __half ev[kTokPerWarp];
#pragma unroll
        for (int i = 0; i < kTokPerWarp; ++i) {
          const int t = kTokPerWarp * ew + i;
          float v = 0.f;
          if (t0 + t < L) v = __expf(logits[h * (kTile + 1) + t] - m);
          ssum += v;
          ev[i] = __float2half_rn(v);
        }
        uint4* dst = reinterpret_cast<uint4*>(p.e16 + ((int64_t)b * p.num_heads + hq) * p.l_pad + t0 + kTokPerWarp * ew);
#pragma unroll
        for (int i = 0; i < kTokPerWarp / 8; ++i) dst[i] = reinterpret_cast<const uint4*>(ev)[i];
        red_l[ew * H + h] = ssum;
      }
      if (!epi_sync()) break;
      if (ew == 0) {
        for (int h = lane; h < H; h += 32) {
          float m = red_m[h], l = red_l[h];
          for (int w2 = 1; w2 < kEpiWarps; ++w2) {
            m = fmaxf(m, red_m[w2 * H + h]);
            l += red_l[w2 * H + h];
          }
          const int hq = h * p.group + j;
          const int64_t mi = ((int64_t)b * p.num_heads + hq) * p.n_tiles + tile;
          p.m_tile[mi] = m;
          (void)l;
          atomic_max_f32(p.m_seq + (int64_t)b * p.num_heads + hq, m);
        }
      }
      // clear the logits for the next tile's atomic flushes
      for (int i = threadIdx.x - 64; i < H * (kTile + 1); i += 32 * kEpiWarps) logits[i] = 0.f;
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
  const bool f16 = p.cache_dtype == STARKV_F16;
  const void* fn = quant ? (const void*)scores_kernel<true, false>
                         : (f16 ? (const void*)scores_kernel<false, true> : (const void*)scores_kernel<false, false>);
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return STARKV_ECUDA;
  const int grid = num_sms;
  if (quant)
    scores_kernel<true, false><<<grid, Epi<true>::kThreads, smem, stream>>>(tm_cs, tm_ab, tm_codes, tm_scales, p);
  else if (f16)
    scores_kernel<false, true><<<grid, Epi<false>::kThreads, smem, stream>>>(tm_cs, tm_ab, tm_codes, tm_scales, p);
  else
    scores_kernel<false, false><<<grid, Epi<false>::kThreads, smem, stream>>>(tm_cs, tm_ab, tm_codes, tm_scales, p);
  return cudaGetLastError() == cudaSuccess ? STARKV_OK : STARKV_ECUDA;
}

}  // namespace starkv
