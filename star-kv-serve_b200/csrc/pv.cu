// V side of the paged decode: pv[b, h, c] = sum_t p[b, h, t] * V[b, t, c]
// (unnormalised; the lift divides by the softmax denominator).
//
// Replaces paged_decode.py:105-147 + :220 (_paged_pv_fwd and the segment sum)
// and paged_quant.py:311-354 (_paged_pv_fold).
//
// V is one latent shared by every head (checkpoint.py:140-153), so one CTA owns
// all heads of a token range and reads each V code once. The contraction runs on
// tcgen05 in swap-AB form, D[c, h] += V^T[c, t] . P^T[t, h]: M = 128 code
// channels, N = heads (rounded to 16), K = 16 tokens (one page) per instruction,
// f32 accumulators in TMEM across the whole token range.
//   bf16 codes: A = V^T straight from the TMA page tile (MN-major, 128 B swizzle).
//   3.2-bit codes: worker warps turn each nibble n into the exact f16 n - 8 (even
//   channels) or 16 (n - 8) (odd channels): one bit operation per channel pair
//   makes 1024 + n or 1024 + 16 n, one f16 subtraction removes the bias exactly;
//   the flush scales odd-channel rows by 1/16. The per-token scale folds into P
//   (one P per outlier / inlier block, as paged_quant.py:320-346 does), so A
//   stays exact.
// P = e16 * exp(m_tile - m_seq) is built per page by the worker warps.
//
// Work split: the pages of all sequences are concatenated and cut into equal
// contiguous ranges, one per CTA (x the channel ranges when the accumulator of
// all channels does not fit TMEM), so every CTA streams the same number of bytes
// whatever the length mix. A CTA range crossing a sequence boundary flushes its
// accumulator with f32 atomics into the small L2-resident pv buffer.
//
// Warps: 0 TMA producer, 1 MMA issuer + TMEM owner, 2-13 workers (P, dequant,
// accumulator flush; the three warps of a TMEM lane quarter split the M-tiles).
#include "pv_common.cuh"
#include "starkv_common.cuh"
#include "starkv_kernels.h"

namespace starkv {

using namespace pvc;

namespace {

constexpr int kMaxStages = 4;
constexpr int kWorkers = 12;                 // worker warps (3 per TMEM lane quarter)
constexpr int kWorkerThreads = 32 * kWorkers;
constexpr int kPvThreads = 64 + kWorkerThreads;

struct PvCtl {
  uint64_t vfull[kMaxStages], vempty[kMaxStages];
  uint64_t pfull[kMaxStages], pempty[kMaxStages];
  uint64_t accfull, accempty;
  uint32_t tmem_base;
  int abort_flag;
};

struct PvLayout {
  int v_bytes;      // TMA tile bytes per stage
  int a_bytes;      // dequantized A tiles per stage (3.2-bit)
  int e_bytes;      // TMA tile of e16 (heads x 16 tokens) per stage
  int p_bytes;      // P operand(s) per stage
  int stage_bytes;  // all of the above, 1024-aligned
  int stages;
  int total;        // dynamic smem (+ control)
};

__host__ __device__ inline PvLayout pv_layout(bool quant, const PvParams& p) {
  PvLayout L;
  L.v_bytes = quant ? p.v_boxes * 2048 : p.mt_per_range * 4096;
  L.a_bytes = quant ? p.mt_per_range * 4096 : 0;
  L.e_bytes = (p.num_heads * 32 + 127) & ~127;
  L.p_bytes = (quant ? 2 : 1) * p.nh * 32;
  L.stage_bytes = (L.v_bytes + L.a_bytes + L.e_bytes + L.p_bytes + 1023) & ~1023;
  int s = (200 * 1024) / L.stage_bytes;
  L.stages = s > kMaxStages ? kMaxStages : s;
  L.total = L.stages * L.stage_bytes + (int)sizeof(PvCtl) + 1024 + 64;
  return L;
}

}  // namespace

size_t pv_smem_bytes(bool quant, const PvParams& p) {
  return (size_t)pv_layout(quant, p).total + (size_t)(2 * p.n + 1) * 4;
}

template <bool QUANT>
__global__ void __launch_bounds__(kPvThreads, 1) pv_kernel(const __grid_constant__ CUtensorMap tm_v,
                                                    const __grid_constant__ CUtensorMap tm_e, const PvParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const PvLayout LY = pv_layout(QUANT, p);
  PvCtl* ctl = reinterpret_cast<PvCtl*>(smem + LY.stages * LY.stage_bytes);
  int* pprefix = reinterpret_cast<int*>(ctl + 1);   // [n+1] page prefix over this rank's pages
  int* pbeg = pprefix + p.n + 1;                     // [n] first page of this rank in each sequence
  volatile int* abort_flag = &ctl->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = LY.stages;

  if (threadIdx.x == 0) {
    pvc::page_ranges(p, pprefix, pbeg);
    for (int s = 0; s < S; ++s) {
      mbar_init(&ctl->vfull[s], 1);
      mbar_init(&ctl->vempty[s], QUANT ? kWorkers : 1);
      mbar_init(&ctl->pfull[s], kWorkers);
      mbar_init(&ctl->pempty[s], 1);
    }
    mbar_init(&ctl->accfull, 1);
    mbar_init(&ctl->accempty, kWorkers);
    ctl->abort_flag = 0;
    fence_barrier_init();
  }
  uint32_t tmem_cols = 32;
  while (tmem_cols < (uint32_t)(p.mt_per_range * p.nh)) tmem_cols <<= 1;
  if (warp == 1) tmem_alloc(&ctl->tmem_base, tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const int total_pages = pprefix[p.n];
  const long long units = (long long)p.n_ranges * total_pages;
  const int u_begin = (int)(units * blockIdx.x / gridDim.x);
  const int u_end = (int)(units * (blockIdx.x + 1) / gridDim.x);

  if (warp == 0) {
    // ================= TMA producer =================
    // All 32 lanes fetch block-table entries (32 pages per batch, one batch
    // ahead, so the table's latency is never on the issue path); lane 0 issues
    // the copies.
    if (lane == 0) {
      tma_prefetch(&tm_v);
      tma_prefetch(&tm_e);
    }
    const int e_bytes = p.num_heads * 32;
    auto block_of = [&](int b, int page, int npages_end) -> int {
      if (page >= npages_end) return 0;
      const int col = (page * 16) / p.block_size;
      int blk = -1;
      if (col < p.max_blocks) blk = p.block_table[(int64_t)b * p.bt_s0 + (int64_t)col * p.bt_s1];
      if (blk < 0 || blk >= p.num_blocks) {
        record_status(p.status, STARKV_EBOUNDS);
        blk = 0;
      }
      return blk;
    };
    uint32_t it = 0;
    int u = u_begin;
    SubItem si;
    bool stop = false;
    while (!stop && next_sub(u, u_end, total_pages, pprefix, pbeg, p.n, si)) {
      const int mt0 = si.range * p.mt_per_range;
      const int mt1 = min(mt0 + p.mt_per_range, p.n_mtiles);
      const int pend = si.page0 + si.npages;
      int ids_cur = block_of(si.b, si.page0 + lane, pend);
      int ids_nxt = block_of(si.b, si.page0 + 32 + lane, pend);
      for (int pg = 0; pg < si.npages; ++pg, ++it) {
        if (pg > 0 && (pg & 31) == 0) {
          ids_cur = ids_nxt;
          ids_nxt = block_of(si.b, si.page0 + pg + 32 + lane, pend);
        }
        const int blk = __shfl_sync(0xffffffffu, ids_cur, pg & 31);
        int ok = 1;
        if (lane == 0) {
          const int s = it % S;
          ok = mbar_wait(&ctl->vempty[s], ((it / S) & 1) ^ 1, abort_flag, p.status) ? 1 : 0;
          if (ok) {
            const int t = (si.page0 + pg) * 16;
            const int slot = t % p.block_size;
            uint8_t* st = smem + s * LY.stage_bytes;
            if (QUANT) {
              mbar_arrive_expect_tx(&ctl->vfull[s], p.v_boxes * 2048 + e_bytes);
              for (int jb = 0; jb < p.v_boxes; ++jb)
                tma_load_3d(st + jb * 2048, &tm_v, &ctl->vfull[s], p.vx0 + 128 * jb, slot, blk);
            } else {
              mbar_arrive_expect_tx(&ctl->vfull[s], (mt1 - mt0) * 4096 + e_bytes);
              for (int m = mt0; m < mt1; ++m)
                for (int i = 0; i < 2; ++i)
                  tma_load_3d(st + (m - mt0) * 4096 + i * 2048, &tm_v, &ctl->vfull[s], p.k_width + m * 128 + 64 * i,
                              slot, blk);
            }
            // e16 rows of this sequence's heads for the page's 16 tokens
            tma_load_2d(st + LY.v_bytes + LY.a_bytes, &tm_e, &ctl->vfull[s], t, si.b * p.num_heads);
          }
        }
        if (!__shfl_sync(0xffffffffu, ok, 0)) {
          stop = true;
          break;
        }
      }
    }
  } else if (warp == 1) {
    // ================= MMA issuer =================
    if (lane == 0) {
      const uint32_t fmt = QUANT ? 0u : (p.cache_dtype == STARKV_BF16 ? 1u : 0u);
      const uint32_t idesc = instr_desc_f16(fmt, /*A MN-major*/ 1, /*B K-major*/ 0, 128, p.nh);
      uint32_t it = 0, acc_cnt = 0;
      int u = u_begin;
      SubItem si;
      while (!*abort_flag && next_sub(u, u_end, total_pages, pprefix, pbeg, p.n, si)) {
        const int mt0 = si.range * p.mt_per_range;
        const int nmt = min(mt0 + p.mt_per_range, p.n_mtiles) - mt0;
        if (!mbar_wait(&ctl->accempty, (acc_cnt & 1) ^ 1, abort_flag, p.status)) break;
        tc_fence_after();
        for (int pg = 0; pg < si.npages; ++pg, ++it) {
          const int s = it % S;
          if (!QUANT && !mbar_wait(&ctl->vfull[s], (it / S) & 1, abort_flag, p.status)) break;
          if (!mbar_wait(&ctl->pfull[s], (it / S) & 1, abort_flag, p.status)) break;
          tc_fence_after();
          const uint32_t st = smem_u32(smem + s * LY.stage_bytes);
          const uint32_t pbase = st + LY.v_bytes + LY.a_bytes + LY.e_bytes;
          for (int m = 0; m < nmt; ++m) {
            uint64_t da, db;
            if (QUANT) {
              da = smem_desc(st + LY.v_bytes + m * 4096, 2048, 128, kSwizzleNone);
              const int blk = (mt0 + m) < p.t_out ? 0 : 1;
              db = smem_desc(pbase + blk * p.nh * 32, 128, 256, kSwizzleNone);
            } else {
              da = smem_desc(st + m * 4096, 2048, 1024, kSwizzle128B);
              db = smem_desc(pbase, 128, 256, kSwizzleNone);
            }
            umma_f16(tmem + m * p.nh, da, db, idesc, pg > 0);
          }
          if (!QUANT) umma_commit(&ctl->vempty[s]);
          umma_commit(&ctl->pempty[s]);
        }
        umma_commit(&ctl->accfull);
        ++acc_cnt;
      }
    }
  } else {
    // ================= workers: P (+ dequant), accumulator flush =================
    const int wt = threadIdx.x - 64;     // 0..kWorkerThreads-1
    const int q = warp & 3;
    const int wpair = (warp - 2) >> 2;   // which of the kWorkers / 4 warps of lane quarter q
    // P tasks (head, 4 tokens) start at the threads with the fewest dequant tasks: the
    // last 128 worker threads take P tasks 0..127 (the 4 threads of a head stay in
    // adjacent lanes)
    const int pw = (wt + 128) % kWorkerThreads;
    uint32_t it = 0, acc_cnt = 0;
    int u = u_begin;
    SubItem si;
    bool ok = true;
    while (ok && !*abort_flag && next_sub(u, u_end, total_pages, pprefix, pbeg, p.n, si)) {
      const int b = si.b;
      const int L = min(max(p.seq_lens[b], 0), p.max_seq_len);
      const int mt0 = si.range * p.mt_per_range;
      const int nmt = min(mt0 + p.mt_per_range, p.n_mtiles) - mt0;
      const float* mtb = p.m_tile + (int64_t)b * p.num_heads * p.n_tiles;
      const float* msb = p.m_seq + (int64_t)b * p.num_heads;
      float lsum[4] = {0.f, 0.f, 0.f, 0.f};   // sum of P of this thread's (head, 4-token) tasks
      // 3.2-bit dequant tasks of this thread (the same on every page): (M-tile, token,
      // 16-byte window = 32 channels) -> the two aligned staged chunks it spans, the
      // byte shift that cuts the window out of them, and its A-tile destination
      constexpr int kMaxDq = 3;
      int dq_src0[kMaxDq], dq_src1[kMaxDq], dq_dst[kMaxDq], dq_sh[kMaxDq];
      int ndq = 0;
      if (QUANT) {
        const int nvq = p.v_boxes * 8 - 1;    // last staged 16-byte chunk index
#pragma unroll
        for (int i = 0; i < kMaxDq; ++i) {
          const int task = wt + kWorkerThreads * i;
          dq_src0[i] = dq_src1[i] = dq_dst[i] = dq_sh[i] = 0;
          if (task >= nmt * 64) continue;
          ndq = i + 1;
          const int m = task >> 6, tt = task & 63;
          const int k = tt & 15, j = tt >> 4;
          const int gm = mt0 + m;
          const bool outl = gm < p.t_out;
          const int jt = outl ? gm : gm - p.t_out;
          const int bb = (outl ? p.vq_off : p.vq_off + p.v_nbo) - p.vx0;   // block start in the staged row
          const int win = bb + 64 * jt + 16 * j;
          const int c0 = min(win >> 4, nvq), c1 = min((win >> 4) + 1, nvq);
          dq_src0[i] = k * 128 + (c0 >> 3) * 2048 + (((c0 & 7) ^ (k & 7)) << 4);
          dq_src1[i] = k * 128 + (c1 >> 3) * 2048 + (((c1 & 7) ^ (k & 7)) << 4);
          dq_dst[i] = LY.v_bytes + m * 4096 + (k >> 3) * 2048 + (4 * j) * 128 + (k & 7) * 16;
          dq_sh[i] = (bb & 15) * 8;   // bit offset of the window inside the 32 staged bytes
        }
      }
      // P = e16 * exp(m_tile - m_seq): the factor of the current 128-token tile (8 pages),
      // and the next tile's max loaded as soon as the current tile starts, so its
      // latency is covered by 8 pages of work
      int cur_tile = (si.page0 * 16) >> 7;
      const int last_tile = ((si.page0 + si.npages - 1) * 16) >> 7;
      float mseq[4], f_cur[4], mt_nt[4];
#pragma unroll
      for (int tk = 0; tk < 4; ++tk) {
        const int h = min((pw + kWorkerThreads * tk) >> 2, p.num_heads - 1);
        mseq[tk] = msb[h];
        f_cur[tk] = __expf(mtb[(int64_t)h * p.n_tiles + cur_tile] - mseq[tk]);
        mt_nt[tk] = mtb[(int64_t)h * p.n_tiles + min(cur_tile + 1, last_tile)];
      }
      for (int pg = 0; pg < si.npages; ++pg, ++it) {
        const int s = it % S;
        if (!mbar_wait(&ctl->pempty[s], ((it / S) & 1) ^ 1, abort_flag, p.status)) { ok = false; break; }
        if (!mbar_wait(&ctl->vfull[s], (it / S) & 1, abort_flag, p.status)) { ok = false; break; }
        uint8_t* st = smem + s * LY.stage_bytes;
        uint8_t* pb = st + LY.v_bytes + LY.a_bytes + LY.e_bytes;
        const uint8_t* es = st + LY.v_bytes + LY.a_bytes;   // e16 [heads][16 tokens]
        const int t0 = (si.page0 + pg) * 16;
        if ((t0 >> 7) != cur_tile) {   // entering the next tile (uniform across the CTA)
          cur_tile = t0 >> 7;
#pragma unroll
          for (int tk = 0; tk < 4; ++tk) {
            const int h = min((pw + kWorkerThreads * tk) >> 2, p.num_heads - 1);
            f_cur[tk] = __expf(mt_nt[tk] - mseq[tk]);
            mt_nt[tk] = mtb[(int64_t)h * p.n_tiles + min(cur_tile + 1, last_tile)];
          }
        }
        // P rows: thread -> (head, 4 consecutive tokens)
#pragma unroll
        for (int tk = 0; tk < 4; ++tk) {
          const int task = pw + kWorkerThreads * tk;
          if (task >= p.nh * 4) break;
          const int h = task >> 2, kq = task & 3;
          float pv4[4] = {0.f, 0.f, 0.f, 0.f};
          if (h < p.num_heads) {
            const float f = f_cur[tk];
            const uint2 raw = *reinterpret_cast<const uint2*>(es + h * 32 + 8 * kq);
            const __half2 e01 = *reinterpret_cast<const __half2*>(&raw.x);
            const __half2 e23 = *reinterpret_cast<const __half2*>(&raw.y);
            const float2 a = __half22float2(e01), c = __half22float2(e23);
            pv4[0] = a.x * f; pv4[1] = a.y * f; pv4[2] = c.x * f; pv4[3] = c.y * f;
#pragma unroll
            for (int i = 0; i < 4; ++i)
              if (t0 + 4 * kq + i >= L) pv4[i] = 0.f;
            lsum[tk] += (pv4[0] + pv4[1]) + (pv4[2] + pv4[3]);
          }
          if (QUANT) {
#pragma unroll
            for (int blk = 0; blk < 2; ++blk) {
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int k = 4 * kq + i;
                const int o = p.vs_off - p.vx0 + 2 * blk;      // bf16 scale of this block
                const uint8_t* rowp = st + k * 128;
                const uint16_t sbits = *reinterpret_cast<const uint16_t*>(
                    rowp + ((((o >> 4) ^ (k & 7)) << 4) | (o & 15)));
                const float sc = __uint_as_float((uint32_t)sbits << 16);
                // tokens past the sequence get P = 0 whatever their stale scale bytes hold
                *reinterpret_cast<__half*>(pb + blk * p.nh * 32 + kmajor_off(h, k)) =
                    __float2half_rn(t0 + k < L ? pv4[i] * sc : 0.f);
              }
            }
          } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int k = 4 * kq + i;
              if (p.cache_dtype == STARKV_BF16)
                *reinterpret_cast<__nv_bfloat16*>(pb + kmajor_off(h, k)) = __float2bfloat16_rn(pv4[i]);
              else
                *reinterpret_cast<__half*>(pb + kmajor_off(h, k)) = __float2half_rn(pv4[i]);
            }
          }
        }
        if (QUANT) {
          // Dequantize: per task 32 nibbles -> 4 x 8 f16 values n - 8 (channels 0,2,4,6
          // of each group of 8) or 16 (n - 8) (channels 1,3,5,7), pairs (e, e + 4) per
          // 32-bit word in the order e0 e4 e1 e5 e2 e6 e3 e7. Channels past a block's end
          // get values too; their accumulator rows are never flushed.
          const __half2 bias1 = __float2half2_rn(1032.f), bias16 = __float2half2_rn(1152.f);
          auto unbias = [](uint32_t bits, __half2 bias) -> uint32_t {
            const __half2 v = __hsub2(*reinterpret_cast<const __half2*>(&bits), bias);
            return *reinterpret_cast<const uint32_t*>(&v);
          };
#pragma unroll
          for (int i = 0; i < kMaxDq; ++i) {
            if (i >= ndq) break;
            const uint4 A0 = *reinterpret_cast<const uint4*>(st + dq_src0[i]);
            const uint4 A1 = *reinterpret_cast<const uint4*>(st + dq_src1[i]);
            const uint32_t W8[8] = {A0.x, A0.y, A0.z, A0.w, A1.x, A1.y, A1.z, A1.w};
            const int sh = dq_sh[i] & 31, wsel = dq_sh[i] >> 5;
            uint32_t w[4];
            switch (wsel) {
              case 0:
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) w[q4] = __funnelshift_r(W8[q4], W8[q4 + 1], sh);
                break;
              case 1:
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) w[q4] = __funnelshift_r(W8[q4 + 1], W8[q4 + 2], sh);
                break;
              case 2:
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) w[q4] = __funnelshift_r(W8[q4 + 2], W8[q4 + 3], sh);
                break;
              default:
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) w[q4] = __funnelshift_r(W8[q4 + 3], W8[q4 + 4], sh);
                break;
            }
            uint8_t* dst = st + dq_dst[i];
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
              const uint32_t hi8 = w[q4] >> 8;
              *reinterpret_cast<uint4*>(dst + q4 * 128) =
                  make_uint4(unbias((w[q4] & 0x000F000Fu) | 0x64006400u, bias1),
                             unbias((w[q4] & 0x00F000F0u) | 0x64006400u, bias16),
                             unbias((hi8 & 0x000F000Fu) | 0x64006400u, bias1),
                             unbias((hi8 & 0x00F000F0u) | 0x64006400u, bias16));
            }
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&ctl->pfull[s]);
          if (QUANT) mbar_arrive(&ctl->vempty[s]);
        }
      }
      if (!ok) break;
      // softmax denominator: the 4 threads of a head sit in adjacent lanes
      if (si.range == 0) {
#pragma unroll
        for (int tk = 0; tk < 4; ++tk) {
          float v = lsum[tk];
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          const int task = pw + kWorkerThreads * tk;
          const int h = task >> 2;
          if ((task & 3) == 0 && task < p.nh * 4 && h < p.num_heads) atomicAdd(p.l_seq + (int64_t)b * p.num_heads + h, v);
        }
      }
      // ---- flush the accumulator of this sub-item ----
      if (!mbar_wait(&ctl->accfull, acc_cnt & 1, abort_flag, p.status)) break;
      tc_fence_after();
      const int row = q * 32 + lane;
      float* pvb = p.pv + (int64_t)b * p.num_heads * p.pv_stride;
      for (int m = wpair; m < nmt; m += kWorkers / 4) {
        const int gm = mt0 + m;
        int ch, ch_end;
        const float rscale = QUANT && ((row >> 1) & 1) ? 0.0625f : 1.f;   // 3.2-bit odd channels hold 16 (n - 8)
        if (QUANT) {
          // A rows hold each 8-channel group in the order e0 e4 e1 e5 e2 e6 e3 e7
          const bool outl = gm < p.t_out;
          const int r7 = row & 7;
          ch = (outl ? 128 * gm : p.v_nout + 128 * (gm - p.t_out)) + (row & ~7) + ((r7 >> 1) | ((r7 & 1) << 2));
          ch_end = outl ? p.v_nout : p.v_rank;
        } else {
          ch = gm * 128 + row;
          ch_end = p.v_rank;
        }
        for (int c0 = 0; c0 < p.nh; c0 += 16) {
          float v[16];
          tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + m * p.nh + c0, v);
          if (ch < ch_end) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int h = c0 + i;
              if (h >= p.num_heads) continue;
              atomicAdd(pvb + (int64_t)h * p.pv_stride + ch, v[i] * rscale);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->accempty);
      ++acc_cnt;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, tmem_cols);
  }
}

int launch_pv(bool quant, const CUtensorMap& tm_v, const CUtensorMap& tm_e, const PvParams& p, int num_sms,
              cudaStream_t stream) {
  const PvLayout L = pv_layout(quant, p);
  if (L.stages < 2) return STARKV_EINVAL;
  const size_t smem = pv_smem_bytes(quant, p);
  if (smem > 227 * 1024) return STARKV_EINVAL;
  const void* fn = quant ? (const void*)pv_kernel<true> : (const void*)pv_kernel<false>;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return STARKV_ECUDA;
  if (quant)
    pv_kernel<true><<<num_sms, kPvThreads, smem, stream>>>(tm_v, tm_e, p);
  else
    pv_kernel<false><<<num_sms, kPvThreads, smem, stream>>>(tm_v, tm_e, p);
  return cudaGetLastError() == cudaSuccess ? STARKV_OK : STARKV_ECUDA;
}

}  // namespace starkv
