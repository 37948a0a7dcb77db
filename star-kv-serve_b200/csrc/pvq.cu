// V side of the 3.2-bit paged decode: pv[b, h, c] = sum_t p[b, h, t] * V[b, t, c]
// (unnormalised; the lift divides by the softmax denominator).
//
// Replaces paged_quant.py:311-354 (_paged_pv_fold). Same contraction as the bf16
// P.V kernel (pv.cu): swap-AB tcgen05, D[c, h] += V^T[c, t] . P^T[t, h], M = 128
// code channels, N = heads (rounded to 16), K = 16 tokens (one page), f32
// accumulators in TMEM over the CTA's page range.
//
// The A operand is not in the cache: worker warps build it per page from the
// nibbles, so the copy of a page (12-13 KB of V bytes) is small next to its A
// tiles (4 KB per 128 channels). The two therefore live in separate rings: a deep
// ring of staged page rows (one TMA box per page, a whole row's V part in one
// 8-byte-element box row, plus the page's e16 probabilities), filled far ahead of
// use, and a 2-stage ring of A tiles + P that the workers fill while the MMA reads
// the other stage.
//
// Dequantization: nibble n -> the exact f16 n - 8 (even channels of each group of
// 8) or 16 (n - 8) (odd channels): one bit operation per channel pair makes
// 1024 + n or 1024 + 16 n, one f16 subtraction removes the bias; the flush scales
// odd-channel rows by 1/16. The per-token scale folds into P (one P per outlier /
// inlier block, as paged_quant.py:320-346 does), so A stays exact. A thread's
// dequant tasks (M-tile, token, 32-channel window) are the same on every page, so
// their addresses are worked out once per page range.
//
// Warps: 0 TMA producer, 1 MMA issuer + TMEM owner, 2-13 workers, 14 second MMA
// issuer (each issuer takes half of a page's M-tiles: one thread issues an N = 32
// MMA no faster than every ~50 cycles, so one issuer alone cannot keep up with a
// page's 13 tiles).
#include "pv_common.cuh"
#include "starkv_common.cuh"
#include "starkv_kernels.h"

namespace starkv {

using namespace pvc;

namespace {

constexpr int kMaxVStages = 8;
constexpr int kAStages = 2;
constexpr int kWorkers = 12;                 // worker warps (3 per TMEM lane quarter)
constexpr int kWorkerThreads = 32 * kWorkers;
constexpr int kIssuer2 = 2 + kWorkers;       // warp index of the second MMA issuer
constexpr int kThreads = 32 * (kIssuer2 + 1);
constexpr int kSmemBudget = 224 * 1024;
constexpr int kMaxDq = 3;                    // dequant tasks per thread and page (M-tiles <= 18)
constexpr int kMaxP = 3;                     // P tasks (head, token pair) per thread and page (heads <= 144)

struct Ctl {
  uint64_t vfull[kMaxVStages], vempty[kMaxVStages];
  uint64_t afull[kAStages], aempty[kAStages];
  uint64_t accfull, accempty;
  uint32_t tmem_base;
  int abort_flag;
};

struct Layout {
  int v_rows;       // staged page rows (16 x pitch)
  int v_stage;      // + e16 [heads][16 tokens]
  int a_tiles;      // A tiles of one page (mt_per_range x 4 KB)
  int a_stage;      // + P of the two scale blocks, 1024-aligned
  int sv;           // page ring depth
  int total;        // dynamic smem
};

__host__ __device__ inline Layout layout(const PvParams& p) {
  Layout L;
  L.v_rows = 16 * p.v_pitch;
  L.v_stage = (L.v_rows + ((p.num_heads * 32 + 127) & ~127) + 127) & ~127;
  L.a_tiles = p.mt_per_range * 4096;
  L.a_stage = (L.a_tiles + 2 * p.nh * 32 + 1023) & ~1023;
  const int fixed = kAStages * L.a_stage + (int)sizeof(Ctl) + 1024 + 64 + (2 * p.n + 1) * 4;
  const int sv = (kSmemBudget - fixed) / (L.v_stage > 0 ? L.v_stage : 1);
  L.sv = sv > kMaxVStages ? kMaxVStages : sv;
  L.total = kAStages * L.a_stage + L.sv * L.v_stage + (int)sizeof(Ctl) + 1024 + 64 + (2 * p.n + 1) * 4;
  return L;
}

}  // namespace

int pvq_max_dequant_tasks() { return kMaxDq * kWorkerThreads; }

size_t pvq_smem_bytes(const PvParams& p) { return (size_t)layout(p).total; }
int pvq_page_stages(const PvParams& p) { return layout(p).sv; }

__global__ void __launch_bounds__(kThreads, 1) pvq_kernel(const __grid_constant__ CUtensorMap tm_v,
                                                          const __grid_constant__ CUtensorMap tm_e, const PvParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Layout LY = layout(p);
  uint8_t* a_ring = smem;                                    // [kAStages][a_stage], 1024-aligned
  uint8_t* v_ring = smem + kAStages * LY.a_stage;            // [sv][v_stage]
  Ctl* ctl = reinterpret_cast<Ctl*>(v_ring + LY.sv * LY.v_stage);
  int* pprefix = reinterpret_cast<int*>(ctl + 1);   // [n+1] page prefix over this rank's pages
  int* pbeg = pprefix + p.n + 1;                     // [n] first page of this rank in each sequence
  volatile int* abort_flag = &ctl->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int SV = LY.sv;

  if (threadIdx.x == 0) {
    page_ranges(p, pprefix, pbeg);
    for (int s = 0; s < SV; ++s) {
      mbar_init(&ctl->vfull[s], 1);
      mbar_init(&ctl->vempty[s], kWorkers);
    }
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(&ctl->afull[s], kWorkers);
      mbar_init(&ctl->aempty[s], 2);   // one commit per issuer
    }
    mbar_init(&ctl->accfull, 2);
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
    // All 32 lanes fetch block-table entries (32 pages per batch, one batch ahead);
    // lane 0 issues one box of the page's 16 rows and the page's e16 box.
    if (lane == 0) {
      tma_prefetch(&tm_v);
      tma_prefetch(&tm_e);
    }
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
    const uint32_t stage_tx = LY.v_rows + p.num_heads * 32;
    uint32_t it = 0;
    int u = u_begin;
    SubItem si;
    bool stop = false;
    while (!stop && next_sub(u, u_end, total_pages, pprefix, pbeg, p.n, si)) {
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
          const int s = it % SV;
          ok = mbar_wait(&ctl->vempty[s], ((it / SV) & 1) ^ 1, abort_flag, p.status) ? 1 : 0;
          if (ok) {
            const int t = (si.page0 + pg) * 16;
            uint8_t* st = v_ring + s * LY.v_stage;
            mbar_arrive_expect_tx(&ctl->vfull[s], stage_tx);
            tma_load_3d(st, &tm_v, &ctl->vfull[s], p.vx0 / 8, t % p.block_size, blk);
            tma_load_2d(st + LY.v_rows, &tm_e, &ctl->vfull[s], t, si.b * p.num_heads);
          }
        }
        if (!__shfl_sync(0xffffffffu, ok, 0)) {
          stop = true;
          break;
        }
      }
    }
  } else if (warp == 1 || warp == kIssuer2) {
    // ================= MMA issuers: warp 1 the first half of the M-tiles, the other the rest =================
    if (lane == 0) {
      const bool second = warp == kIssuer2;
      const uint32_t idesc = instr_desc_f16(/*f16*/ 0, /*A MN-major*/ 1, /*B K-major*/ 0, 128, p.nh);
      uint32_t it = 0, acc_cnt = 0;
      int u = u_begin;
      SubItem si;
      while (!*abort_flag && next_sub(u, u_end, total_pages, pprefix, pbeg, p.n, si)) {
        const int mt0 = si.range * p.mt_per_range;
        const int nmt = min(mt0 + p.mt_per_range, p.n_mtiles) - mt0;
        if (!mbar_wait(&ctl->accempty, (acc_cnt & 1) ^ 1, abort_flag, p.status)) break;
        tc_fence_after();
        for (int pg = 0; pg < si.npages; ++pg, ++it) {
          const int s = it % kAStages;
          if (!mbar_wait(&ctl->afull[s], (it / kAStages) & 1, abort_flag, p.status)) break;
          tc_fence_after();
          const uint32_t st = smem_u32(a_ring + s * LY.a_stage);
          const uint32_t pbase = st + LY.a_tiles;
          // A tiles are 4 KB apart (descriptor address field in 16-byte units); the
          // outlier tiles take the first block's P, the rest the second's. Issued in
          // unrolled groups of 4: a loop branch after every MMA costs ~3x its issue time.
          // Each issuer commits its own MMAs; the stage is free after both commits.
          const uint64_t da0 = smem_desc(st, 2048, 128, kSwizzleNone);   // 8 ch x 8 tok cores
          const uint64_t db_out = smem_desc(pbase, 128, 256, kSwizzleNone);
          const uint64_t db_in = smem_desc(pbase + p.nh * 32, 128, 256, kSwizzleNone);
          const uint32_t acc = pg > 0 ? 1u : 0u;
          const int mh = (nmt + 1) >> 1, mhi = second ? nmt : mh;
          int m = second ? mh : 0;
          for (; m + 4 <= mhi; m += 4) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
              umma_f16(tmem + (m + i) * p.nh, da0 + (uint64_t)((m + i) * 256), mt0 + m + i < p.t_out ? db_out : db_in,
                       idesc, acc);
          }
          for (; m < mhi; ++m)
            umma_f16(tmem + m * p.nh, da0 + (uint64_t)(m * 256), mt0 + m < p.t_out ? db_out : db_in, idesc, acc);
          umma_commit(&ctl->aempty[s]);
        }
        umma_commit(&ctl->accfull);
        ++acc_cnt;
      }
    }
  } else {
    // ================= workers: P, A tiles, accumulator flush =================
    const int wt = threadIdx.x - 64;     // 0..kWorkerThreads-1
    const int q = warp & 3;
    const int wpair = (warp - 2) >> 2;   // which of the kWorkers / 4 warps of lane quarter q
    // P tasks (head, token pair), pt = head * 8 + pair, start at worker thread 64: the
    // first 64 threads carry the third dequant task. The 8 tasks of a head sit in 8
    // adjacent lanes.
    const int pbase = (wt + kWorkerThreads - 64) % kWorkerThreads;
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
      float lsum[kMaxP];   // sum of P (before the row scale) of this thread's tasks
      // P = e16 * exp(m_tile - m_seq): the factor of the current 128-token tile, and
      // the next tile's max loaded as soon as the current tile starts
      int cur_tile = (si.page0 * 16) >> 7;
      const int last_tile = ((si.page0 + si.npages - 1) * 16) >> 7;
      float mseq[kMaxP], f_cur[kMaxP], mt_nt[kMaxP];
#pragma unroll
      for (int j = 0; j < kMaxP; ++j) {
        const int h = min((pbase + kWorkerThreads * j) >> 3, p.num_heads - 1);
        lsum[j] = 0.f;
        mseq[j] = msb[h];
        f_cur[j] = __expf(mtb[(int64_t)h * p.n_tiles + cur_tile] - mseq[j]);
        mt_nt[j] = mtb[(int64_t)h * p.n_tiles + min(cur_tile + 1, last_tile)];
      }
      // this thread's dequant tasks: (M-tile, token, 16-byte window = 32 channels) ->
      // source offset in the staged row (the two 16-byte chunks the window spans),
      // bit shift that cuts the window out of them, A-tile destination
      int dq_src[kMaxDq], dq_src1[kMaxDq], dq_dst[kMaxDq], dq_sh[kMaxDq];
      int ndq = 0;
#pragma unroll
      for (int i = 0; i < kMaxDq; ++i) {
        const int task = wt + kWorkerThreads * i;
        dq_src[i] = dq_src1[i] = dq_dst[i] = dq_sh[i] = 0;
        if (task >= nmt * 64) continue;
        ndq = i + 1;
        const int m = task >> 6, tt = task & 63;
        const int k = tt & 15, j = tt >> 4;
        const int gm = mt0 + m;
        const bool outl = gm < p.t_out;
        const int jt = outl ? gm : gm - p.t_out;
        const int bb = (outl ? p.vq_off : p.vq_off + p.v_nbo) - p.vx0;   // block start in the staged row
        // the window's two 16-byte chunks; at the end of the staged row the second is
        // the first again (the bytes it would hold lie past the block)
        const int nvq = p.v_pitch / 16 - 1;
        const int c0 = min((bb + 64 * jt + 16 * j) >> 4, nvq), c1 = min(c0 + 1, nvq);
        dq_src[i] = k * p.v_pitch + c0 * 16;
        dq_src1[i] = k * p.v_pitch + c1 * 16;
        dq_dst[i] = m * 4096 + (k >> 3) * 2048 + (4 * j) * 128 + (k & 7) * 16;
        dq_sh[i] = (bb & 15) * 8;   // bits 5-6: word, bits 0-4: shift inside the word
      }
      const __half2 bias1 = __float2half2_rn(1032.f), bias16 = __float2half2_rn(1152.f);
      auto unbias = [](uint32_t bits, __half2 bias) -> uint32_t {
        const __half2 v = __hsub2(*reinterpret_cast<const __half2*>(&bits), bias);
        return *reinterpret_cast<const uint32_t*>(&v);
      };
      for (int pg = 0; pg < si.npages; ++pg, ++it) {
        const int sv = it % SV, sa = it % kAStages;
        // the page's rows first: the loads of all dequant tasks are in flight while
        // this thread waits for its A stage to be released by the MMA
        if (!mbar_wait(&ctl->vfull[sv], (it / SV) & 1, abort_flag, p.status)) { ok = false; break; }
        const uint8_t* vs = v_ring + sv * LY.v_stage;      // [16 rows][pitch], then e16 [heads][16]
        const uint8_t* es = vs + LY.v_rows;
        uint4 src0[kMaxDq], src1[kMaxDq];
#pragma unroll
        for (int i = 0; i < kMaxDq; ++i) {
          if (i < ndq) {
            src0[i] = *reinterpret_cast<const uint4*>(vs + dq_src[i]);
            src1[i] = *reinterpret_cast<const uint4*>(vs + dq_src1[i]);
          } else {
            src0[i] = src1[i] = make_uint4(0u, 0u, 0u, 0u);
          }
        }
        if (!mbar_wait(&ctl->aempty[sa], ((it / kAStages) & 1) ^ 1, abort_flag, p.status)) { ok = false; break; }
        uint8_t* as = a_ring + sa * LY.a_stage;           // A tiles, then P of the two blocks
        uint8_t* pb = as + LY.a_tiles;
        const int t0 = (si.page0 + pg) * 16;
        if ((t0 >> 7) != cur_tile) {   // entering the next tile (uniform across the CTA)
          cur_tile = t0 >> 7;
#pragma unroll
          for (int j = 0; j < kMaxP; ++j) {
            const int h = min((pbase + kWorkerThreads * j) >> 3, p.num_heads - 1);
            f_cur[j] = __expf(mt_nt[j] - mseq[j]);
            mt_nt[j] = mtb[(int64_t)h * p.n_tiles + min(cur_tile + 1, last_tile)];
          }
        }
        // P of the two scale blocks for (head, tokens k0, k0 + 1): one 4-byte store per
        // block. Tokens past the sequence get P = 0 whatever their stale bytes hold.
#pragma unroll
        for (int j = 0; j < kMaxP; ++j) {
          const int pt = pbase + kWorkerThreads * j;
          if (pt >= p.nh * 8) break;
          const int h = pt >> 3, k0 = (pt & 7) * 2;
          const bool in0 = h < p.num_heads && t0 + k0 < L, in1 = h < p.num_heads && t0 + k0 + 1 < L;
          float2 e = make_float2(0.f, 0.f);
          if (h < p.num_heads) e = __half22float2(*reinterpret_cast<const __half2*>(es + h * 32 + k0 * 2));
          const float e0 = in0 ? e.x * f_cur[j] : 0.f, e1 = in1 ? e.y * f_cur[j] : 0.f;
          lsum[j] += e0 + e1;
          // (outlier, inlier) bf16 scales of tokens k0 and k0 + 1
          const uint32_t s0 = *reinterpret_cast<const uint32_t*>(vs + k0 * p.v_pitch + p.vs_off - p.vx0);
          const uint32_t s1 = *reinterpret_cast<const uint32_t*>(vs + (k0 + 1) * p.v_pitch + p.vs_off - p.vx0);
          const __half2 po = __floats2half2_rn(in0 ? e0 * __uint_as_float(s0 << 16) : 0.f,
                                               in1 ? e1 * __uint_as_float(s1 << 16) : 0.f);
          const __half2 pi = __floats2half2_rn(in0 ? e0 * __uint_as_float(s0 & 0xFFFF0000u) : 0.f,
                                               in1 ? e1 * __uint_as_float(s1 & 0xFFFF0000u) : 0.f);
          *reinterpret_cast<__half2*>(pb + kmajor_off(h, k0)) = po;
          *reinterpret_cast<__half2*>(pb + p.nh * 32 + kmajor_off(h, k0)) = pi;
        }
        // dequant: 32 nibbles -> 4 x 8 f16 (n - 8 or 16 (n - 8)), pairs (e, e + 4) per
        // word in the order e0 e4 e1 e5 e2 e6 e3 e7; channels past a block's end get
        // values too, their accumulator rows are never flushed
#pragma unroll
        for (int i = 0; i < kMaxDq; ++i) {
          if (i >= ndq) break;
          const uint4 A0 = src0[i], A1 = src1[i];
          const uint32_t W8[8] = {A0.x, A0.y, A0.z, A0.w, A1.x, A1.y, A1.z, A1.w};
          const int sh = dq_sh[i] & 31;
          uint32_t w[4];
          switch (dq_sh[i] >> 5) {
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
          uint8_t* dst = as + dq_dst[i];
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
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&ctl->afull[sa]);
          mbar_arrive(&ctl->vempty[sv]);
        }
      }
      if (!ok) break;
      // softmax denominator: the 8 threads of a head sit in adjacent lanes
      if (si.range == 0) {
#pragma unroll
        for (int j = 0; j < kMaxP; ++j) {
          float v = lsum[j];
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          v += __shfl_xor_sync(0xffffffffu, v, 4);
          const int pt = pbase + kWorkerThreads * j;
          const int h = pt >> 3;
          if ((pt & 7) == 0 && pt < p.nh * 8 && h < p.num_heads)
            atomicAdd(p.l_seq + (int64_t)b * p.num_heads + h, v);
        }
      }
      // ---- flush the accumulator of this sub-item ----
      if (!mbar_wait(&ctl->accfull, acc_cnt & 1, abort_flag, p.status)) break;
      tc_fence_after();
      const int row = q * 32 + lane;
      // A rows hold each 8-channel group in the order e0 e4 e1 e5 e2 e6 e3 e7; odd
      // channels (rows 2,3,6,7 of each 8) hold 16 (n - 8)
      const int r7 = row & 7;
      const float rscale = ((row >> 1) & 1) ? 0.0625f : 1.f;
      float* pvb = p.pv + (int64_t)b * p.num_heads * p.pv_stride;
      for (int m = wpair; m < nmt; m += kWorkers / 4) {
        const int gm = mt0 + m;
        const bool outl = gm < p.t_out;
        const int ch = (outl ? 128 * gm : p.v_nout + 128 * (gm - p.t_out)) + (row & ~7) + ((r7 >> 1) | ((r7 & 1) << 2));
        const int ch_end = outl ? p.v_nout : p.v_rank;
        for (int c0 = 0; c0 < p.nh; c0 += 16) {
          float v[16];
          tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + m * p.nh + c0, v);
          if (ch < ch_end) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int h = c0 + i;
              if (h < p.num_heads) atomicAdd(pvb + (int64_t)h * p.pv_stride + ch, v[i] * rscale);
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

int launch_pvq(const CUtensorMap& tm_v, const CUtensorMap& tm_e, const PvParams& p, int num_sms,
               cudaStream_t stream) {
  const Layout L = layout(p);
  if (L.sv < 2) return STARKV_EINVAL;
  if (L.total > 227 * 1024) return STARKV_EINVAL;
  if (p.mt_per_range * 64 > kMaxDq * kWorkerThreads) return STARKV_EINVAL;   // dequant tasks per thread
  if (p.nh * 8 > kMaxP * kWorkerThreads) return STARKV_EINVAL;               // P tasks per thread
  if (cudaFuncSetAttribute(pvq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total) != cudaSuccess)
    return STARKV_ECUDA;
  pvq_kernel<<<num_sms, kThreads, L.total, stream>>>(tm_v, tm_e, p);
  return cudaGetLastError() == cudaSuccess ? STARKV_OK : STARKV_ECUDA;
}

}  // namespace starkv
