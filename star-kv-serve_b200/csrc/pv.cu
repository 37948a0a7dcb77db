// V side of the paged decode over bf16 / f16 codes:
// pv[b, h, c] = sum_t p[b, h, t] * V[b, t, c] (unnormalised; the lift divides by
// the softmax denominator). The 3.2-bit codes have their own kernel (pvq.cu).
//
// Replaces paged_decode.py:105-147 + :220 (_paged_pv_fwd and the segment sum).
//
// V is one latent shared by every head (checkpoint.py:140-153), so one CTA owns
// all heads of a token range and reads each V code once. The contraction runs on
// tcgen05 in swap-AB form, D[c, h] += V^T[c, t] . P^T[t, h]: M = 128 code
// channels, N = heads (rounded to 16), K = 16 tokens (one page) per instruction,
// f32 accumulators in TMEM across the whole token range. A = V^T straight from
// the TMA page tile (MN-major, 128 B swizzle; all whole 64-channel tiles of a page
// in one 4D box); P = e16 * exp(m_tile - m_seq) is
// built per page by the worker warps.
//
// Work split: the pages of all sequences are concatenated and cut into equal
// contiguous ranges, one per CTA (x the channel ranges when the accumulator of
// all channels does not fit TMEM), so every CTA streams the same number of bytes
// whatever the length mix. A CTA range crossing a sequence boundary flushes its
// accumulator with f32 atomics into the small L2-resident pv buffer.
//
// Warps: 0 TMA producer, 1 MMA issuer + TMEM owner, 2-13 workers (P, accumulator
// flush; the three warps of a TMEM lane quarter split the M-tiles), 14 second MMA
// issuer (each issuer takes half of a page's M-tiles: one thread issues an N = 32
// MMA no faster than every ~50 cycles).
#include "pv_common.cuh"
#include "starkv_common.cuh"
#include "starkv_kernels.h"

namespace starkv {

using namespace pvc;

namespace {

constexpr int kMaxStages = 4;
constexpr int kPageStages = 3;
constexpr int kWorkers = 12;                 // worker warps (3 per TMEM lane quarter)
constexpr int kWorkerThreads = 32 * kWorkers;
constexpr int kIssuer2 = 2 + kWorkers;       // warp index of the second MMA issuer
constexpr int kPvThreads = 32 * (kIssuer2 + 1);

struct PvCtl {
  uint64_t vfull[kMaxStages], vempty[kMaxStages];
  uint64_t pfull[kMaxStages], pempty[kMaxStages];
  uint64_t accfull, accempty;
  uint32_t tmem_base;
  int abort_flag;
};

struct PvLayout {
  int v_bytes;      // TMA tile bytes per stage
  int e_bytes;      // TMA tile of e16 (heads x 16 tokens) per stage
  int p_bytes;      // P operand(s) per stage
  int stage_bytes;  // all of the above, 1024-aligned
  int stages;
  int total;        // dynamic smem (+ control)
};

__host__ __device__ inline PvLayout pv_layout(const PvParams& p) {
  PvLayout L;
  L.v_bytes = p.mt_per_range * 4096;
  L.e_bytes = (p.num_heads * 32 + 127) & ~127;
  L.p_bytes = p.nh * 32;
  L.stage_bytes = (L.v_bytes + L.e_bytes + L.p_bytes + 1023) & ~1023;
  // three pages in flight: a fourth measured slower (more bytes outstanding per SM
  // than the memory system serves best)
  int s = (200 * 1024) / L.stage_bytes;
  L.stages = s > kPageStages ? kPageStages : s;
  L.total = L.stages * L.stage_bytes + (int)sizeof(PvCtl) + 1024 + 64;
  return L;
}

}  // namespace

int pv_page_stages(const PvParams& p) { return pv_layout(p).stages; }

size_t pv_smem_bytes(const PvParams& p) {
  return (size_t)pv_layout(p).total + (size_t)(2 * p.n + 1) * 4;
}

__global__ void __launch_bounds__(kPvThreads, 1) pv_kernel(const __grid_constant__ CUtensorMap tm_v,
                                                    const __grid_constant__ CUtensorMap tm_va,
                                                    const __grid_constant__ CUtensorMap tm_vb,
                                                    const __grid_constant__ CUtensorMap tm_e, const PvParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const PvLayout LY = pv_layout(p);
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
      mbar_init(&ctl->vempty[s], 2);   // one commit per issuer
      mbar_init(&ctl->pfull[s], kWorkers);
      mbar_init(&ctl->pempty[s], 2);
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
    // All 32 lanes fetch block-table entries (32 pages per batch, one batch
    // ahead, so the table's latency is never on the issue path); lane 0 issues
    // the copies.
    if (lane == 0) {
      tma_prefetch(&tm_v);
      if (p.box_a > 0) tma_prefetch(&tm_va);
      if (p.box_b > 0) tma_prefetch(&tm_vb);
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
      const bool last_range = si.range == p.n_ranges - 1;
      const int nfull = last_range ? p.box_b : p.box_a;          // whole 64-channel tiles, one 4D box
      const bool tail = last_range && p.v_tail;                   // + the trailing 32-channel tile
      const uint32_t stage_tx = (nfull + (tail ? 1 : 0)) * 2048 + e_bytes;
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
            // tiles past the tail are not loaded: they only feed accumulator rows of
            // channels >= v_rank, which are never flushed
            mbar_arrive_expect_tx(&ctl->vfull[s], stage_tx);
            if (nfull > 0) tma_load_4d(st, last_range ? &tm_vb : &tm_va, &ctl->vfull[s], 0, slot, 2 * mt0, blk);
            if (tail)
              tma_load_3d(st + (p.v_full - 2 * mt0) * 2048, &tm_v, &ctl->vfull[s], p.k_width + 64 * p.v_full, slot,
                          blk);
            // e16 rows of this sequence's heads for the page's 16 tokens
            tma_load_2d(st + LY.v_bytes, &tm_e, &ctl->vfull[s], t, si.b * p.num_heads);
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
      const uint32_t fmt = p.cache_dtype == STARKV_BF16 ? 1u : 0u;
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
          if (!mbar_wait(&ctl->vfull[s], (it / S) & 1, abort_flag, p.status)) break;
          if (!mbar_wait(&ctl->pfull[s], (it / S) & 1, abort_flag, p.status)) break;
          tc_fence_after();
          const uint32_t st = smem_u32(smem + s * LY.stage_bytes);
          // V tiles are 4 KB apart (descriptor address field in 16-byte units); issued
          // in unrolled groups of 4: a loop branch after every MMA costs ~3x its issue time
          const uint64_t da0 = smem_desc(st, 2048, 1024, kSwizzle128B);
          const uint64_t db = smem_desc(st + LY.v_bytes + LY.e_bytes, 128, 256, kSwizzleNone);
          const uint32_t acc = pg > 0 ? 1u : 0u;
          const int mh = (nmt + 1) >> 1, mhi = second ? nmt : mh;
          int m = second ? mh : 0;
          for (; m + 4 <= mhi; m += 4) {
#pragma unroll
            for (int i = 0; i < 4; ++i) umma_f16(tmem + (m + i) * p.nh, da0 + (uint64_t)((m + i) * 256), db, idesc, acc);
          }
          for (; m < mhi; ++m) umma_f16(tmem + m * p.nh, da0 + (uint64_t)(m * 256), db, idesc, acc);
          umma_commit(&ctl->vempty[s]);
          umma_commit(&ctl->pempty[s]);
        }
        umma_commit(&ctl->accfull);
        ++acc_cnt;
      }
    }
  } else {
    // ================= workers: P, accumulator flush =================
    const int wt = threadIdx.x - 64;     // 0..kWorkerThreads-1
    const int q = warp & 3;
    const int wpair = (warp - 2) >> 2;   // which of the kWorkers / 4 warps of lane quarter q
    // P tasks: thread -> (head, 4 consecutive tokens); the 4 threads of a head sit in
    // adjacent lanes
    const int pw = wt;
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
        uint8_t* pb = st + LY.v_bytes + LY.e_bytes;
        const uint8_t* es = st + LY.v_bytes;   // e16 [heads][16 tokens]
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
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int k = 4 * kq + i;
            if (p.cache_dtype == STARKV_BF16)
              *reinterpret_cast<__nv_bfloat16*>(pb + kmajor_off(h, k)) = __float2bfloat16_rn(pv4[i]);
            else
              *reinterpret_cast<__half*>(pb + kmajor_off(h, k)) = __float2half_rn(pv4[i]);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->pfull[s]);
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
        const int ch = gm * 128 + row;
        for (int c0 = 0; c0 < p.nh; c0 += 16) {
          float v[16];
          tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + m * p.nh + c0, v);
          if (ch < p.v_rank) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int h = c0 + i;
              if (h >= p.num_heads) continue;
              atomicAdd(pvb + (int64_t)h * p.pv_stride + ch, v[i]);
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

int launch_pv(const CUtensorMap& tm_v, const CUtensorMap& tm_va, const CUtensorMap& tm_vb, const CUtensorMap& tm_e,
              const PvParams& p, int num_sms, cudaStream_t stream) {
  const PvLayout L = pv_layout(p);
  if (L.stages < 2) return STARKV_EINVAL;
  const size_t smem = pv_smem_bytes(p);
  if (smem > 227 * 1024) return STARKV_EINVAL;
  if (cudaFuncSetAttribute(pv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return STARKV_ECUDA;
  if (p.box_a < 0 || p.box_b < 0 || p.box_a > 256 || p.box_b > 256) return STARKV_EINVAL;
  pv_kernel<<<num_sms, kPvThreads, smem, stream>>>(tm_v, tm_va, tm_vb, tm_e, p);
  return cudaGetLastError() == cudaSuccess ? STARKV_OK : STARKV_ECUDA;
}

}  // namespace starkv
