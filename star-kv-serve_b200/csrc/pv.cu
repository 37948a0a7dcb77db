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
//   3.2-bit codes: worker warps dequantize nibbles to integer-valued f16 (n - 8,
//   exact) into an MN-major A tile; the per-token scale folds into P (one P per
//   outlier / inlier block, as paged_quant.py:320-346 does), so A stays exact.
// P = e16 * exp(m_tile - m_seq) is built per page by the worker warps.
//
// Work split: the pages of all sequences are concatenated and cut into equal
// contiguous ranges, one per CTA (x the channel ranges when the accumulator of
// all channels does not fit TMEM), so every CTA streams the same number of bytes
// whatever the length mix. A CTA range crossing a sequence boundary flushes its
// accumulator with f32 atomics into the small L2-resident pv buffer.
//
// Warps: 0 TMA producer, 1 MMA issuer + TMEM owner, 2-5 workers (P, dequant,
// accumulator flush).
#include "starkv_common.cuh"
#include "starkv_kernels.h"

namespace starkv {

namespace {

constexpr int kMaxStages = 4;

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
  int p_bytes;      // P operand(s) per stage
  int stage_bytes;  // all of the above, 1024-aligned
  int stages;
  int total;        // dynamic smem (+ control)
};

__host__ __device__ inline PvLayout pv_layout(bool quant, const PvParams& p) {
  PvLayout L;
  L.v_bytes = quant ? p.v_boxes * 2048 : p.mt_per_range * 4096;
  L.a_bytes = quant ? p.mt_per_range * 4096 : 0;
  L.p_bytes = (quant ? 2 : 1) * p.nh * 32;
  L.stage_bytes = (L.v_bytes + L.a_bytes + L.p_bytes + 1023) & ~1023;
  int s = (200 * 1024) / L.stage_bytes;
  L.stages = s > kMaxStages ? kMaxStages : s;
  L.total = L.stages * L.stage_bytes + (int)sizeof(PvCtl) + 1024 + 64;
  return L;
}

__device__ __forceinline__ int find_le(const int* prefix, int n, int v) {
  int lo = 0, hi = n;
  while (hi - lo > 1) {
    int mid = (lo + hi) >> 1;
    if (prefix[mid] <= v) lo = mid; else hi = mid;
  }
  return lo;
}

// Offset of element (row n, k) in a no-swizzle K-major operand of 16 k-elements.
__device__ __forceinline__ int kmajor_off(int n, int k) {
  return (n >> 3) * 256 + (k >> 3) * 128 + (n & 7) * 16 + (k & 7) * 2;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Sub-item iteration shared by all roles: the CTA's unit range [u, u_end) cut at
// channel-range and sequence boundaries.
struct SubItem {
  int range, b, page0, npages;
};

__device__ __forceinline__ bool next_sub(int& u, int u_end, int total_pages, const int* pprefix, int n,
                                         SubItem& si) {
  if (u >= u_end) return false;
  si.range = u / total_pages;
  const int pi = u % total_pages;
  si.b = find_le(pprefix, n, pi);
  si.page0 = pi - pprefix[si.b];
  const int seq_end = si.range * total_pages + pprefix[si.b + 1];
  const int e = min(u_end, seq_end);
  si.npages = e - u;
  u = e;
  return true;
}

}  // namespace

size_t pv_smem_bytes(bool quant, const PvParams& p) {
  return (size_t)pv_layout(quant, p).total + (size_t)(p.n + 1) * 4;
}

template <bool QUANT>
__global__ void __launch_bounds__(192, 1) pv_kernel(const __grid_constant__ CUtensorMap tm_v, const PvParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const PvLayout LY = pv_layout(QUANT, p);
  PvCtl* ctl = reinterpret_cast<PvCtl*>(smem + LY.stages * LY.stage_bytes);
  int* pprefix = reinterpret_cast<int*>(ctl + 1);   // [n+1] page prefix
  volatile int* abort_flag = &ctl->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = LY.stages;

  if (threadIdx.x == 0) {
    int acc = 0;
    for (int b = 0; b < p.n; ++b) {
      pprefix[b] = acc;
      const int L = min(max(p.seq_lens[b], 0), p.max_seq_len);
      acc += (L + 15) >> 4;
    }
    pprefix[p.n] = acc;
    for (int s = 0; s < S; ++s) {
      mbar_init(&ctl->vfull[s], 1);
      mbar_init(&ctl->vempty[s], QUANT ? 4 : 1);
      mbar_init(&ctl->pfull[s], 4);
      mbar_init(&ctl->pempty[s], 1);
    }
    mbar_init(&ctl->accfull, 1);
    mbar_init(&ctl->accempty, 4);
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
    if (lane == 0) {
      tma_prefetch(&tm_v);
      uint32_t it = 0;
      int u = u_begin;
      SubItem si;
      while (!*abort_flag && next_sub(u, u_end, total_pages, pprefix, p.n, si)) {
        const int mt0 = si.range * p.mt_per_range;
        const int mt1 = min(mt0 + p.mt_per_range, p.n_mtiles);
        for (int pg = 0; pg < si.npages; ++pg, ++it) {
          const int s = it % S;
          if (!mbar_wait(&ctl->vempty[s], ((it / S) & 1) ^ 1, abort_flag, p.status)) break;
          const int t = (si.page0 + pg) * 16;
          const int col = t / p.block_size;
          int blk = -1;
          if (col < p.max_blocks) blk = p.block_table[(int64_t)si.b * p.bt_s0 + (int64_t)col * p.bt_s1];
          if (blk < 0 || blk >= p.num_blocks) {
            record_status(p.status, STARKV_EBOUNDS);
            blk = 0;
          }
          const int slot = t % p.block_size;
          uint8_t* st = smem + s * LY.stage_bytes;
          if (QUANT) {
            mbar_arrive_expect_tx(&ctl->vfull[s], p.v_boxes * 2048);
            for (int jb = 0; jb < p.v_boxes; ++jb)
              tma_load_3d(st + jb * 2048, &tm_v, &ctl->vfull[s], p.vx0 + 128 * jb, slot, blk);
          } else {
            mbar_arrive_expect_tx(&ctl->vfull[s], (mt1 - mt0) * 4096);
            for (int m = mt0; m < mt1; ++m)
              for (int i = 0; i < 2; ++i)
                tma_load_3d(st + (m - mt0) * 4096 + i * 2048, &tm_v, &ctl->vfull[s], p.k_width + m * 128 + 64 * i,
                            slot, blk);
          }
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
      while (!*abort_flag && next_sub(u, u_end, total_pages, pprefix, p.n, si)) {
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
          const uint32_t pbase = st + LY.v_bytes + LY.a_bytes;
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
    const int wt = threadIdx.x - 64;     // 0..127
    const int q = warp & 3;
    uint32_t it = 0, acc_cnt = 0;
    int u = u_begin;
    SubItem si;
    bool ok = true;
    while (ok && !*abort_flag && next_sub(u, u_end, total_pages, pprefix, p.n, si)) {
      const int b = si.b;
      const int L = min(max(p.seq_lens[b], 0), p.max_seq_len);
      const int mt0 = si.range * p.mt_per_range;
      const int nmt = min(mt0 + p.mt_per_range, p.n_mtiles) - mt0;
      const __half* e16b = p.e16 + (int64_t)b * p.num_heads * p.l_pad;
      const float* mtb = p.m_tile + (int64_t)b * p.num_heads * p.n_tiles;
      const float* msb = p.m_seq + (int64_t)b * p.num_heads;
      for (int pg = 0; pg < si.npages; ++pg, ++it) {
        const int s = it % S;
        if (!mbar_wait(&ctl->pempty[s], ((it / S) & 1) ^ 1, abort_flag, p.status)) { ok = false; break; }
        if (QUANT && !mbar_wait(&ctl->vfull[s], (it / S) & 1, abort_flag, p.status)) { ok = false; break; }
        uint8_t* st = smem + s * LY.stage_bytes;
        uint8_t* pb = st + LY.v_bytes + LY.a_bytes;
        const int t0 = (si.page0 + pg) * 16;
        const int tile = t0 >> 7;
        // P rows: thread -> (head, 4 consecutive tokens)
        for (int task = wt; task < p.nh * 4; task += 128) {
          const int h = task >> 2, kq = task & 3;
          float pv4[4] = {0.f, 0.f, 0.f, 0.f};
          if (h < p.num_heads) {
            const float f = __expf(mtb[(int64_t)h * p.n_tiles + tile] - msb[h]);
            const uint2 raw = *reinterpret_cast<const uint2*>(e16b + (int64_t)h * p.l_pad + t0 + 4 * kq);
            const __half2 e01 = *reinterpret_cast<const __half2*>(&raw.x);
            const __half2 e23 = *reinterpret_cast<const __half2*>(&raw.y);
            const float2 a = __half22float2(e01), c = __half22float2(e23);
            pv4[0] = a.x * f; pv4[1] = a.y * f; pv4[2] = c.x * f; pv4[3] = c.y * f;
#pragma unroll
            for (int i = 0; i < 4; ++i)
              if (t0 + 4 * kq + i >= L) pv4[i] = 0.f;
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
                *reinterpret_cast<__half*>(pb + blk * p.nh * 32 + kmajor_off(h, k)) = __float2half_rn(pv4[i] * sc);
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
          // dequantize this page's V nibbles into MN-major f16 A tiles
          uint8_t* ab = st + LY.v_bytes;
          for (int task = wt; task < nmt * 256; task += 128) {
            const int m = task >> 8, tt = task & 255;
            const int k = ((tt >> 7) << 3) | (tt & 7);
            const int g = (tt >> 3) & 15;
            const int gm = mt0 + m;
            const bool outl = gm < p.t_out;
            const int jt = outl ? gm : gm - p.t_out;
            const int ch_first = (outl ? 0 : p.v_nout) + 128 * jt + 8 * g;
            const int ch_end = outl ? p.v_nout : p.v_rank;
            const int byte0 = (outl ? p.vq_off : p.vq_off + p.v_nbo) + 64 * jt + 4 * g - p.vx0;
            uint32_t packed[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int o = byte0 + i;
              const int c0 = ch_first + 2 * i;
              uint32_t byte = 0x88u;
              if (c0 < ch_end) {   // bytes past the block are never read
                const uint8_t* bx = st + (o >> 7) * 2048 + k * 128;
                const int w = o & 127;
                byte = bx[(((w >> 4) ^ (k & 7)) << 4) | (w & 15)];
              }
              const float lo = (c0 < ch_end) ? (float)((int)(byte & 15u) - 8) : 0.f;
              const float hi = (c0 + 1 < ch_end) ? (float)((int)(byte >> 4) - 8) : 0.f;
              const __half2 hv = __floats2half2_rn(lo, hi);
              packed[i] = *reinterpret_cast<const uint32_t*>(&hv);
            }
            *reinterpret_cast<uint4*>(ab + m * 4096 + tt * 16) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
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
      // ---- flush the accumulator of this sub-item ----
      if (!mbar_wait(&ctl->accfull, acc_cnt & 1, abort_flag, p.status)) break;
      tc_fence_after();
      const int row = q * 32 + lane;
      float* pvb = p.pv + (int64_t)b * p.num_heads * p.v_rank;
      for (int m = 0; m < nmt; ++m) {
        const int gm = mt0 + m;
        int ch, ch_end;
        if (QUANT) {
          const bool outl = gm < p.t_out;
          ch = (outl ? 128 * gm : p.v_nout + 128 * (gm - p.t_out)) + row;
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
              if (h < p.num_heads) atomicAdd(pvb + (int64_t)h * p.v_rank + ch, v[i]);
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

int launch_pv(bool quant, const CUtensorMap& tm_v, const PvParams& p, int num_sms, cudaStream_t stream) {
  const PvLayout L = pv_layout(quant, p);
  if (L.stages < 2) return STARKV_EINVAL;
  const size_t smem = pv_smem_bytes(quant, p);
  if (smem > 227 * 1024) return STARKV_EINVAL;
  const void* fn = quant ? (const void*)pv_kernel<true> : (const void*)pv_kernel<false>;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return STARKV_ECUDA;
  if (quant)
    pv_kernel<true><<<num_sms, 192, smem, stream>>>(tm_v, p);
  else
    pv_kernel<false><<<num_sms, 192, smem, stream>>>(tm_v, p);
  return cudaGetLastError() == cudaSuccess ? STARKV_OK : STARKV_ECUDA;
}

}  // namespace starkv
