// Causal attention of whole prompts for the dense prefill (attention.py:219-251):
// replaces the flash_attn_varlen_func call (attention.py:246-250) that attends each
// prompt over its own lifted, rotated K and V.
//
// One CTA per (128-query tile of a prompt, query head). Per 128-key tile j of the
// causal range:
//   S_j = Q . K_j^T       tcgen05 (M = 128 queries, N = 128 keys, K = 128 dims),
//                         f32 in TMEM, three buffers: S_{j+2} is issued right after
//                         the P.V of tile j, so it runs while the softmax works on
//                         S_{j+1} and never delays a P.V;
//   P_j = exp(S_j - m)    online softmax by 4 warps (one query row per thread, a
//                         TMEM lane each), the running output rescaled in TMEM when
//                         a row's max grows by more than 2^8; P_j (bf16 / f16)
//                         written to shared memory in the 128-byte-swizzled K-major
//                         MMA layout;
//   O  += P_j . V_j       tcgen05 (N = 128 dims, K = 128 keys), f32 in TMEM.
// Q, K and V tiles come by TMA (128-byte swizzle, two 64-dim boxes per tile); K and
// V have two slots each, freed by the S and the P.V that read them. The last tile is masked causally (key > query) and every
// tile by the prompt length.
//
// Warps: 0 TMA producer, 1 TMEM owner and MMA issuer, 2-5 softmax (TMEM lane
// quarters 2, 3, 0, 1). All pipeline waits are bounded (STARKV_ETIMEOUT).
#include "starkv_common.cuh"
#include "starkv_kernels.h"

namespace starkv {

namespace {

constexpr int kRows = 128;                    // queries per tile, keys per tile
constexpr int kHalfBytes = kRows * 128;       // one 64-dim half of a tile: [128 rows][128 B]
constexpr int kTileBytes = 2 * kHalfBytes;    // 32 KB
constexpr int kThreads = 192;

struct PrefillCtl {
  uint64_t q_full;
  uint64_t k_full[2], k_empty[2], v_full[2], v_empty[2];
  uint64_t s_full[3], s_free[3];
  uint64_t p_full, o_done, drain;
  uint32_t tmem_base;
  int abort_flag;
  int prompt, tile, start, len;
};

// Shared memory: Q | K0 K1 | V0 V1 | P, each 32 KB and 1024-aligned, then control.
// TMEM: three S buffers (columns 0, 128, 256) and the output (384).
constexpr int kSmemQ = 0;
constexpr int kSmemK = kTileBytes;
constexpr int kSmemV = kSmemK + 2 * kTileBytes;
constexpr int kSmemP = kSmemV + 2 * kTileBytes;
constexpr int kOCol = 3 * kRows;
constexpr int kSmemCtl = kSmemP + kTileBytes;
constexpr int kSmemBytes = kSmemCtl + (int)sizeof(PrefillCtl) + 1024;

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 2^x by the hardware approximation (ex2.approx.ftz: -inf -> +0)
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Bounded wait that ignores the abort flag: used at teardown so that no copy or MMA
// of this CTA is still writing its shared memory or TMEM when the CTA exits.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity, int32_t* status) {
  for (uint32_t i = 0; i < kWaitLimit; ++i)
    if (mbar_try_wait(bar, parity)) return;
  record_status(status, STARKV_ETIMEOUT);
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// K-major, 128-byte-swizzled operand tile [2 halves of 64 K-elements][128 rows][128 B]:
// descriptor for K-step kk (16 elements).
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int kk) {
  return smem_desc(base + (kk >> 2) * kHalfBytes + (kk & 3) * 32, 16, 1024, kSwizzle128B);
}

}  // namespace

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const PrefillParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PrefillCtl* ctl = reinterpret_cast<PrefillCtl*>(smem + kSmemCtl);
  volatile int* abort_flag = &ctl->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hq = blockIdx.y;

  if (threadIdx.x == 0) {
    // this CTA's prompt and query tile: blockIdx.x counts the 128-query tiles of all
    // prompts in order
    int acc = 0, prompt = -1, tile = 0, start = 0, len = 0;
    for (int i = 0; i < p.n_prompts; ++i) {
      const int s0 = p.cu_seqlens[i], s1 = p.cu_seqlens[i + 1];
      const int L = s1 - s0;
      if (s0 < 0 || L < 0 || s1 > p.num_tokens) {
        record_status(p.status, STARKV_EBOUNDS);
        break;
      }
      const int nt = (L + kRows - 1) / kRows;
      if ((int)blockIdx.x < acc + nt) {
        prompt = i; tile = blockIdx.x - acc; start = s0; len = L;
        break;
      }
      acc += nt;
    }
    ctl->prompt = prompt; ctl->tile = tile; ctl->start = start; ctl->len = len;
    mbar_init(&ctl->q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&ctl->k_full[s], 1);
      mbar_init(&ctl->k_empty[s], 1);
      mbar_init(&ctl->v_full[s], 1);
      mbar_init(&ctl->v_empty[s], 1);
    }
    for (int s = 0; s < 3; ++s) {
      mbar_init(&ctl->s_full[s], 1);
      mbar_init(&ctl->s_free[s], 4);
    }
    mbar_init(&ctl->p_full, 4);
    mbar_init(&ctl->o_done, 1);
    mbar_init(&ctl->drain, 1);
    ctl->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&ctl->tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const int prompt = ctl->prompt;
  const uint32_t tmem = ctl->tmem_base;
  const int qt = ctl->tile, start = ctl->start, L = ctl->len;
  const int nt = qt + 1;   // key tiles 0..qt (causal)
  const int hk = hq / p.k_group, hv = hq / p.v_group;

  if (prompt >= 0) {
    if (warp == 0) {
      // ================= TMA producer =================
      if (lane == 0) {
        tma_prefetch(&tm_q);
        tma_prefetch(&tm_k);
        tma_prefetch(&tm_v);
        mbar_arrive_expect_tx(&ctl->q_full, kTileBytes);
        for (int h = 0; h < 2; ++h)
          tma_load_3d(smem + kSmemQ + h * kHalfBytes, &tm_q, &ctl->q_full, 64 * h, hq, start + kRows * qt);
        // K and V tiles in separate rings: K_j's slot frees when S_j is done, V_j's when
        // the P.V of tile j is, so the next S is never queued behind a P.V
        int last_k[2] = {-1, -1}, last_v[2] = {-1, -1};   // last load issued into each slot
        for (int j = 0; j < nt; ++j) {
          const int s = j & 1;
          if (!mbar_wait(&ctl->k_empty[s], ((j >> 1) & 1) ^ 1, abort_flag, p.status)) break;
          last_k[s] = j;
          uint8_t* kd = smem + kSmemK + s * kTileBytes;
          mbar_arrive_expect_tx(&ctl->k_full[s], kTileBytes);
          for (int h = 0; h < 2; ++h)
            tma_load_3d(kd + h * kHalfBytes, &tm_k, &ctl->k_full[s], 64 * h, hk, start + kRows * j);
          if (!mbar_wait(&ctl->v_empty[s], ((j >> 1) & 1) ^ 1, abort_flag, p.status)) break;
          last_v[s] = j;
          uint8_t* vd = smem + kSmemV + s * kTileBytes;
          mbar_arrive_expect_tx(&ctl->v_full[s], kTileBytes);
          for (int h = 0; h < 2; ++h)
            tma_load_3d(vd + h * kHalfBytes, &tm_v, &ctl->v_full[s], 64 * h, hv, start + kRows * j);
        }
        // every copy has landed before the CTA may exit (consumed ones return at once)
        drain_wait(&ctl->q_full, 0, p.status);
        for (int s = 0; s < 2; ++s) {
          if (last_k[s] >= 0) drain_wait(&ctl->k_full[s], (last_k[s] >> 1) & 1, p.status);
          if (last_v[s] >= 0) drain_wait(&ctl->v_full[s], (last_v[s] >> 1) & 1, p.status);
        }
      }
    } else if (warp == 1) {
      // ================= MMA issuer =================
      if (lane == 0) {
        const uint32_t fmt = p.dtype == STARKV_BF16 ? 1u : 0u;
        const uint32_t idesc_s = instr_desc_f16(fmt, 0, 0, kRows, kRows);        // Q . K^T, both K-major
        const uint32_t idesc_o = instr_desc_f16(fmt, 0, 1, kRows, 128);          // P . V, V MN-major
        const uint32_t q_addr = smem_u32(smem + kSmemQ), p_addr = smem_u32(smem + kSmemP);
        // S_j into TMEM buffer j % 3; S_0 and S_1 first, then after each P.V_j the
        // S two tiles ahead, so a P.V never waits behind an S in the tensor pipe
        auto issue_s = [&](int j) -> bool {
          const int s = j & 1, b = j % 3;
          if (!mbar_wait(&ctl->k_full[s], (j >> 1) & 1, abort_flag, p.status) ||
              !mbar_wait(&ctl->s_free[b], ((j / 3) & 1) ^ 1, abort_flag, p.status))
            return false;
          tc_fence_after();
          const uint32_t k_addr = smem_u32(smem + kSmemK + s * kTileBytes);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_f16(tmem + b * kRows, kmajor_desc(q_addr, kk), kmajor_desc(k_addr, kk), idesc_s, kk > 0);
          umma_commit(&ctl->s_full[b]);
          umma_commit(&ctl->k_empty[s]);
          return true;
        };
        bool ok = mbar_wait(&ctl->q_full, 0, abort_flag, p.status);
        for (int j = 0; ok && j < 2 && j < nt; ++j) ok = issue_s(j);
        for (int j = 0; ok && j < nt; ++j) {
          const int s = j & 1;
          if (!mbar_wait(&ctl->p_full, j & 1, abort_flag, p.status) ||
              !mbar_wait(&ctl->v_full[s], (j >> 1) & 1, abort_flag, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t v_addr = smem_u32(smem + kSmemV + s * kTileBytes);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_f16(tmem + kOCol, kmajor_desc(p_addr, kk),
                     smem_desc(v_addr + kk * 2048, kHalfBytes, 1024, kSwizzle128B), idesc_o, j > 0 || kk > 0);
          umma_commit(&ctl->o_done);
          umma_commit(&ctl->v_empty[s]);
          if (j + 2 < nt) ok = issue_s(j + 2);
        }
        // every MMA issued here has completed before TMEM is freed
        umma_commit(&ctl->drain);
        drain_wait(&ctl->drain, 0, p.status);
      }
    } else {
      // ================= softmax, P, output (warps 2-5) =================
      const int q4 = warp & 3;
      const int row = q4 * 32 + lane;
      const int qi = kRows * qt + row;                 // query index in the prompt
      const uint32_t lane_base = tmem + ((uint32_t)(q4 * 32) << 16);
      uint8_t* prow = smem + kSmemP + row * 128;
      float m = -INFINITY, l = 0.f;
      bool ok = true;
      for (int j = 0; j < nt; ++j) {
        const int s = j % 3;   // S buffer of tile j
        if (!mbar_wait(&ctl->s_full[s], (j / 3) & 1, abort_flag, p.status)) { ok = false; break; }
        tc_fence_after();
        uint32_t sr[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32_issue(lane_base + s * kRows + 32 * c, sr[c]);
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_wait(sr[c]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->s_free[s]);
        // keys of this tile a query may see: k <= qi and k < L
        const int kend = min(qi + 1, L) - kRows * j;   // valid columns [0, kend)
        // masked logits become -inf (their exponentials 0); eight independent max and
        // sum chains keep the pass from serialising on one accumulator
        if (!__all_sync(0xffffffffu, kend >= kRows)) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (32 * c + i >= kend) sr[c][i] = __float_as_uint(-INFINITY);
        }
        float mx[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) mx[e] = -INFINITY;
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) mx[i & 7] = fmaxf(mx[i & 7], __uint_as_float(sr[c][i]));
#pragma unroll
        for (int e = 0; e < 4; ++e) mx[e] = fmaxf(mx[e], mx[e + 4]);
        const float mraw = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
        const float mt = mraw * p.scale_log2;   // scale_log2 > 0
        // The reference max m moves only when the tile max exceeds it by more than
        // 2^8 (log2 units): P = exp2(s - m) <= 256 then, exact enough in f32 sums and
        // bf16 / f16 P, and the output is rescaled far less often. The result is the
        // same softmax: numerator and denominator share the reference.
        const bool move = mt > m + 8.f;
        const float m_new = move ? mt : m;
        const float alpha = (move && m != -INFINITY) ? exp2f(m - m_new) : 1.f;
        // exponentials before waiting for the previous P . V: they overlap its MMAs
        float sum8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) sum8[e] = 0.f;
        const float mneg = m_new == -INFINITY ? 0.f : -m_new;   // a row with no key yet: all -inf -> 0
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float pv = ex2_approx(fmaf(__uint_as_float(sr[c][i]), p.scale_log2, mneg));
            sum8[i & 7] += pv;
            sr[c][i] = __float_as_uint(pv);
          }
#pragma unroll
        for (int e = 0; e < 4; ++e) sum8[e] += sum8[e + 4];
        const float rs = (sum8[0] + sum8[1]) + (sum8[2] + sum8[3]);
        l = l * alpha + rs;
        m = m_new;
        // the previous P . V must be complete before P is overwritten and O rescaled
        if (j > 0 && !mbar_wait(&ctl->o_done, (j - 1) & 1, abort_flag, p.status)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {   // 8 keys = one 16-byte chunk
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
              w[e] = pack2<T>(__uint_as_float(sr[c][8 * g + 2 * e]), __uint_as_float(sr[c][8 * g + 2 * e + 1]));
            const int chunk = (4 * c + g) & 7, half = c >> 1;
            *reinterpret_cast<uint4*>(prow + half * kHalfBytes + ((chunk ^ (row & 7)) << 4)) =
                make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
        if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
          // rescale this warp's rows of the running output
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tmem_ld32_issue(lane_base + kOCol + 32 * c, o);
            tmem_wait(o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(lane_base + kOCol + 32 * c, o);
          }
          tmem_st_wait();
        }
        fence_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->p_full);
      }
      if (ok && mbar_wait(&ctl->o_done, (nt - 1) & 1, abort_flag, p.status)) {
        tc_fence_after();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        T* orow = reinterpret_cast<T*>(p.out) + (int64_t)(start + qi) * p.o_s0 + (int64_t)hq * p.o_s1;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32_issue(lane_base + kOCol + 32 * c, o);
          tmem_wait(o);
          if (qi < L) {
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              uint4 u;
              u.x = pack2<T>(__uint_as_float(o[8 * g + 0]) * inv, __uint_as_float(o[8 * g + 1]) * inv);
              u.y = pack2<T>(__uint_as_float(o[8 * g + 2]) * inv, __uint_as_float(o[8 * g + 3]) * inv);
              u.z = pack2<T>(__uint_as_float(o[8 * g + 4]) * inv, __uint_as_float(o[8 * g + 5]) * inv);
              u.w = pack2<T>(__uint_as_float(o[8 * g + 6]) * inv, __uint_as_float(o[8 * g + 7]) * inv);
              *reinterpret_cast<uint4*>(orow + 32 * c + 8 * g) = u;
            }
          }
        }
      }
    }
  }

  // ---- teardown (the producer and the issuer drained their copies and MMAs) ----
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

int launch_prefill(const CUtensorMap& tm_q, const CUtensorMap& tm_k, const CUtensorMap& tm_v, const PrefillParams& p,
                   int q_tiles, cudaStream_t stream) {
  if (q_tiles <= 0 || p.num_heads <= 0) return STARKV_OK;
  const dim3 grid(q_tiles, p.num_heads);
  if (p.dtype == STARKV_BF16) {
    if (cudaFuncSetAttribute(prefill_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmemBytes) != cudaSuccess)
      return STARKV_ECUDA;
    prefill_kernel<__nv_bfloat16><<<grid, kThreads, kSmemBytes, stream>>>(tm_q, tm_k, tm_v, p);
  } else {
    if (cudaFuncSetAttribute(prefill_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
        cudaSuccess)
      return STARKV_ECUDA;
    prefill_kernel<__half><<<grid, kThreads, kSmemBytes, stream>>>(tm_q, tm_k, tm_v, p);
  }
  return cudaGetLastError() == cudaSuccess ? STARKV_OK : STARKV_ECUDA;
}

}  // namespace starkv
