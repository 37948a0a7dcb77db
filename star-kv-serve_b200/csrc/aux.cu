// Small kernels around the two tensor-core passes:
//   fold_kernel   AB = fold(q, U) * scale (paged_quant.py:223-255), the f16 copy of
//                 the rotary table rows, and per-call accumulator init;
//   lift_kernel   out[b,h,:] = pv[b,h,:] / l[b,h] . v_up_by_q[h] (paged_decode.py:222-226), for
//                 layouts the cluster lift (lift.cu) does not take (f32 or strided v_up);
//   pack_k/v      3.2-bit write side (paged_quant.py:139-216), bit-exact with
//                 kv_quant._q (kv_quant.py:111-121): IEEE division, round half even;
//   cache_write   bf16 cache write (attention.py:179-185).
#include "starkv_common.cuh"
#include "starkv_kernels.h"

namespace starkv {

// ---------------------------------------------------------------------------
// fold + rotary table + init (one launch)
// ---------------------------------------------------------------------------

constexpr int kFoldLanes = 64;   // K lanes per fold block
constexpr int kFoldRows = 16;    // lanes one pass of the block covers (8 threads x 8 values each)
constexpr int kFoldSeqs = 4;     // (sequence, query head of the group) pairs per fold block
constexpr int kFoldQHeads = 8;   // query rows staged per pair (the heads of 64 lanes)
constexpr int kFoldUPitch = 128 + 8;   // staged k_up row (elements): 16-byte aligned, banks spread

// 8 consecutive elements (stride `st`) as floats: one or two 16-byte loads when the
// run is contiguous and aligned, scalar loads otherwise.
template <class T>
__device__ __forceinline__ void load8(const T* p, int64_t st, float (&v)[8]) {
  if (st == 1 && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
    if constexpr (sizeof(T) == 2) {
      const uint4 u = *reinterpret_cast<const uint4*>(p);
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = to_f32(e[k]);
    } else {
      const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = to_f32(p[(int64_t)k * st]);
  }
}

template <class TQ, class TU>
__global__ void __launch_bounds__(128) fold_kernel(const FoldParams p, int n_fold_blocks, int n_cs_blocks) {
  const int bid = blockIdx.x;
  if (bid < n_fold_blocks) {
    // block -> (64 lanes, kFoldSeqs (b, j) pairs). The lanes' k_up rows are staged
    // once and serve every pair; each pair's query rows of the lanes' heads are
    // staged too, so global memory sees each input about once. thread -> 8
    // consecutive i of 0..63 of lanes lr, lr + 16, lr + 32, lr + 48.
    __shared__ int head_of[kFoldLanes];
    __shared__ int hmin_s;
    __shared__ __align__(16) TU u_s[kFoldLanes][kFoldUPitch];
    __shared__ __align__(16) float q_s[kFoldQHeads][128];
    const int lane_tiles = (p.k_width + kFoldLanes - 1) / kFoldLanes;
    const int r0 = (bid % lane_tiles) * kFoldLanes;
    const int bj0 = (bid / lane_tiles) * kFoldSeqs;
    const int bj1 = min(bj0 + kFoldSeqs, p.n * p.group);
    if (threadIdx.x < kFoldLanes) {
      const int r = r0 + threadIdx.x;
      int head = -1;
      if (r < p.k_width) {
        if (p.head_of_lane) {
          head = p.head_of_lane[r];
          if (head < 0 || head >= p.num_kv_heads) {
            record_status(p.status, STARKV_EBOUNDS);
            head = -1;
          }
        } else {
          for (int h = 0; h < p.num_kv_heads; ++h) {
            const int off = p.k_head_offsets[h], rk = p.k_ranks[h];
            if (r >= off && r < off + ((rk + 15) & ~15)) {
              head = (r - off) < rk ? h : -1;   // lanes past the rank get zero rows
              break;
            }
          }
        }
      }
      head_of[threadIdx.x] = head;
    }
    {
      // k_up rows of the 64 lanes (zero past k_width): thread -> (row, half of 64 values)
      const int row = threadIdx.x >> 1, c0 = (threadIdx.x & 1) * 64;
      const int r = r0 + row;
      const TU* up = reinterpret_cast<const TU*>(p.k_up) + (int64_t)r * p.ku_s0 + (int64_t)c0 * p.ku_s1;
      const bool vec = p.ku_s1 == 1 && (reinterpret_cast<uintptr_t>(up) & 15) == 0;
#pragma unroll
      for (int k = 0; k < 64; k += 16 / (int)sizeof(TU)) {
        constexpr int kPer = 16 / (int)sizeof(TU);
        if (r < p.k_width && vec) {
          *reinterpret_cast<uint4*>(&u_s[row][c0 + k]) = *reinterpret_cast<const uint4*>(up + k);
        } else {
#pragma unroll
          for (int e = 0; e < kPer; ++e) u_s[row][c0 + k + e] = r < p.k_width ? up[(int64_t)(k + e) * p.ku_s1] : TU{};
        }
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int m = p.num_kv_heads;
      for (int i = 0; i < kFoldLanes; ++i)
        if (head_of[i] >= 0) m = min(m, head_of[i]);
      hmin_s = m;
    }
    __syncthreads();
    const int hmin = hmin_s;
    const int i0 = (threadIdx.x & 7) * 8;
    for (int bj = bj0; bj < bj1; ++bj) {
      const int b = bj / p.group, j = bj % p.group;
      // query rows of heads hmin .. hmin + 7 (the lanes' heads, lanes being in head order)
      for (int e = threadIdx.x; e < kFoldQHeads * 16; e += blockDim.x) {
        const int hh = e >> 4, c = (e & 15) * 8;
        const int h = hmin + hh;
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (h < p.num_kv_heads) {
          const TQ* qp = reinterpret_cast<const TQ*>(p.q) + (int64_t)b * p.q_s0 + (int64_t)(h * p.group + j) * p.q_s1;
          load8(qp + (int64_t)c * p.q_s2, p.q_s2, v);
        }
        *reinterpret_cast<float4*>(&q_s[hh][c]) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4*>(&q_s[hh][c + 4]) = make_float4(v[4], v[5], v[6], v[7]);
      }
      __syncthreads();
#pragma unroll
      for (int pass = 0; pass < kFoldLanes / kFoldRows; ++pass) {
        const int lr = pass * kFoldRows + (threadIdx.x >> 3);
        const int r = r0 + lr;
        if (r >= p.k_width) break;
        const int head = head_of[lr];
        __align__(16) __half av[8], bv[8];
        if (head < 0) {
#pragma unroll
          for (int k = 0; k < 8; ++k) av[k] = bv[k] = __float2half_rn(0.f);
        } else {
          float q0[8], q1[8], u0[8], u1[8];
          if (head - hmin < kFoldQHeads) {
            const float* qr = q_s[head - hmin];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              q0[k] = qr[i0 + k];
              q1[k] = qr[i0 + 64 + k];
            }
          } else {   // lanes of more than 8 heads in one block (not from k_tables): read directly
            const TQ* qp = reinterpret_cast<const TQ*>(p.q) + (int64_t)b * p.q_s0 + (int64_t)(head * p.group + j) * p.q_s1;
            load8(qp + (int64_t)i0 * p.q_s2, p.q_s2, q0);
            load8(qp + (int64_t)(i0 + 64) * p.q_s2, p.q_s2, q1);
          }
          load8(&u_s[lr][i0], 1, u0);
          load8(&u_s[lr][i0 + 64], 1, u1);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float a0 = q0[k], a1 = q1[k], w0 = u0[k], w1 = u1[k];
            av[k] = __float2half_rn((a0 * w0 + a1 * w1) * p.scale);
            bv[k] = __float2half_rn((a1 * w0 - a0 * w1) * p.scale);
          }
        }
        if (p.ab_image) {
          // the 128-byte-swizzled K-major tile the score MMA reads as its B operand
          const int nc = (p.k_width + 127) / 128;
          const int c = r >> 7, half = (r >> 6) & 1, i = r & 63;
          __half* blk = p.ab + ((((int64_t)bj * nc + c) * 2 + half) << 13);   // 8192 halves per block
          const int unit = (threadIdx.x & 7) ^ (i & 7);
          *reinterpret_cast<uint4*>(blk + i * 64 + unit * 8) = *reinterpret_cast<const uint4*>(av);
          *reinterpret_cast<uint4*>(blk + 4096 + i * 64 + unit * 8) = *reinterpret_cast<const uint4*>(bv);
        } else {
          __half* dst = p.ab + ((int64_t)bj * p.k_width + r) * 128;
          *reinterpret_cast<uint4*>(dst + i0) = *reinterpret_cast<const uint4*>(av);
          *reinterpret_cast<uint4*>(dst + 64 + i0) = *reinterpret_cast<const uint4*>(bv);
        }
      }
      __syncthreads();   // q_s is rewritten for the next pair
    }
    return;
  }
  if (bid < n_fold_blocks + n_cs_blocks) {
    // rotary table rows -> f16 (zero past the table / max_seq_len), written as the
    // 128-byte-swizzled K-major tiles the score MMA reads as its A operand; thread =
    // one 16-byte unit (8 columns) of a row
    const int64_t e = (int64_t)(bid - n_fold_blocks) * 128 + threadIdx.x;
    const int64_t row = e >> 4;
    const int u = (int)(e & 15), col0 = u * 8;
    if (row >= p.l_pad) return;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (row < p.cs_rows && row < p.max_seq_len) {
      with_float_type(p.cs_dtype, [&](auto tc) {
        using TC = decltype(tc);
        load8(reinterpret_cast<const TC*>(p.cs) + row * p.cs_s0 + (int64_t)col0 * p.cs_s1, p.cs_s1, v);
      });
    }
    __align__(16) __half hv[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) hv[k] = __float2half_rn(v[k]);
    const int t = (int)(row & 127), kh = u >> 3, unit = (u & 7) ^ (t & 7);
    *reinterpret_cast<uint4*>(p.cs16 + ((row >> 7) << 14) + kh * 8192 + t * 64 + unit * 8) =
        *reinterpret_cast<const uint4*>(hv);
    return;
  }
  // init: sequence max = -inf, pv = 0
  const int64_t t = (int64_t)(bid - n_fold_blocks - n_cs_blocks) * 128 + threadIdx.x;
  const int64_t stride = (int64_t)(gridDim.x - n_fold_blocks - n_cs_blocks) * 128;
  for (int64_t k = t; k < p.m_count; k += stride) {
    p.m_seq[k] = -INFINITY;
    p.l_seq[k] = 0.f;
  }
  float4* pv4 = reinterpret_cast<float4*>(p.pv);
  const int64_t n4 = p.pv_count >> 2;
  for (int64_t k = t; k < n4; k += stride) pv4[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t k = (n4 << 2) + t; k < p.pv_count; k += stride) p.pv[k] = 0.f;
}

int launch_fold(const FoldParams& p, bool quant, cudaStream_t stream) {
  (void)quant;
  const int lane_tiles = (p.k_width + kFoldLanes - 1) / kFoldLanes;
  const int n_fold = lane_tiles * ((p.n * p.group + kFoldSeqs - 1) / kFoldSeqs);
  const int n_cs = (int)(((int64_t)p.l_pad * 16 + 127) / 128);   // one thread per 16-byte unit
  // the accumulator clear: up to 8 blocks per SM of float4 stores in a grid-stride loop
  const int64_t init_work = p.m_count + (p.pv_count >> 2);
  const int n_init = (int)(init_work < 1184 * 128 ? (init_work + 127) / 128 + 1 : 1184);
  with_float_type(p.q_dtype, [&](auto tq) {
    with_float_type(p.k_up_dtype, [&](auto tu) {
      fold_kernel<decltype(tq), decltype(tu)><<<n_fold + n_cs + n_init, 128, 0, stream>>>(p, n_fold, n_cs);
    });
  });
  return cudaGetLastError() == cudaSuccess ? STARKV_OK : STARKV_ECUDA;
}

// ---------------------------------------------------------------------------
// lift: out[b, h, :] = (pv[b, h, :] / l[b, h]) . v_up_by_q[h]
//
// Per head a [n x rv] x [rv x 128] product on mma.sync m16n8k16 (bf16 in, f32
// accumulate). The normalised pv row is split into bf16 hi + lo parts (two MMAs)
// so the product keeps ~16 mantissa bits, well past the reference's bf16 cast
// (paged_decode.py:225). Block = (head, 32 output columns, 32 sequences), four
// groups of two warps splitting the V channels; warp w of a group owns sequences
// [16w, 16w+16); v_up_by_q tiles are staged through shared memory and read with
// ldmatrix.trans. (64 sequences per block left one 512-thread block per SM and the
// kernel latency-bound.)
// ---------------------------------------------------------------------------

constexpr int kLiftBT = 32;    // sequences per block
constexpr int kLiftVT = 64;    // V channels staged per step
constexpr int kLiftLd = 40;    // staged row stride (elements): 80 B, conflict-free ldmatrix

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

constexpr int kLiftGroups = 4;   // warp groups splitting the V channels of a block
constexpr int kLiftGT = 64;      // threads per group (kLiftBT / 16 warps)
constexpr int kLiftPvtFloats = kLiftBT * (kLiftVT + 4);
constexpr int kLiftGroupBytes = kLiftPvtFloats * 4 + kLiftVT * kLiftLd * 2;
constexpr int kLiftSmem = kLiftGroups * kLiftGroupBytes + kLiftBT * 4;

template <class TV, bool VEC>
__global__ void __launch_bounds__(kLiftGT * kLiftGroups) lift_kernel(const LiftParams p) {
  const int h = blockIdx.x;
  const int d0 = blockIdx.y * 32;
  const int b0 = blockIdx.z * kLiftBT;
  const int grp = threadIdx.x / kLiftGT;        // this group's V steps: grp, grp + 4, ...
  const int tid = threadIdx.x % kLiftGT, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  extern __shared__ __align__(16) uint8_t lift_smem[];
  float (*pvt)[kLiftVT + 4] = reinterpret_cast<float (*)[kLiftVT + 4]>(lift_smem + grp * kLiftGroupBytes);   // [b][v]
  __nv_bfloat16 (*vt)[kLiftLd] =
      reinterpret_cast<__nv_bfloat16 (*)[kLiftLd]>(lift_smem + grp * kLiftGroupBytes + kLiftPvtFloats * 4);  // [v][d]
  float* inv_l = reinterpret_cast<float*>(lift_smem + kLiftGroups * kLiftGroupBytes);
  if (threadIdx.x < kLiftBT) {
    const int b = b0 + threadIdx.x;
    if (p.l_seq) {
      const float l = b < p.n ? p.l_seq[(int64_t)b * p.num_heads + h] : 0.f;
      inv_l[threadIdx.x] = l > 0.f ? 1.f / l : 0.f;   // empty sequence -> 0, as the reference
    } else {
      inv_l[threadIdx.x] = 1.f;                        // partial (context-parallel) output: unnormalised
    }
  }
  // per-thread share of one staged step: 8 x float4 of pv (32 rows x 16), and 2048
  // v_up elements (64 v x 32 d): 4 x 8 consecutive d (VEC: 16-byte loads) or 32 scalars
  constexpr int kVu = VEC ? 4 : 32;
  float4 rp[8];
  uint4 rvv[VEC ? 4 : 1];
  TV rv[VEC ? 1 : 32];
  int vnext = 0;
  auto fetch = [&](int v0) {
    vnext = v0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = tid + kLiftGT * i;
      const int bb = e >> 4, vq = (e & 15) * 4;
      const int b = min(b0 + bb, p.n - 1);
      rp[i] = *reinterpret_cast<const float4*>(p.pv + ((int64_t)b * p.num_heads + h) * p.pv_stride + v0 + vq);
    }
    if constexpr (VEC) {
#pragma unroll
      for (int i = 0; i < kVu; ++i) {
        const int e = tid + kLiftGT * i;       // 256 = 64 v x 4 runs of 8 d
        const int v = min(v0 + (e >> 2), p.v_rank - 1);
        rvv[i] = *reinterpret_cast<const uint4*>(reinterpret_cast<const TV*>(p.v_up) + (int64_t)h * p.vu_s0 +
                                                 (int64_t)v * p.vu_s1 + d0 + (e & 3) * 8);
      }
    } else {
#pragma unroll
      for (int i = 0; i < kVu; ++i) {
        const int e = tid + kLiftGT * i;       // 2048 = 64 v x 32 d
        const int vv = e >> 5, dd = e & 31;
        const int v = v0 + vv;
        const int64_t o = (int64_t)h * p.vu_s0 + (int64_t)min(v, p.v_rank - 1) * p.vu_s1 +
                          (int64_t)min(d0 + dd, p.head_dim - 1) * p.vu_s2;
        rv[i] = reinterpret_cast<const TV*>(p.v_up)[o];   // raw load; range masked at the stash
      }
    }
  };
  int vbase = 0;   // first V channel of the step held in rv
  auto stash = [&]() {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = tid + kLiftGT * i;
      *reinterpret_cast<float4*>(&pvt[e >> 4][(e & 15) * 4]) = rp[i];
    }
    if constexpr (VEC) {
#pragma unroll
      for (int i = 0; i < kVu; ++i) {
        const int e = tid + kLiftGT * i;
        const int vv = e >> 2, dq = (e & 3) * 8;
        const bool in = vbase + vv < p.v_rank;
        const TV* x = reinterpret_cast<const TV*>(&rvv[i]);
        __align__(16) __nv_bfloat16 o[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = __float2bfloat16_rn(in ? to_f32(x[k]) : 0.f);
        *reinterpret_cast<uint4*>(&vt[vv][dq]) = *reinterpret_cast<const uint4*>(o);
      }
    } else {
#pragma unroll
      for (int i = 0; i < kVu; ++i) {
        const int e = tid + kLiftGT * i;
        const int vv = e >> 5, dd = e & 31;
        const bool in = (vbase + vv < p.v_rank) && (d0 + dd < p.head_dim);
        vt[vv][dd] = __float2bfloat16_rn(in ? to_f32(rv[i]) : 0.f);
      }
    }
  };
  // named barrier per group (ids 1..4)
  auto group_sync = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(grp + 1), "n"(kLiftGT) : "memory"); };
  const int rA = 16 * warp + g, rB = rA + 8;   // rows within the block's 64 sequences
  float acc[4][4] = {};
  const int vstride = kLiftVT * kLiftGroups;
  const int vfirst = kLiftVT * grp;
  if (vfirst < p.v_rank) fetch(vfirst);
  __syncthreads();   // inv_l ready
  const float sA = inv_l[rA], sB = inv_l[rB];
  for (int v0 = vfirst; v0 < p.v_rank; v0 += vstride) {
    group_sync();
    vbase = vnext;
    stash();
    group_sync();
    if (v0 + vstride < p.v_rank) fetch(v0 + vstride);   // next step's loads overlap this step's MMAs
#pragma unroll
    for (int ks = 0; ks < kLiftVT / 16; ++ks) {
      const int c0 = ks * 16 + 2 * t, c1 = c0 + 8;
      const float2 xa0 = *reinterpret_cast<const float2*>(&pvt[rA][c0]);
      const float2 xb0 = *reinterpret_cast<const float2*>(&pvt[rB][c0]);
      const float2 xa1 = *reinterpret_cast<const float2*>(&pvt[rA][c1]);
      const float2 xb1 = *reinterpret_cast<const float2*>(&pvt[rB][c1]);
      const float x[8] = {xa0.x * sA, xa0.y * sA, xb0.x * sB, xb0.y * sB,
                          xa1.x * sA, xa1.y * sA, xb1.x * sB, xb1.y * sB};
      uint32_t hi[4], lo[4];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const float e0 = x[2 * jj], e1 = x[2 * jj + 1];
        const float h0 = __bfloat162float(__float2bfloat16_rn(e0)), h1 = __bfloat162float(__float2bfloat16_rn(e1));
        hi[jj] = pack_bf16x2(h0, h1);
        lo[jj] = pack_bf16x2(e0 - h0, e1 - h1);
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        // B fragment (k = v, n = d) from the staged [v][d] tile, transposed by ldmatrix
        uint32_t b0r, b1r;
        const __nv_bfloat16* rowp = &vt[ks * 16 + (lane & 15)][nt * 8];
        asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];"
                     : "=r"(b0r), "=r"(b1r)
                     : "r"(smem_u32(rowp)));
        mma_bf16_16816(acc[nt], hi, b0r, b1r);
        mma_bf16_16816(acc[nt], lo, b0r, b1r);
      }
    }
  }
  // reduce the groups' partial sums through shared memory (reusing the staging area)
  __syncthreads();
  float* red = reinterpret_cast<float*>(lift_smem);   // [group - 1][16][kLiftGT]
  if (grp > 0) {
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int k = 0; k < 4; ++k) red[((grp - 1) * 16 + nt * 4 + k) * kLiftGT + tid] = acc[nt][k];
  }
  __syncthreads();
  if (grp > 0) return;
#pragma unroll
  for (int gg = 0; gg < kLiftGroups - 1; ++gg)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int k = 0; k < 4; ++k) acc[nt][k] += red[(gg * 16 + nt * 4 + k) * kLiftGT + tid];
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    const int d = d0 + nt * 8 + 2 * t;
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      const int b = b0 + (jj ? rB : rA);
      if (b >= p.n) continue;
      const int64_t o = (int64_t)b * p.o_s0 + (int64_t)h * p.o_s1;
      if (d < p.head_dim) store_elem(p.out, o + (int64_t)d * p.o_s2, p.out_dtype, acc[nt][2 * jj]);
      if (d + 1 < p.head_dim) store_elem(p.out, o + (int64_t)(d + 1) * p.o_s2, p.out_dtype, acc[nt][2 * jj + 1]);
    }
  }
}

int launch_lift(const LiftParams& p, cudaStream_t stream) {
  const int fast = launch_lift_cluster(p, stream);   // the common layout (lift.cu)
  if (fast >= 0) return fast;
  dim3 grid(p.num_heads, (p.head_dim + 31) / 32, (p.n + kLiftBT - 1) / kLiftBT);
  // 16-byte v_up loads: 2-byte elements, unit stride along d, every run of 8 aligned
  const int es = p.v_up_dtype == STARKV_F32 ? 4 : 2;
  const bool vec = es == 2 && p.vu_s2 == 1 && p.head_dim % 32 == 0 && p.vu_s0 % 8 == 0 && p.vu_s1 % 8 == 0 &&
                   (reinterpret_cast<uintptr_t>(p.v_up) & 15) == 0;
  const void* fn = p.v_up_dtype == STARKV_BF16 ? (vec ? (const void*)lift_kernel<__nv_bfloat16, true>
                                                      : (const void*)lift_kernel<__nv_bfloat16, false>)
                   : p.v_up_dtype == STARKV_F16 ? (vec ? (const void*)lift_kernel<__half, true>
                                                       : (const void*)lift_kernel<__half, false>)
                                                : (const void*)lift_kernel<float, false>;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kLiftSmem) != cudaSuccess)
    return STARKV_ECUDA;
  void* args[] = {const_cast<LiftParams*>(&p)};
  if (cudaLaunchKernel(fn, grid, dim3(kLiftGT * kLiftGroups), args, kLiftSmem, stream) != cudaSuccess)
    return STARKV_ECUDA;
  return cudaGetLastError() == cudaSuccess ? STARKV_OK : STARKV_ECUDA;
}

// ---------------------------------------------------------------------------
// 3.2-bit packing (write side)
// ---------------------------------------------------------------------------

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float m = red[0];
  for (int i = 1; i < nw; ++i) m = fmaxf(m, red[i]);
  return m;
}

// code = clamp(rint(x / s), -(qmax+1), qmax) + 8 with IEEE division (kv_quant.py:119-120)
__device__ __forceinline__ uint32_t quant_code(float x, float s, float qmax) {
  float q = rintf(__fdiv_rn(x, s));
  q = fminf(fmaxf(q, -(qmax + 1.f)), qmax);
  return (uint32_t)(int)(q + 8.f);
}

__device__ __forceinline__ uint8_t* slot_row(const StarKVPackArgs& a, int i, bool& ok) {
  int64_t slot = load_slot(a.slot_mapping, i, a.slot_dtype);
  if (slot < 0) slot = 0;   // CUDA-graph padding tokens -> reserved null block
  const int64_t blk = slot / a.block_size;
  ok = blk < a.num_blocks;
  if (!ok) {
    record_status(a.status, STARKV_EBOUNDS);
    return nullptr;
  }
  return reinterpret_cast<uint8_t*>(a.cache) + blk * a.cache_stride[0] + (slot % a.block_size) * a.cache_stride[1];
}

// one block per (token, K head) with 128 threads, plus one block per token for V
__global__ void __launch_bounds__(256) pack_kernel(const StarKVPackArgs a) {
  __shared__ float red[8];
  const int i = blockIdx.x;
  const int h = blockIdx.y;
  bool ok;
  uint8_t* row = slot_row(a, i, ok);
  if (!ok) return;
  const float eps = 1e-5f;
  if (h < a.num_kv_heads) {
    const int R = a.k_ranks[h], NOUT = a.k_nouts[h], off = a.k_offsets[h];
    const int WH = (R + 15) & ~15;   // stored width; lanes past R carry the codes given (zero)
    if (R <= 0 || WH > 128 || off < 0 || (off & 15) || off + WH > a.k_width || NOUT < 0 || NOUT > R) {
      if (threadIdx.x == 0) record_status(a.status, STARKV_EINVAL);
      return;
    }
    const int t = threadIdx.x;
    float x = 0.f;
    if (t < WH && t < 128) x = load_elem(a.k_codes, (int64_t)i * a.k_stride0 + off + t, a.k_dtype);
    const float a_out = block_max((t < NOUT) ? fabsf(x) : 0.f, red);
    const float a_in = block_max((t >= NOUT && t < WH) ? fabsf(x) : 0.f, red);
    const float s_out = __fdiv_rn(fmaxf(a_out, eps), 7.f);
    const float s_in = __fdiv_rn(fmaxf(a_in, eps), 3.f);
    const uint32_t code = (t < NOUT) ? quant_code(x, s_out, 7.f) : quant_code(x, s_in, 3.f);
    const uint32_t hi = __shfl_down_sync(0xffffffffu, code, 1);
    if (t < WH && (t & 1) == 0) row[off / 2 + t / 2] = (uint8_t)(code | (hi << 4));
    if (t == 0) {
      __nv_bfloat16* ks = reinterpret_cast<__nv_bfloat16*>(row + a.ks_off) + 2 * h;
      ks[0] = __float2bfloat16_rn(NOUT > 0 ? s_out : 1.f);
      ks[1] = __float2bfloat16_rn(s_in);
    }
    return;
  }
  // V: outlier block [0, nout) at 4 bits, inlier block [nout, R) at 3 bits
  const int R = a.v_rank, NOUT = a.v_nout;
  float mo = 0.f, mi = 0.f;
  for (int c = threadIdx.x; c < R; c += blockDim.x) {
    const float x = fabsf(load_elem(a.v_codes, (int64_t)i * a.v_stride0 + c, a.v_dtype));
    if (c < NOUT) mo = fmaxf(mo, x); else mi = fmaxf(mi, x);
  }
  const float a_out = block_max(mo, red);
  const float a_in = block_max(mi, red);
  const float s_out = __fdiv_rn(fmaxf(a_out, eps), 7.f);
  const float s_in = __fdiv_rn(fmaxf(a_in, eps), 3.f);
  for (int j = threadIdx.x; j < a.v_bytes; j += blockDim.x) {
    const bool outl = j < a.v_nbo;
    const int c_lo = outl ? 2 * j : NOUT + 2 * (j - a.v_nbo);
    const int c_end = outl ? NOUT : R;
    const float s = outl ? s_out : s_in;
    const float qm = outl ? 7.f : 3.f;
    uint32_t nl = 8, nh = 8;   // pad nibble
    if (c_lo < c_end) nl = quant_code(load_elem(a.v_codes, (int64_t)i * a.v_stride0 + c_lo, a.v_dtype), s, qm);
    if (c_lo + 1 < c_end) nh = quant_code(load_elem(a.v_codes, (int64_t)i * a.v_stride0 + c_lo + 1, a.v_dtype), s, qm);
    row[a.vq_off + j] = (uint8_t)(nl | (nh << 4));
  }
  if (threadIdx.x == 0) {
    __nv_bfloat16* vs = reinterpret_cast<__nv_bfloat16*>(row + a.vs_off);
    vs[0] = __float2bfloat16_rn(NOUT > 0 ? s_out : 1.f);
    vs[1] = __float2bfloat16_rn(s_in);
  }
}

}  // namespace starkv

extern "C" int starkv_pack_kv_q32(const StarKVPackArgs* a, void* stream) {
  using namespace starkv;
  if (!a || a->n < 0 || a->num_kv_heads <= 0 || a->block_size <= 0 || a->num_blocks <= 0) return STARKV_EINVAL;
  if (a->n == 0) return STARKV_OK;
  if (!a->k_codes || !a->v_codes || !a->cache || !a->slot_mapping || !a->k_ranks || !a->k_offsets || !a->k_nouts)
    return STARKV_EINVAL;
  if (a->slot_dtype != STARKV_I32 && a->slot_dtype != STARKV_I64) return STARKV_EDTYPE;
  for (int dt : {a->k_dtype, a->v_dtype})
    if (dt != STARKV_BF16 && dt != STARKV_F16 && dt != STARKV_F32) return STARKV_EDTYPE;
  if (a->v_bytes <= 0 || a->v_nbo < 0 || a->v_nout < 0 || a->v_nout > a->v_rank) return STARKV_EINVAL;
  dim3 grid(a->n, a->num_kv_heads + 1);
  pack_kernel<<<grid, 128, 0, (cudaStream_t)stream>>>(*a);
  return cudaGetLastError() == cudaSuccess ? STARKV_OK : STARKV_ECUDA;
}

// ---------------------------------------------------------------------------
// bf16 cache write: cache[slot // bs, slot % bs] = cat(key, value)
// ---------------------------------------------------------------------------

namespace starkv {
__global__ void __launch_bounds__(256) cache_write_kernel(const StarKVCacheWriteArgs a) {
  const int i = blockIdx.x;
  int64_t slot = load_slot(a.slot_mapping, i, a.slot_dtype);
  if (slot < 0) slot = 0;
  const int64_t blk = slot / a.block_size;
  if (blk >= a.num_blocks) {
    record_status(a.status, STARKV_EBOUNDS);
    return;
  }
  const int64_t base = blk * a.cache_stride[0] + (slot % a.block_size) * a.cache_stride[1];
  const int width = a.k_width + a.v_rank;
  for (int c = threadIdx.x; c < width; c += blockDim.x) {
    const float v = c < a.k_width ? load_elem(a.key, (int64_t)i * a.key_stride0 + c, a.key_dtype)
                                  : load_elem(a.value, (int64_t)i * a.value_stride0 + (c - a.k_width), a.value_dtype);
    store_elem(a.cache, base + (int64_t)c * a.cache_stride[2], a.cache_dtype, v);
  }
}
}  // namespace starkv

extern "C" int starkv_cache_write_bf16(const StarKVCacheWriteArgs* a, void* stream) {
  using namespace starkv;
  if (!a || a->n < 0 || a->block_size <= 0 || a->num_blocks <= 0 || a->k_width < 0 || a->v_rank < 0)
    return STARKV_EINVAL;
  if (a->n == 0) return STARKV_OK;
  if (!a->key || !a->value || !a->cache || !a->slot_mapping) return STARKV_EINVAL;
  if (a->slot_dtype != STARKV_I32 && a->slot_dtype != STARKV_I64) return STARKV_EDTYPE;
  if (a->cache_dtype != STARKV_BF16 && a->cache_dtype != STARKV_F16) return STARKV_EDTYPE;
  cache_write_kernel<<<a->n, 256, 0, (cudaStream_t)stream>>>(*a);
  return cudaGetLastError() == cudaSuccess ? STARKV_OK : STARKV_ECUDA;
}

// ---------------------------------------------------------------------------
// context-parallel combine: parts = world packed partials, each
//   [n, H, 128] out_r | [n, H] m_r | [n, H] l_r   (f32, rank-major)
// out[b, h, :] = sum_r exp(m_r - M) out_r / sum_r exp(m_r - M) l_r, M = max_r m_r
// (0 when no rank holds a token of the sequence, as the reference's empty case)
// ---------------------------------------------------------------------------
namespace starkv {

__global__ void __launch_bounds__(128) cp_combine_kernel(const float* __restrict__ parts, int world, int n, int H,
                                                         void* out, int64_t o0, int64_t o1, int64_t o2, int out_dtype) {
  const int bh = blockIdx.x;                 // (b, h)
  const int d = threadIdx.x;                 // 0..127
  const int64_t nh = (int64_t)n * H;
  const int64_t part = nh * 130;
  float M = -INFINITY;
  for (int r = 0; r < world; ++r) M = fmaxf(M, parts[r * part + nh * 128 + bh]);
  float num = 0.f, den = 0.f;
  if (M > -INFINITY) {
    for (int r = 0; r < world; ++r) {
      const float* pr = parts + r * part;
      const float s = __expf(pr[nh * 128 + bh] - M);
      num += s * pr[(int64_t)bh * 128 + d];
      den += s * pr[nh * 129 + bh];
    }
  }
  const int b = bh / H, h = bh - b * H;
  store_elem(out, (int64_t)b * o0 + (int64_t)h * o1 + (int64_t)d * o2, out_dtype, den > 0.f ? num / den : 0.f);
}

}  // namespace starkv

extern "C" int starkv_cp_combine(const float* parts, int32_t world, int32_t n, int32_t num_heads, void* out,
                                 const int64_t out_stride[3], int32_t out_dtype, void* stream) {
  using namespace starkv;
  if (!parts || !out || !out_stride || world < 1 || n < 0 || num_heads <= 0) return STARKV_EINVAL;
  if (out_dtype != STARKV_BF16 && out_dtype != STARKV_F16 && out_dtype != STARKV_F32) return STARKV_EDTYPE;
  if (n == 0) return STARKV_OK;
  cp_combine_kernel<<<n * num_heads, 128, 0, (cudaStream_t)stream>>>(parts, world, n, num_heads, out, out_stride[0],
                                                                     out_stride[1], out_stride[2], out_dtype);
  return cudaGetLastError() == cudaSuccess ? STARKV_OK : STARKV_ECUDA;
}

// ---------------------------------------------------------------------------
// Self-test of the bounded pipeline wait: one thread waits on an mbarrier that
// nothing arrives on; the wait must give up after its poll limit, record
// STARKV_ETIMEOUT in the status word and return, leaving the context usable.
// ---------------------------------------------------------------------------
namespace starkv {
__global__ void wait_timeout_kernel(int32_t* status) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && mbar_wait(&bar, 0, &abort_flag, status)) record_status(status, STARKV_EINVAL);
}
}  // namespace starkv

extern "C" int starkv_selftest_wait_timeout(int32_t* status, void* stream) {
  if (!status) return STARKV_EINVAL;
  starkv::wait_timeout_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(status);
  return cudaGetLastError() == cudaSuccess ? STARKV_OK : STARKV_ECUDA;
}
