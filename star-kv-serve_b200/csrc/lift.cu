// Lift of the P.V sums to head_dim, the common layout (2-byte v_up_by_q with
// unit stride along head_dim, head_dim 128):
//   out[b, h, :] = (pv[b, h, :] / l[b, h]) . v_up_by_q[h]     (paged_decode.py:222-226)
//
// Per head a [n x rv] x [rv x 128] product. A cluster of 4 CTAs splits the V
// channels of one (head, 32 sequences) tile, so each CTA streams a quarter of
// that head's pv rows (f32) and v_up rows once; the four partial 32 x 128 tiles
// are summed through distributed shared memory, each CTA reducing and storing
// a quarter of the rows. Inside a CTA, 3-stage cp.async staging of 64-channel slabs;
// the normalised pv slab is split once into bf16 hi + lo halves (two MMAs per
// k-step keep ~16 mantissa bits, well past the reference's bf16 cast; f16
// v_up takes f16 halves and the f16 MMA), then 8
// warps (16 output columns each, all the CTA's sequences) run mma.sync m16n8k16 with
// ldmatrix fragments.
#include <cooperative_groups.h>

#include <type_traits>

#include "starkv_common.cuh"
#include "starkv_kernels.h"

namespace starkv {

namespace cg = cooperative_groups;

namespace {

constexpr int kSeq = 32;          // sequences per CTA (a multiple of 16: kSeq / 16 MMA row tiles)
constexpr int kMt = kSeq / 16;
constexpr int kSplit = 4;         // CTAs per cluster (channel split)
constexpr int kSlab = 64;         // channels per stage
constexpr int kStages = 3;
constexpr int kThreads = 256;     // 8 warps
constexpr int kPvLd = kSlab + 4;  // f32 row pitch of a staged pv slab (conflict-free float4 rows)
constexpr int kALd = kSlab + 8;   // bf16 row pitch of the hi / lo slabs (ldmatrix: 144 B rows)
constexpr int kVLd = 128 + 8;     // bf16 row pitch of a staged v_up slab (272 B rows)
constexpr int kPvBytes = kSeq * kPvLd * 4;
constexpr int kVBytes = kSlab * kVLd * 2;
constexpr int kStageBytes = kPvBytes + kVBytes;
constexpr int kABytes = kSeq * kALd * 2;                 // one of hi / lo
constexpr int kRedLd = 128 + 4;
constexpr int kSmem = kStages * kStageBytes + 2 * kABytes + kSeq * 4;

static_assert(kSeq * kRedLd * 4 <= kStages * kStageBytes, "reduction tile reuses the staging ring");
static_assert((kSeq / kSplit) * 128 % (4 * kThreads) == 0, "whole float4 runs per reducing thread");

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// D += A . B on m16n8k16, A and B of the 2-byte type T (bf16 or f16), f32 accumulate
template <class T>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __half>::value)
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void to_t(float x, __nv_bfloat16& v) { v = __float2bfloat16_rn(x); }
__device__ __forceinline__ void to_t(float x, __half& v) { v = __float2half_rn(x); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

}  // namespace

// grid (kSplit, H, ceil(n / kSeq)), cluster (kSplit, 1, 1); v_up rows are 2-byte TV
template <class TV>
__global__ void __launch_bounds__(kThreads, 1) lift_cluster_kernel(const LiftParams p) {
  extern __shared__ __align__(16) uint8_t sm[];
  cg::cluster_group cluster = cg::this_cluster();
  const int ks = (int)cluster.block_rank();
  const int h = blockIdx.y;
  const int b0 = blockIdx.z * kSeq;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint8_t* ring = sm;
  TV* a_hi = reinterpret_cast<TV*>(sm + kStages * kStageBytes);
  TV* a_lo = a_hi + kSeq * kALd;
  float* inv_l = reinterpret_cast<float*>(sm + kStages * kStageBytes + 2 * kABytes);

  // this CTA's slabs of the (zero-padded) pv row: [s_beg, s_end) of pv_stride / 64
  const int n_slabs = p.pv_stride / kSlab;
  const int s_beg = n_slabs * ks / kSplit, s_end = n_slabs * (ks + 1) / kSplit;
  const TV* vu = reinterpret_cast<const TV*>(p.v_up) + (int64_t)h * p.vu_s0;

  if (tid < kSeq) {
    const int b = b0 + tid;
    float s = 1.f;   // partial (context-parallel) output: unnormalised
    if (p.l_seq) {
      const float l = b < p.n ? p.l_seq[(int64_t)b * p.num_heads + h] : 0.f;
      s = l > 0.f ? 1.f / l : 0.f;   // empty sequence -> 0, as the reference
    }
    inv_l[tid] = s;
  }

  // stage i of this CTA: pv [kSeq seq][64 ch] f32 and v_up [64 ch][128 d]
  auto load_stage = [&](int slab, int buf) {
    uint8_t* st = ring + buf * kStageBytes;
    float* pvs = reinterpret_cast<float*>(st);
    TV* vs = reinterpret_cast<TV*>(st + kPvBytes);
    const int c0 = slab * kSlab;
#pragma unroll
    for (int i = 0; i < (kSeq * kSlab / 4) / kThreads; ++i) {   // kSeq x 16 float4 chunks
      const int e = tid + kThreads * i;
      const int r = e >> 4, q = (e & 15) * 4;
      const int b = min(b0 + r, p.n - 1);
      cp_async16(pvs + r * kPvLd + q, p.pv + ((int64_t)b * p.num_heads + h) * p.pv_stride + c0 + q);
    }
#pragma unroll
    for (int i = 0; i < (kSlab * 128 / 8) / kThreads; ++i) {    // 1024 16-byte chunks
      const int e = tid + kThreads * i;
      const int r = e >> 4, q = (e & 15) * 8;
      const int c = min(c0 + r, p.v_rank - 1);                   // rows past rank meet pv = 0
      cp_async16(vs + r * kVLd + q, vu + (int64_t)c * p.vu_s1 + q);
    }
  };

  float acc[kMt][2][4] = {};
  const int ns = s_end - s_beg;
#pragma unroll
  for (int i = 0; i < kStages - 1; ++i) {
    if (i < ns) load_stage(s_beg + i, i);
    cp_async_commit();
  }
  for (int i = 0; i < ns; ++i) {
    cp_async_wait<kStages - 2>();   // stage i landed (this thread's copies)
    __syncthreads();                // ...every thread's; iteration i - 1 no longer reads its ring slot
    if (i + kStages - 1 < ns) load_stage(s_beg + i + kStages - 1, (i + kStages - 1) % kStages);
    cp_async_commit();              // (an empty group keeps the count uniform)
    const uint8_t* st = ring + (i % kStages) * kStageBytes;
    const float* pvs = reinterpret_cast<const float*>(st);
    const TV* vs = reinterpret_cast<const TV*>(st + kPvBytes);
    // normalise and split the slab once into v_up's 2-byte type: hi = T(x), lo = T(x - hi)
#pragma unroll
    for (int k = 0; k < (kSeq * kSlab / 4) / kThreads; ++k) {
      const int e = tid + kThreads * k;
      const int r = e >> 4, q = (e & 15) * 4;
      const float4 x4 = *reinterpret_cast<const float4*>(pvs + r * kPvLd + q);
      const float sc = inv_l[r];
      const float x[4] = {x4.x * sc, x4.y * sc, x4.z * sc, x4.w * sc};
      __align__(8) TV hi[4], lo[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        to_t(x[j], hi[j]);
        to_t(x[j] - to_f32(hi[j]), lo[j]);
      }
      *reinterpret_cast<uint2*>(a_hi + r * kALd + q) = *reinterpret_cast<const uint2*>(hi);
      *reinterpret_cast<uint2*>(a_lo + r * kALd + q) = *reinterpret_cast<const uint2*>(lo);
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kSlab / 16; ++kk) {
      // B: v_up[16 ch][16 d] of this warp's columns, transposed by ldmatrix (4 8x8 tiles)
      uint32_t bf[4];
      {
        const int rr = kk * 16 + (lane & 15), cc = warp * 16 + (lane >> 4) * 8;
        ldsm_x4_trans(bf, vs + rr * kVLd + cc);
      }
#pragma unroll
      for (int m = 0; m < kMt; ++m) {
        uint32_t ah[4], al[4];
        const int rr = m * 16 + (lane & 15), cc = kk * 16 + (lane >> 4) * 8;
        ldsm_x4(ah, a_hi + rr * kALd + cc);
        ldsm_x4(al, a_lo + rr * kALd + cc);
        mma16816<TV>(acc[m][0], ah, bf[0], bf[1]);
        mma16816<TV>(acc[m][0], al, bf[0], bf[1]);
        mma16816<TV>(acc[m][1], ah, bf[2], bf[3]);
        mma16816<TV>(acc[m][1], al, bf[2], bf[3]);
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();   // every warp is done with the ring: reuse it for the partial tile

  // partial kSeq x 128 tile of this CTA -> its shared memory, then the cluster sums
  float* red = reinterpret_cast<float*>(ring);
  {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int m = 0; m < kMt; ++m)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int col = warp * 16 + nt * 8 + 2 * t;
        *reinterpret_cast<float2*>(red + (m * 16 + g) * kRedLd + col) = make_float2(acc[m][nt][0], acc[m][nt][1]);
        *reinterpret_cast<float2*>(red + (m * 16 + g + 8) * kRedLd + col) =
            make_float2(acc[m][nt][2], acc[m][nt][3]);
      }
  }
  cluster.sync();   // all four partial tiles written (release / acquire across the cluster)
  {
    // CTA ks reduces and stores rows [kRows ks, kRows ks + kRows): thread -> (row, kCols columns)
    constexpr int kRows = kSeq / kSplit, kCols = kRows * 128 / kThreads;
    constexpr int kThreadsPerRow = 128 / kCols;
    const int r = ks * kRows + tid / kThreadsPerRow, c0 = (tid % kThreadsPerRow) * kCols;
    float s[kCols] = {};
#pragma unroll
    for (int q = 0; q < kSplit; ++q) {
      const float* rem = cluster.map_shared_rank(red, q) + r * kRedLd + c0;
#pragma unroll
      for (int v4 = 0; v4 < kCols / 4; ++v4) {
        const float4 u = *reinterpret_cast<const float4*>(rem + 4 * v4);
        s[4 * v4] += u.x; s[4 * v4 + 1] += u.y; s[4 * v4 + 2] += u.z; s[4 * v4 + 3] += u.w;
      }
    }
    const int b = b0 + r;
    if (b < p.n) {
      const int64_t o = (int64_t)b * p.o_s0 + (int64_t)h * p.o_s1;
#pragma unroll
      for (int j = 0; j < kCols; ++j) store_elem(p.out, o + (int64_t)(c0 + j) * p.o_s2, p.out_dtype, s[j]);
    }
  }
  cluster.sync();   // no CTA leaves while another still reads its tile
}

// The cluster lift when the layout allows it (2-byte v_up with unit stride along a
// 128-wide head_dim, 16-byte aligned rows); returns -1 when it does not.
int launch_lift_cluster(const LiftParams& p, cudaStream_t stream) {
  const int es = p.v_up_dtype == STARKV_F32 ? 4 : 2;
  const bool ok = es == 2 && p.head_dim == 128 && p.vu_s2 == 1 && p.vu_s0 % 8 == 0 && p.vu_s1 % 8 == 0 &&
                  (reinterpret_cast<uintptr_t>(p.v_up) & 15) == 0 && p.pv_stride % kSlab == 0 &&
                  (reinterpret_cast<uintptr_t>(p.pv) & 15) == 0 && p.n > 0;
  if (!ok) return -1;
  const void* fn = p.v_up_dtype == STARKV_BF16 ? (const void*)lift_cluster_kernel<__nv_bfloat16>
                                               : (const void*)lift_cluster_kernel<__half>;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess)
    return STARKV_ECUDA;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kSplit;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(kSplit, p.num_heads, (p.n + kSeq - 1) / kSeq);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {const_cast<LiftParams*>(&p)};
  if (cudaLaunchKernelExC(&cfg, fn, args) != cudaSuccess) return STARKV_ECUDA;
  return STARKV_OK;
}

}  // namespace starkv
