// The step's K/V down-projection fused with the bf16 / f16 cache write:
//   cache[slot_t] = hidden_t . kv_down^T     (model.py:70 codes = F.linear(hidden,
//                                              kv_down); attention.py:179-185 writes
//                                              cat(k_codes, v_codes) at the slot)
// so the codes never leave the chip between the GEMM and the cache.
//
// Swap-AB tcgen05 GEMM: D[c, t] = kv_down[c, :] . hidden[t, :], M = 128 code
// channels per tile, N = the step's tokens (rounded to 16, at most 256 per launch
// column), K = hidden. A decode step has few tokens, so the weight read (W x hidden
// x 2 B) is the cost; it is spread over the whole GPU by splitting K eight ways
// across a cluster of 8 CTAs per channel tile. Each CTA accumulates its K share in
// TMEM, writes the f32 partial to its own shared memory, and after a cluster barrier
// CTA r adds channels [16 r, 16 r + 16) of all eight partials through distributed
// shared memory, rounds them and stores them into the token rows of the cache.
// A slot of -1 (CUDA-graph padding) is written to slot 0, the reserved null block,
// as attention.py:181 does with clamp(min=0).
//
// Warps: 0 TMA producer, 1 TMEM owner and MMA issuer; all four read back their TMEM
// lane quarter. Pipeline waits are bounded; both cluster barriers are reached on
// every path.
#include <cooperative_groups.h>

#include "starkv_common.cuh"
#include "starkv_kernels.h"

namespace starkv {

namespace {

namespace cg = cooperative_groups;

constexpr int kSplit = 8;          // CTAs per cluster: the K split
constexpr int kChan = 128;         // channels per tile (MMA M)
constexpr int kKBlk = 64;          // hidden elements per stage (one 128-byte swizzle atom)
constexpr int kThreads = 128;
constexpr int kMaxStages = 4;
constexpr int kWBytes = kChan * kKBlk * 2;   // 16 KB

struct DownCtl {
  uint64_t full[kMaxStages], empty[kMaxStages];
  uint64_t done;
  uint32_t tmem_base;
  int abort_flag;
};

__host__ __device__ inline int tok_bytes(int n_tile) { return n_tile * kKBlk * 2; }
__host__ __device__ inline int stage_bytes(int n_tile) { return (kWBytes + tok_bytes(n_tile) + 1023) & ~1023; }
__host__ __device__ inline int red_pitch(int n_tile) { return n_tile + 4; }   // f32 row pitch of the partial

__device__ __forceinline__ uint16_t bits16(__nv_bfloat16 v) { return __bfloat16_as_ushort(v); }
__device__ __forceinline__ uint16_t bits16(__half v) { return __half_as_ushort(v); }

// K-major, 128-byte-swizzled operand of one 64-element K block: descriptor for K step kk
__device__ __forceinline__ uint64_t atom_desc(uint32_t base, int kk) {
  return smem_desc(base + kk * 32, 16, 1024, kSwizzle128B);
}

}  // namespace

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    kv_down_write_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                         const DownWriteParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int SB = stage_bytes(p.n_tile);
  DownCtl* ctl = reinterpret_cast<DownCtl*>(smem + p.ctl_offset);
  volatile int* abort_flag = &ctl->abort_flag;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();        // K share of this CTA
  const int ch0 = blockIdx.y * kChan, t0 = blockIdx.z * p.n_tile;
  const int nk = p.hidden / (kKBlk * kSplit);          // 64-wide K blocks of this CTA
  const int kb0 = rank * nk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t tcols = 32;
  while (tcols < (uint32_t)p.n_tile) tcols <<= 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    mbar_init(&ctl->done, 1);
    ctl->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&ctl->tmem_base, tcols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  if (warp == 0 && lane == 0) {
    // ================= TMA producer: weight rows and token rows of each K block =================
    tma_prefetch(&tm_w);
    tma_prefetch(&tm_x);
    int last[kMaxStages];
    for (int s = 0; s < kMaxStages; ++s) last[s] = -1;
    for (int i = 0; i < nk; ++i) {
      const int s = i % p.stages;
      if (!mbar_wait(&ctl->empty[s], ((i / p.stages) & 1) ^ 1, abort_flag, p.status)) break;
      last[s] = i;
      uint8_t* st = smem + s * SB;
      mbar_arrive_expect_tx(&ctl->full[s], kWBytes + tok_bytes(p.n_tile));
      tma_load_2d(st, &tm_w, &ctl->full[s], (kb0 + i) * kKBlk, ch0);
      tma_load_2d(st + kWBytes, &tm_x, &ctl->full[s], (kb0 + i) * kKBlk, t0);
    }
    // every copy has landed before shared memory is reused below
    for (int s = 0; s < p.stages; ++s)
      if (last[s] >= 0) {
        for (uint32_t it = 0; it < kWaitLimit; ++it)
          if (mbar_try_wait(&ctl->full[s], (last[s] / p.stages) & 1)) break;
      }
  } else if (warp == 1 && lane == 0) {
    // ================= MMA issuer =================
    const uint32_t idesc = instr_desc_f16(p.dtype == STARKV_BF16 ? 1u : 0u, 0, 0, kChan, p.n_tile);
    for (int i = 0; i < nk; ++i) {
      const int s = i % p.stages;
      if (!mbar_wait(&ctl->full[s], (i / p.stages) & 1, abort_flag, p.status)) break;
      tc_fence_after();
      const uint32_t w_addr = smem_u32(smem + s * SB), x_addr = w_addr + kWBytes;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) umma_f16(tmem, atom_desc(w_addr, kk), atom_desc(x_addr, kk), idesc, i > 0 || kk > 0);
      umma_commit(&ctl->empty[s]);
    }
    umma_commit(&ctl->done);   // every MMA issued here (also after an abort)
  }
  __syncwarp();
  // ---- read back this CTA's partial [128 channels][n_tile tokens] f32 into shared memory ----
  bool ok = mbar_wait(&ctl->done, 0, abort_flag, p.status) && !*abort_flag;
  __syncthreads();   // the producer's copies have landed: the stage area is free
  tc_fence_after();
  float* red = reinterpret_cast<float*>(smem);
  const int pitch = red_pitch(p.n_tile);
  {
    const int row = warp * 32 + lane;   // channel of the tile (warp w reads TMEM lanes 32 w ..)
    for (int c0 = 0; c0 < p.n_tile; c0 += 32) {
      float v[32];
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + c0, v);
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (c0 + i < p.n_tile) red[row * pitch + c0 + i] = ok ? v[i] : 0.f;   // n_tile need not be a multiple of 32
    }
  }
  tc_fence_before();
  cluster.sync();   // all eight partials are in place
  // ---- CTA r: channels [16 r, 16 r + 16) of the tile, summed over the eight partials ----
  const int n_items = p.n_tile * 2;
  for (int item = threadIdx.x; item < n_items; item += kThreads) {
    const int t = item >> 1, ch = rank * 16 + (item & 1) * 8;
    if (t0 + t >= p.n) continue;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int src = 0; src < kSplit; ++src) {
      const float* rem = cluster.map_shared_rank(red, src);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += rem[(ch + e) * pitch + t];
    }
    int64_t slot = load_slot(p.slot_mapping, t0 + t, p.slot_dtype);
    if (slot < 0) slot = 0;   // padding row: the reserved null block (attention.py:181)
    const int64_t blk = slot / p.block_size, off = slot % p.block_size;
    if (blk >= p.num_blocks) {
      record_status(p.status, STARKV_EBOUNDS);
      continue;
    }
    const int gc = ch0 + ch;
    T* dst = reinterpret_cast<T*>(p.cache) + blk * p.c_s0 + off * p.c_s1 + gc;
    if (gc + 8 <= p.out_width) {
      uint4 u;
      uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) w[e] = (uint32_t)bits16(T(acc[2 * e])) | ((uint32_t)bits16(T(acc[2 * e + 1])) << 16);
      *reinterpret_cast<uint4*>(dst) = u;
    } else {
      for (int e = 0; e < 8 && gc + e < p.out_width; ++e) store_elem(dst, e, p.dtype, acc[e]);
    }
  }
  cluster.sync();   // no CTA leaves while a peer may still read its partial
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, tcols);
  }
}

size_t kv_down_smem_bytes(int n_tile, int stages) {
  const size_t st = (size_t)stages * stage_bytes(n_tile);
  const size_t red = (size_t)kChan * red_pitch(n_tile) * 4;
  return ((st > red ? st : red) + 15) / 16 * 16 + sizeof(DownCtl) + 1024;
}

int kv_down_ctl_offset(int n_tile, int stages) {
  const size_t st = (size_t)stages * stage_bytes(n_tile);
  const size_t red = (size_t)kChan * red_pitch(n_tile) * 4;
  return (int)(((st > red ? st : red) + 15) / 16 * 16);
}

int launch_kv_down_write(const CUtensorMap& tm_w, const CUtensorMap& tm_x, const DownWriteParams& p, cudaStream_t stream) {
  const int m_tiles = (p.out_width + kChan - 1) / kChan;
  const int cols = (p.n + p.n_tile - 1) / p.n_tile;
  const size_t smem = kv_down_smem_bytes(p.n_tile, p.stages);
  if (smem > 227 * 1024 || p.stages < 1 || p.stages > kMaxStages) return STARKV_EINVAL;
  const void* fn = p.dtype == STARKV_BF16 ? (const void*)kv_down_write_kernel<__nv_bfloat16>
                                          : (const void*)kv_down_write_kernel<__half>;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return STARKV_ECUDA;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kSplit;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(kSplit, m_tiles, cols);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {const_cast<CUtensorMap*>(&tm_w), const_cast<CUtensorMap*>(&tm_x), const_cast<DownWriteParams*>(&p)};
  if (cudaLaunchKernelExC(&cfg, fn, args) != cudaSuccess) return STARKV_ECUDA;
  return STARKV_OK;
}

int kv_down_split() { return kSplit; }

}  // namespace starkv
