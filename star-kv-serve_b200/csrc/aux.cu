// Small kernels around the two tensor-core passes:
//   fold_kernel   AB = fold(q, U) * scale (paged_quant.py:223-255), the f16 copy of
//                 the rotary table rows, and per-call accumulator init;
//   lift_kernel   out[b,h,:] = pv[b,h,:] / l[b,h] . v_up_by_q[h] (paged_decode.py:222-226);
//   pack_k/v      3.2-bit write side (paged_quant.py:139-216), bit-exact with
//                 kv_quant._q (kv_quant.py:111-121): IEEE division, round half even;
//   cache_write   bf16 cache write (attention.py:179-185).
#include "starkv_common.cuh"
#include "starkv_kernels.h"

namespace starkv {

// ---------------------------------------------------------------------------
// fold + rotary table + init (one launch)
// ---------------------------------------------------------------------------

constexpr int kFoldLanes = 4;   // K lanes per 256-thread block (64 threads each)

__global__ void __launch_bounds__(256) fold_kernel(const FoldParams p, int n_fold_blocks, int n_cs_blocks) {
  const int bid = blockIdx.x;
  if (bid < n_fold_blocks) {
    // block -> (b, j, 4 lanes); thread -> (lane, i in 0..63)
    const int lanes_per_seq = (p.k_width + kFoldLanes - 1) / kFoldLanes;
    const int bj = bid / lanes_per_seq;
    const int r = (bid % lanes_per_seq) * kFoldLanes + (threadIdx.x >> 6);
    const int i = threadIdx.x & 63;
    const int b = bj / p.group, j = bj % p.group;
    if (r >= p.k_width) return;
    int head = -1;
    bool live = true;
    if (p.head_of_lane) {
      head = p.head_of_lane[r];
    } else {
      for (int h = 0; h < p.num_kv_heads; ++h) {
        const int off = p.k_head_offsets[h], rk = p.k_ranks[h];
        const int w = (rk + 15) & ~15;
        if (r >= off && r < off + w) {
          head = h;
          live = (r - off) < rk;
          break;
        }
      }
    }
    __half* dst = p.ab + ((int64_t)bj * p.k_width + r) * 128;
    if (head < 0 || head >= p.num_kv_heads || !live) {
      if (head >= p.num_kv_heads) record_status(p.status, STARKV_EBOUNDS);
      dst[i] = __float2half_rn(0.f);
      dst[i + 64] = __float2half_rn(0.f);
      return;
    }
    const int hq = head * p.group + j;
    const int64_t qo = (int64_t)b * p.q_s0 + (int64_t)hq * p.q_s1;
    const float q0 = load_elem(p.q, qo + (int64_t)i * p.q_s2, p.q_dtype);
    const float q1 = load_elem(p.q, qo + (int64_t)(i + 64) * p.q_s2, p.q_dtype);
    const float u0 = load_elem(p.k_up, (int64_t)r * p.ku_s0 + (int64_t)i * p.ku_s1, p.k_up_dtype);
    const float u1 = load_elem(p.k_up, (int64_t)r * p.ku_s0 + (int64_t)(i + 64) * p.ku_s1, p.k_up_dtype);
    dst[i] = __float2half_rn((q0 * u0 + q1 * u1) * p.scale);
    dst[i + 64] = __float2half_rn((q1 * u0 - q0 * u1) * p.scale);
    return;
  }
  if (bid < n_fold_blocks + n_cs_blocks) {
    // rotary table rows -> f16, zero past the table / max_seq_len
    const int64_t e = (int64_t)(bid - n_fold_blocks) * 256 + threadIdx.x;
    const int64_t row = e >> 7;
    const int col = (int)(e & 127);
    if (row >= p.l_pad) return;
    float v = 0.f;
    if (row < p.cs_rows && row < p.max_seq_len) v = load_elem(p.cs, row * p.cs_s0 + col * p.cs_s1, p.cs_dtype);
    p.cs16[e] = __float2half_rn(v);
    return;
  }
  // init: sequence max = -inf, pv = 0
  const int64_t t = (int64_t)(bid - n_fold_blocks - n_cs_blocks) * 256 + threadIdx.x;
  const int64_t stride = (int64_t)(gridDim.x - n_fold_blocks - n_cs_blocks) * 256;
  for (int64_t k = t; k < p.m_count; k += stride) p.m_seq[k] = -INFINITY;
  float4* pv4 = reinterpret_cast<float4*>(p.pv);
  const int64_t n4 = p.pv_count >> 2;
  for (int64_t k = t; k < n4; k += stride) pv4[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t k = (n4 << 2) + t; k < p.pv_count; k += stride) p.pv[k] = 0.f;
}

int launch_fold(const FoldParams& p, bool quant, cudaStream_t stream) {
  (void)quant;
  const int lanes_per_seq = (p.k_width + kFoldLanes - 1) / kFoldLanes;
  const int n_fold = p.n * p.group * lanes_per_seq;
  const int n_cs = (int)(((int64_t)p.l_pad * 128 + 255) / 256);
  const int n_init = 148;
  fold_kernel<<<n_fold + n_cs + n_init, 256, 0, stream>>>(p, n_fold, n_cs);
  return cudaGetLastError() == cudaSuccess ? STARKV_OK : STARKV_ECUDA;
}

// ---------------------------------------------------------------------------
// lift: out[b, h, :] = (pv[b, h, :] / l[b, h]) . v_up_by_q[h]
// ---------------------------------------------------------------------------

constexpr int kLiftB = 16;     // sequences per block
constexpr int kLiftV = 32;     // V channels staged per step

__global__ void __launch_bounds__(128) lift_kernel(const LiftParams p) {
  const int h = blockIdx.x;
  const int b0 = blockIdx.y * kLiftB;
  const int d = threadIdx.x;
  __shared__ float inv_l[kLiftB];
  __shared__ float pvs[kLiftB][kLiftV];
  if (threadIdx.x < kLiftB) {
    const int b = b0 + threadIdx.x;
    float l = 0.f;
    if (b < p.n) {
      const int L = min(max(p.seq_lens[b], 0), p.max_seq_len);
      const int nt = (L + 127) >> 7;
      const float M = p.m_seq[(int64_t)b * p.num_heads + h];
      const int64_t base = ((int64_t)b * p.num_heads + h) * p.n_tiles;
      for (int t = 0; t < nt; ++t) l += p.l_tile[base + t] * __expf(p.m_tile[base + t] - M);
    }
    inv_l[threadIdx.x] = l > 0.f ? 1.f / l : 0.f;   // empty sequence -> 0, as the reference
  }
  float acc[kLiftB];
#pragma unroll
  for (int i = 0; i < kLiftB; ++i) acc[i] = 0.f;
  for (int v0 = 0; v0 < p.v_rank; v0 += kLiftV) {
    __syncthreads();
    for (int e = threadIdx.x; e < kLiftB * kLiftV; e += blockDim.x) {
      const int bb = e / kLiftV, vv = e % kLiftV;
      const int b = b0 + bb, v = v0 + vv;
      pvs[bb][vv] = (b < p.n && v < p.v_rank) ? p.pv[((int64_t)b * p.num_heads + h) * p.v_rank + v] : 0.f;
    }
    __syncthreads();
    if (d < p.head_dim) {
      const int vmax = min(kLiftV, p.v_rank - v0);
      for (int vv = 0; vv < vmax; ++vv) {
        const float w = load_elem(p.v_up, (int64_t)h * p.vu_s0 + (int64_t)(v0 + vv) * p.vu_s1 + (int64_t)d * p.vu_s2,
                                  p.v_up_dtype);
#pragma unroll
        for (int i = 0; i < kLiftB; ++i) acc[i] += pvs[i][vv] * w;
      }
    }
  }
  __syncthreads();
  if (d < p.head_dim) {
    for (int i = 0; i < kLiftB; ++i) {
      const int b = b0 + i;
      if (b < p.n)
        store_elem(p.out, (int64_t)b * p.o_s0 + (int64_t)h * p.o_s1 + (int64_t)d * p.o_s2, p.out_dtype,
                   acc[i] * inv_l[i]);
    }
  }
}

int launch_lift(const LiftParams& p, cudaStream_t stream) {
  dim3 grid(p.num_heads, (p.n + kLiftB - 1) / kLiftB);
  lift_kernel<<<grid, 128, 0, stream>>>(p);
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
