// C ABI entry points of the decode path (include/starkv_b200.h): argument
// validation, workspace layout, TMA descriptor encoding, launch order.
//
// One decode call = 4 launches on the caller's stream, no host synchronisation,
// no allocation:
//   fold_kernel -> scores_kernel (tcgen05) -> pv_kernel (tcgen05) -> lift_kernel
#include <cuda.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <mutex>

#include "starkv_common.cuh"
#include "starkv_kernels.h"

namespace starkv {

namespace {

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

struct DeviceInfo {
  int sms = 0;
  bool sm100 = false;
};

int device_info(DeviceInfo& info) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return STARKV_ECUDA;
  static DeviceInfo cache[64];
  static std::once_flag flags[64];
  if (dev < 0 || dev >= 64) return STARKV_ENODEV;
  std::call_once(flags[dev], [dev] {
    int major = 0, minor = 0, sms = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cache[dev].sms = sms;
    cache[dev].sm100 = (major == 10 && minor == 0);
  });
  info = cache[dev];
  return info.sm100 ? STARKV_OK : STARKV_ENODEV;
}

// Tiled TMA descriptor; dims[0] is the contiguous one, strides in bytes for dims 1..rank-1.
int make_map(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base, const uint64_t* dims,
             const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return STARKV_ECUDA;
  if (reinterpret_cast<uintptr_t>(base) & 15) return STARKV_EALIGN;
  for (int i = 0; i < rank - 1; ++i)
    if (strides_bytes[i] & 15) return STARKV_EALIGN;
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, dt, rank, const_cast<void*>(base), reinterpret_cast<const cuuint64_t*>(dims),
                  reinterpret_cast<const cuuint64_t*>(strides_bytes), reinterpret_cast<const cuuint32_t*>(box), estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? STARKV_OK : STARKV_EALIGN;
}

// Optional per-kernel timing (bench only): a pool of CUDA events recorded on the
// launch stream around each of the 4 decode kernels.
struct Profile {
  bool on = false;
  int max_calls = 0, calls = 0;
  cudaEvent_t* ev = nullptr;   // [max_calls][5]
};
Profile g_prof;

bool is_float_dtype(int d) { return d == STARKV_BF16 || d == STARKV_F16 || d == STARKV_F32; }

}  // namespace

Workspace workspace_layout(int n, int num_heads, int num_kv_heads, int k_width, int v_rank, int max_seq_len) {
  Workspace w{};
  const int group = num_kv_heads > 0 ? num_heads / num_kv_heads : 1;
  w.n_tiles = (max_seq_len + 127) / 128;
  if (w.n_tiles < 1) w.n_tiles = 1;
  w.l_pad = w.n_tiles * 128;
  size_t off = 0;
  w.status = off; off += 256;
  w.ab = off; off = align256(off + (size_t)n * group * ((k_width + 127) / 128) * 128 * 128 * 2);   // MMA image
  w.cs = off; off = align256(off + (size_t)w.l_pad * 128 * 2);
  w.e16 = off; off = align256(off + (size_t)n * num_heads * w.l_pad * 2);
  w.m_tile = off; off = align256(off + (size_t)n * num_heads * w.n_tiles * 4);
  w.l_seq = off; off = align256(off + (size_t)n * num_heads * 4);
  w.m_seq = off; off = align256(off + (size_t)n * num_heads * 4);
  w.pv_stride = (v_rank + 63) / 64 * 64;
  w.pv = off; off = align256(off + (size_t)n * num_heads * w.pv_stride * 4);
  w.total = off;
  return w;
}

// cp_world > 1 (or m_out set): context-parallel partial decode of this rank's share of
// every sequence; out is then f32 and unnormalised (sum_t p_t V_t . v_up with p
// relative to the rank's own per-head max), and the max / softmax denominator go to
// m_out / l_out [n, num_heads] f32.
static int decode_impl(const StarKVDecodeArgs* a, void* workspace, size_t ws_bytes, cudaStream_t stream, bool quant,
                       int cp_rank = 0, int cp_world = 1, float* m_out = nullptr, float* l_out = nullptr) {
  if (!a) return STARKV_EINVAL;
  if (cp_world < 1 || cp_rank < 0 || cp_rank >= cp_world) return STARKV_EINVAL;
  const bool partial = m_out != nullptr || l_out != nullptr;
  if (partial && (!m_out || !l_out || a->out_dtype != STARKV_F32)) return STARKV_EINVAL;
  if (cp_world > 1 && !partial) return STARKV_EINVAL;   // a share of a sequence is only a partial result
  DeviceInfo dev;
  int st = device_info(dev);
  if (st) return st;
  // ---- shape / type validation (reference asserts: paged_decode.py:172-174, paged_quant.py:374-376) ----
  if (a->n < 0 || a->num_heads <= 0 || a->num_kv_heads <= 0 || a->num_heads % a->num_kv_heads) return STARKV_EINVAL;
  if (a->n == 0) return STARKV_OK;
  if (a->head_dim != 128) return STARKV_EINVAL;
  if (a->k_width <= 0 || a->k_width % 16 || a->v_rank <= 0) return STARKV_EINVAL;
  if (a->max_seq_len <= 0 || a->cs_rows < a->max_seq_len) return STARKV_EINVAL;
  if (a->block_size <= 0 || a->block_size % 16 || a->num_blocks <= 0) return STARKV_EINVAL;
  if (a->num_heads > 128 || a->max_blocks <= 0) return STARKV_EINVAL;
  if (!a->query || !a->kv_cache || !a->block_table || !a->seq_lens || !a->k_up || !a->v_up_by_q ||
      !a->cos_sin_cache || !a->out)
    return STARKV_EINVAL;
  if (!is_float_dtype(a->q_dtype) || !is_float_dtype(a->k_up_dtype) || !is_float_dtype(a->v_up_dtype) ||
      !is_float_dtype(a->cs_dtype) || !is_float_dtype(a->out_dtype))
    return STARKV_EDTYPE;
  if (a->cache_stride[2] != 1) return STARKV_EALIGN;
  const int group = a->num_heads / a->num_kv_heads;
  if (quant) {
    if (a->cache_dtype != STARKV_U8) return STARKV_EDTYPE;
    if (group != 1) return STARKV_EINVAL;   // 4-bit decode: MHA (paged_quant.py:374)
    if (!a->head_of_lane || !a->tile_head || !a->tile_nout || !a->tile_last) return STARKV_EINVAL;
    if (a->ks_off != a->k_width / 2 || a->vs_off != a->ks_off + 4 * a->num_kv_heads || a->vq_off != a->vs_off + 4)
      return STARKV_EINVAL;
    if (a->v_nout < 0 || a->v_nout > a->v_rank || a->v_nbo != (a->v_nout + 1) / 2 ||
        a->v_bytes != a->v_nbo + (a->v_rank - a->v_nout + 1) / 2 || a->row_nbytes < a->vq_off + a->v_bytes)
      return STARKV_EINVAL;
  } else {
    if (a->cache_dtype != STARKV_BF16 && a->cache_dtype != STARKV_F16) return STARKV_EDTYPE;
    if (!a->k_ranks || !a->k_head_offsets) return STARKV_EINVAL;
  }

  const Workspace ws = workspace_layout(a->n, a->num_heads, a->num_kv_heads, a->k_width, a->v_rank, a->max_seq_len);
  if (!workspace || ws_bytes < ws.total) return STARKV_EWORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return STARKV_EALIGN;
  uint8_t* W = reinterpret_cast<uint8_t*>(workspace);
  int32_t* status = reinterpret_cast<int32_t*>(W + ws.status);
  __half* ab = reinterpret_cast<__half*>(W + ws.ab);
  __half* cs16 = reinterpret_cast<__half*>(W + ws.cs);
  __half* e16 = reinterpret_cast<__half*>(W + ws.e16);
  float* m_tile = reinterpret_cast<float*>(W + ws.m_tile);
  float* l_seq = reinterpret_cast<float*>(W + ws.l_seq);
  float* m_seq = reinterpret_cast<float*>(W + ws.m_seq);
  float* pv = reinterpret_cast<float*>(W + ws.pv);

  // ---- TMA descriptors ----
  CUtensorMap tm_cs, tm_ab, tm_code, tm_tail, tm_sc, tm_v;
  // Rotary rows and AB are written by the fold kernel as ready-made 128-byte-swizzled
  // MMA tiles; they are copied as 2 KB rows (8-byte elements, no swizzle): one box
  // per 32 KB rotary tile, one per 16 KB half-chunk of AB.
  const int ncp = (a->k_width + 127) / 128;
  {
    const uint64_t dims[2] = {256, (uint64_t)ws.n_tiles * 16};
    const uint64_t str[1] = {2048};
    const uint32_t box[2] = {256, 16};
    if ((st = make_map(&tm_cs, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, cs16, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE)))
      return st;
  }
  {
    const uint64_t dims[2] = {256, (uint64_t)a->n * group * ncp * 2 * 8};
    const uint64_t str[1] = {2048};
    const uint32_t box[2] = {256, 8};
    if ((st = make_map(&tm_ab, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, ab, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE)))
      return st;
  }
  const int es = quant ? 1 : 2;
  const uint64_t row_elems = quant ? (uint64_t)a->row_nbytes : (uint64_t)(a->k_width + a->v_rank);
  if (a->cache_stride[1] < (int64_t)row_elems || a->cache_stride[0] < a->cache_stride[1] * a->block_size)
    return STARKV_EINVAL;
  // P.V (bf16 / f16): V code tiles straight from the cache, 64 channels = 128 B per
  // box row, 128-byte swizzle (the MMA's A layout). The 3.2-bit map is made below.
  if (!quant) {
    const uint64_t dims[3] = {row_elems, (uint64_t)a->block_size, (uint64_t)a->num_blocks};
    const uint64_t str[2] = {(uint64_t)a->cache_stride[1] * es, (uint64_t)a->cache_stride[0] * es};
    const uint32_t box[3] = {64, 16, 1};
    if ((st = make_map(&tm_v, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, a->kv_cache, dims, str, box,
                       CU_TENSOR_MAP_SWIZZLE_128B)))
      return st;
  }
  // Scores: code windows cut from an 8-byte-element view of the cache, unswizzled,
  // with the row pitch the kernel stages them at (an odd multiple of 16 bytes).
  int code_pitch = 0, tail_pitch = 0, n_wins = 0, sc_pitch = 0, sc_x0 = 0;
  {
    const uint64_t row_bytes = row_elems * es;
    if (row_bytes % 8) return STARKV_EALIGN;
    const int win_bytes = scores_window_bytes(quant);
    const int win_lanes = quant ? 2 * win_bytes : win_bytes / 2;
    n_wins = (a->k_width + win_lanes - 1) / win_lanes;
    const int tail_lanes = (a->k_width - (n_wins - 1) * win_lanes + 31) & ~31;   // whole 32-lane groups
    code_pitch = code_pitch_bytes(win_bytes);
    tail_pitch = code_pitch_bytes(quant ? tail_lanes / 2 : tail_lanes * 2);
    const uint64_t dims[3] = {row_bytes / 8, (uint64_t)a->block_size, (uint64_t)a->num_blocks};
    const uint64_t str[2] = {(uint64_t)a->cache_stride[1] * es, (uint64_t)a->cache_stride[0] * es};
    const uint32_t box[3] = {(uint32_t)code_pitch / 8, 16, 1};
    const uint32_t box_t[3] = {(uint32_t)tail_pitch / 8, 16, 1};
    if ((st = make_map(&tm_code, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, a->kv_cache, dims, str, box,
                       CU_TENSOR_MAP_SWIZZLE_NONE)))
      return st;
    if ((st = make_map(&tm_tail, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, a->kv_cache, dims, str, box_t,
                       CU_TENSOR_MAP_SWIZZLE_NONE)))
      return st;
    tm_sc = tm_code;
    if (quant) {
      sc_x0 = a->ks_off & ~15;
      sc_pitch = code_pitch_bytes(a->ks_off + 4 * a->num_kv_heads - sc_x0);
      if (sc_pitch / 8 > 256) return STARKV_EINVAL;
      const uint32_t box_s[3] = {(uint32_t)sc_pitch / 8, 16, 1};
      if ((st = make_map(&tm_sc, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, a->kv_cache, dims, str, box_s,
                         CU_TENSOR_MAP_SWIZZLE_NONE)))
        return st;
    }
  }

  // ---- fold + table + init ----
  FoldParams fp{};
  fp.q = a->query; fp.q_s0 = a->q_stride[0]; fp.q_s1 = a->q_stride[1]; fp.q_s2 = a->q_stride[2];
  fp.q_dtype = a->q_dtype;
  fp.k_up = a->k_up; fp.ku_s0 = a->k_up_stride[0]; fp.ku_s1 = a->k_up_stride[1]; fp.k_up_dtype = a->k_up_dtype;
  fp.head_of_lane = quant ? a->head_of_lane : nullptr;
  fp.k_ranks = a->k_ranks; fp.k_head_offsets = a->k_head_offsets;
  fp.n = a->n; fp.num_heads = a->num_heads; fp.num_kv_heads = a->num_kv_heads; fp.group = group;
  fp.k_width = a->k_width; fp.head_dim = a->head_dim; fp.scale = a->scale; fp.ab = ab; fp.ab_image = 1;
  fp.cs = a->cos_sin_cache; fp.cs_s0 = a->cs_stride[0]; fp.cs_s1 = a->cs_stride[1]; fp.cs_dtype = a->cs_dtype;
  fp.cs_rows = a->cs_rows; fp.cs16 = cs16; fp.l_pad = ws.l_pad; fp.max_seq_len = a->max_seq_len;
  fp.m_seq = m_seq; fp.l_seq = l_seq; fp.m_count = a->n * a->num_heads;
  fp.pv = pv; fp.pv_count = (int64_t)a->n * a->num_heads * ws.pv_stride;
  fp.status = status;
  cudaEvent_t* pev = nullptr;
  if (g_prof.on && g_prof.calls < g_prof.max_calls) pev = g_prof.ev + 5 * g_prof.calls++;
  if (pev) cudaEventRecord(pev[0], stream);
  if ((st = launch_fold(fp, quant, stream))) return st;
  if (pev) cudaEventRecord(pev[1], stream);

  // ---- scores ----
  ScoresParams sp{};
  sp.seq_lens = a->seq_lens; sp.block_table = a->block_table; sp.bt_s0 = a->bt_stride[0]; sp.bt_s1 = a->bt_stride[1];
  sp.max_blocks = a->max_blocks;
  sp.n = a->n; sp.num_heads = a->num_heads; sp.num_kv_heads = a->num_kv_heads; sp.group = group;
  sp.k_width = a->k_width; sp.num_blocks = a->num_blocks; sp.block_size = a->block_size;
  sp.max_seq_len = a->max_seq_len; sp.cache_dtype = a->cache_dtype;
  sp.k_ranks = a->k_ranks; sp.k_head_offsets = a->k_head_offsets;
  sp.tile_head = a->tile_head; sp.tile_nout = a->tile_nout; sp.tile_last = a->tile_last;
  if (quant) sp.ks_off = a->ks_off;
  sp.code_pitch = code_pitch; sp.tail_pitch = tail_pitch; sp.n_wins = n_wins;
  sp.sc_pitch = sc_pitch; sp.sc_x0 = sc_x0;
  sp.e16 = e16; sp.m_tile = m_tile; sp.m_seq = m_seq;
  sp.l_pad = ws.l_pad; sp.n_tiles = ws.n_tiles; sp.status = status;
  sp.cp_rank = cp_rank; sp.cp_world = cp_world;
  if ((st = launch_scores(quant, tm_cs, tm_ab, tm_code, tm_tail, tm_sc, sp, dev.sms, stream))) return st;
  if (pev) cudaEventRecord(pev[2], stream);

  // ---- P.V ----
  PvParams pp{};
  pp.seq_lens = a->seq_lens; pp.block_table = a->block_table; pp.bt_s0 = a->bt_stride[0]; pp.bt_s1 = a->bt_stride[1];
  pp.max_blocks = a->max_blocks;
  pp.n = a->n; pp.num_heads = a->num_heads; pp.k_width = a->k_width; pp.v_rank = a->v_rank;
  pp.num_blocks = a->num_blocks; pp.block_size = a->block_size; pp.max_seq_len = a->max_seq_len;
  pp.nh = ((a->num_heads + 15) / 16) * 16;
  pp.cache_dtype = a->cache_dtype;
  if (quant) {
    pp.v_nout = a->v_nout; pp.v_nbo = a->v_nbo; pp.v_bytes = a->v_bytes; pp.vq_off = a->vq_off;
    pp.vs_off = a->vs_off;
    pp.vx0 = a->vs_off & ~15;
    pp.v_pitch = code_pitch_bytes(a->vq_off + a->v_bytes - pp.vx0);
    if (pp.v_pitch > 2048) return STARKV_EINVAL;   // one box row of at most 256 8-byte elements
    pp.t_out = (a->v_nout + 127) / 128;
    pp.n_mtiles = pp.t_out + (a->v_rank - a->v_nout + 127) / 128;
  } else {
    pp.n_mtiles = (a->v_rank + 127) / 128;
  }
  int mtpr = pp.n_mtiles;
  if (mtpr * pp.nh > 512) mtpr = 512 / pp.nh;
  for (;;) {
    pp.mt_per_range = mtpr;
    if (quant) {
      if (mtpr * 64 <= pvq_max_dequant_tasks() && pvq_page_stages(pp) >= 2 && pvq_smem_bytes(pp) <= 227 * 1024)
        break;
    } else if (pv_page_stages(pp) >= 2 && pv_smem_bytes(pp) <= 227 * 1024) {
      break;
    }
    if (--mtpr < 1) return STARKV_EINVAL;
  }
  pp.n_ranges = (pp.n_mtiles + mtpr - 1) / mtpr;
  pp.mt_per_range = (pp.n_mtiles + pp.n_ranges - 1) / pp.n_ranges;   // balance the ranges
  pp.e16 = e16; pp.m_tile = m_tile; pp.m_seq = m_seq; pp.l_seq = l_seq; pp.pv = pv; pp.pv_stride = ws.pv_stride;
  pp.l_pad = ws.l_pad; pp.n_tiles = ws.n_tiles; pp.status = status;
  pp.cp_rank = cp_rank; pp.cp_world = cp_world;
  CUtensorMap tm_e;
  {
    const uint64_t dims[2] = {(uint64_t)ws.l_pad, (uint64_t)a->n * a->num_heads};
    const uint64_t str[1] = {(uint64_t)ws.l_pad * 2};
    const uint32_t box[2] = {16, (uint32_t)a->num_heads};
    if ((st = make_map(&tm_e, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, e16, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE)))
      return st;
  }
  if (quant) {
    // 3.2-bit: one 8-byte-element box row per token covering the V window
    CUtensorMap tm_vq;
    const uint64_t dims[3] = {row_elems * es / 8, (uint64_t)a->block_size, (uint64_t)a->num_blocks};
    const uint64_t str[2] = {(uint64_t)a->cache_stride[1] * es, (uint64_t)a->cache_stride[0] * es};
    const uint32_t box[3] = {(uint32_t)pp.v_pitch / 8, 16, 1};
    if ((st = make_map(&tm_vq, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, a->kv_cache, dims, str, box,
                       CU_TENSOR_MAP_SWIZZLE_NONE)))
      return st;
    if ((st = launch_pvq(tm_vq, tm_e, pp, dev.sms, stream))) return st;
  } else {
    // whole 64-channel V tiles of a page in one 4D box {64 channels, 16 slots, tiles,
    // 1 block} over the V part of the rows (tile stride 128 B): one TMA request per
    // page instead of one per tile, which the copy engine serves at a far higher rate
    pp.v_full = a->v_rank / 64;
    pp.v_tail = a->v_rank % 64 != 0;
    pp.box_a = pp.n_ranges > 1 ? 2 * pp.mt_per_range : 0;
    pp.box_b = pp.v_full - 2 * pp.mt_per_range * (pp.n_ranges - 1);
    CUtensorMap tm_va{}, tm_vb{};
    const uint64_t dims[4] = {64, (uint64_t)a->block_size, (uint64_t)std::max(pp.v_full, 1), (uint64_t)a->num_blocks};
    const uint64_t str[3] = {(uint64_t)a->cache_stride[1] * es, 128, (uint64_t)a->cache_stride[0] * es};
    const uint8_t* v_base = static_cast<const uint8_t*>(a->kv_cache) + (size_t)a->k_width * es;
    if (pp.box_a > 0) {
      const uint32_t box[4] = {64, 16, (uint32_t)pp.box_a, 1};
      if ((st = make_map(&tm_va, CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, v_base, dims, str, box,
                         CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    }
    if (pp.box_b > 0) {
      const uint32_t box[4] = {64, 16, (uint32_t)pp.box_b, 1};
      if ((st = make_map(&tm_vb, CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, v_base, dims, str, box,
                         CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    }
    if ((st = launch_pv(tm_v, tm_va, tm_vb, tm_e, pp, dev.sms, stream))) return st;
  }
  if (pev) cudaEventRecord(pev[3], stream);

  // ---- lift ----
  LiftParams lp{};
  lp.pv = pv; lp.pv_stride = ws.pv_stride; lp.l_seq = partial ? nullptr : l_seq;   // partial: no normalisation
  lp.v_up = a->v_up_by_q; lp.vu_s0 = a->v_up_stride[0]; lp.vu_s1 = a->v_up_stride[1]; lp.vu_s2 = a->v_up_stride[2];
  lp.v_up_dtype = a->v_up_dtype;
  lp.out = a->out; lp.o_s0 = a->out_stride[0]; lp.o_s1 = a->out_stride[1]; lp.o_s2 = a->out_stride[2];
  lp.out_dtype = a->out_dtype;
  lp.n = a->n; lp.num_heads = a->num_heads; lp.v_rank = a->v_rank;
  lp.head_dim = a->head_dim;
  st = launch_lift(lp, stream);
  if (st == STARKV_OK && partial) {
    const size_t bytes = (size_t)a->n * a->num_heads * sizeof(float);
    if (cudaMemcpyAsync(m_out, m_seq, bytes, cudaMemcpyDeviceToDevice, stream) != cudaSuccess ||
        cudaMemcpyAsync(l_out, l_seq, bytes, cudaMemcpyDeviceToDevice, stream) != cudaSuccess)
      st = STARKV_ECUDA;
  }
  if (pev) cudaEventRecord(pev[4], stream);
  return st;
}

}  // namespace starkv

extern "C" {

size_t starkv_decode_workspace_bytes(int32_t n, int32_t num_heads, int32_t num_kv_heads, int32_t k_width,
                                     int32_t v_rank, int32_t max_seq_len) {
  if (n < 0 || num_heads <= 0 || num_kv_heads <= 0 || k_width < 0 || v_rank < 0) return 0;
  return starkv::workspace_layout(n, num_heads, num_kv_heads, k_width, v_rank, max_seq_len).total;
}

int starkv_paged_decode_bf16(const StarKVDecodeArgs* args, void* workspace, size_t workspace_bytes, void* stream) {
  return starkv::decode_impl(args, workspace, workspace_bytes, (cudaStream_t)stream, false);
}

int starkv_paged_decode_q32(const StarKVDecodeArgs* args, void* workspace, size_t workspace_bytes, void* stream) {
  return starkv::decode_impl(args, workspace, workspace_bytes, (cudaStream_t)stream, true);
}

int starkv_paged_decode_bf16_partial(const StarKVDecodeArgs* args, int32_t cp_rank, int32_t cp_world, float* m_out,
                                     float* l_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (!m_out || !l_out) return STARKV_EINVAL;
  return starkv::decode_impl(args, workspace, workspace_bytes, (cudaStream_t)stream, false, cp_rank, cp_world, m_out,
                             l_out);
}

int starkv_paged_decode_q32_partial(const StarKVDecodeArgs* args, int32_t cp_rank, int32_t cp_world, float* m_out,
                                    float* l_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (!m_out || !l_out) return STARKV_EINVAL;
  return starkv::decode_impl(args, workspace, workspace_bytes, (cudaStream_t)stream, true, cp_rank, cp_world, m_out,
                             l_out);
}

int starkv_fold_q(const void* query, const int64_t q_stride[3], int32_t q_dtype, const void* k_up,
                  const int64_t k_up_stride[2], int32_t k_up_dtype, const int32_t* head_of_lane, int32_t n,
                  int32_t num_heads, int32_t k_width, float scale, void* ab_out, int32_t* status, void* stream) {
  using namespace starkv;
  if (!query || !k_up || !head_of_lane || !ab_out || !q_stride || !k_up_stride || n < 0 || num_heads <= 0 ||
      k_width <= 0 || k_width % 16)
    return STARKV_EINVAL;
  if (!is_float_dtype(q_dtype) || !is_float_dtype(k_up_dtype)) return STARKV_EDTYPE;
  if (reinterpret_cast<uintptr_t>(ab_out) & 15) return STARKV_EALIGN;
  if (n == 0) return STARKV_OK;
  DeviceInfo dev;
  if (const int st = device_info(dev)) return st;
  FoldParams fp{};
  fp.q = query; fp.q_s0 = q_stride[0]; fp.q_s1 = q_stride[1]; fp.q_s2 = q_stride[2]; fp.q_dtype = q_dtype;
  fp.k_up = k_up; fp.ku_s0 = k_up_stride[0]; fp.ku_s1 = k_up_stride[1]; fp.k_up_dtype = k_up_dtype;
  fp.head_of_lane = head_of_lane;
  fp.n = n; fp.num_heads = num_heads; fp.num_kv_heads = num_heads; fp.group = 1; fp.k_width = k_width;
  fp.head_dim = 128; fp.scale = scale; fp.ab = reinterpret_cast<__half*>(ab_out);
  fp.l_pad = 0; fp.m_count = 0; fp.pv_count = 0;
  fp.status = status;   // a head_of_lane entry outside [0, num_heads) is recorded here (its row is zero)
  return launch_fold(fp, true, (cudaStream_t)stream);
}

int starkv_prefill_attention(const void* q, const int64_t q_stride[2], const void* k, const int64_t k_stride[2],
                             const void* v, const int64_t v_stride[2], int32_t dtype, int32_t num_tokens,
                             int32_t num_heads, int32_t num_k_heads, int32_t num_v_heads, const int32_t* cu_seqlens,
                             int32_t n_prompts, int32_t q_tiles, float scale, void* out, const int64_t o_stride[2],
                             int32_t* status, void* stream) {
  using namespace starkv;
  if (!q || !k || !v || !out || !cu_seqlens || !q_stride || !k_stride || !v_stride || !o_stride || num_tokens < 0 ||
      n_prompts < 0 || q_tiles < 0 || num_heads <= 0 || num_k_heads <= 0 || num_v_heads <= 0 ||
      num_heads % num_k_heads || num_heads % num_v_heads || !(scale > 0.f))
    return STARKV_EINVAL;
  if (dtype != STARKV_BF16 && dtype != STARKV_F16) return STARKV_EDTYPE;
  if (num_tokens == 0 || n_prompts == 0 || q_tiles == 0) return STARKV_OK;
  const int64_t* strides[4] = {q_stride, k_stride, v_stride, o_stride};
  for (const int64_t* s : strides)
    if (s[0] <= 0 || s[1] <= 0 || s[0] % 8 || s[1] % 8) return STARKV_EALIGN;
  for (const void* ptr : {q, k, v, (const void*)out})
    if (reinterpret_cast<uintptr_t>(ptr) & 15) return STARKV_EALIGN;
  DeviceInfo dev;
  if (const int st = device_info(dev)) return st;
  // one 3D map per operand: {128 dims, heads, tokens}, box {64 dims, 1 head, 128
  // tokens}, 128-byte swizzle (the MMA operand layout); tokens past T read as zero
  CUtensorMap maps[3];
  const void* bases[3] = {q, k, v};
  const int heads[3] = {num_heads, num_k_heads, num_v_heads};
  for (int i = 0; i < 3; ++i) {
    const uint64_t dims[3] = {128, (uint64_t)heads[i], (uint64_t)num_tokens};
    const uint64_t str[2] = {(uint64_t)strides[i][1] * 2, (uint64_t)strides[i][0] * 2};
    const uint32_t box[3] = {64, 1, 128};
    if (const int st = make_map(&maps[i], dtype == STARKV_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                             : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                                3, bases[i], dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return st;
  }
  PrefillParams pp{};
  pp.cu_seqlens = cu_seqlens; pp.n_prompts = n_prompts; pp.num_tokens = num_tokens;
  pp.num_heads = num_heads; pp.k_group = num_heads / num_k_heads; pp.v_group = num_heads / num_v_heads;
  pp.dtype = dtype; pp.scale_log2 = scale * 1.4426950408889634f;
  pp.out = out; pp.o_s0 = o_stride[0]; pp.o_s1 = o_stride[1]; pp.status = status;
  return launch_prefill(maps[0], maps[1], maps[2], pp, q_tiles, (cudaStream_t)stream);
}

int starkv_kv_down_cache_write(const void* hidden, int64_t h_stride0, const void* kv_down, int64_t w_stride0,
                               int32_t dtype, int32_t n, int32_t hidden_dim, int32_t out_width, void* kv_cache,
                               const int64_t cache_stride[2], int32_t num_blocks, int32_t block_size,
                               const void* slot_mapping, int32_t slot_dtype, int32_t* status, void* stream) {
  using namespace starkv;
  if (!hidden || !kv_down || !kv_cache || !cache_stride || !slot_mapping || n < 0 || out_width <= 0 ||
      hidden_dim <= 0 || hidden_dim % (64 * kv_down_split()) || num_blocks <= 0 || block_size <= 0 ||
      cache_stride[1] < out_width || cache_stride[0] < cache_stride[1] * block_size || h_stride0 < hidden_dim ||
      w_stride0 < hidden_dim || (slot_dtype != STARKV_I32 && slot_dtype != STARKV_I64))
    return STARKV_EINVAL;
  if (dtype != STARKV_BF16 && dtype != STARKV_F16) return STARKV_EDTYPE;
  if (h_stride0 % 8 || w_stride0 % 8 || cache_stride[0] % 8 || cache_stride[1] % 8) return STARKV_EALIGN;
  for (const void* ptr : {hidden, kv_down, (const void*)kv_cache})
    if (reinterpret_cast<uintptr_t>(ptr) & 15) return STARKV_EALIGN;
  if (n == 0) return STARKV_OK;
  DeviceInfo dev;
  if (const int st = device_info(dev)) return st;
  DownWriteParams dp{};
  dp.n = n; dp.hidden = hidden_dim; dp.out_width = out_width;
  dp.n_tile = std::min(256, (n + 15) / 16 * 16);
  dp.stages = std::min(4, hidden_dim / (64 * kv_down_split()));
  dp.ctl_offset = kv_down_ctl_offset(dp.n_tile, dp.stages);
  dp.dtype = dtype; dp.cache = kv_cache; dp.c_s0 = cache_stride[0]; dp.c_s1 = cache_stride[1];
  dp.num_blocks = num_blocks; dp.block_size = block_size; dp.slot_mapping = slot_mapping;
  dp.slot_dtype = slot_dtype; dp.status = status;
  const CUtensorMapDataType tdt = dtype == STARKV_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tm_w, tm_x;
  {
    // weight rows: box {64 hidden, 128 channels}, 128-byte swizzle; channels past out_width read as zero
    const uint64_t dims[2] = {(uint64_t)hidden_dim, (uint64_t)out_width};
    const uint64_t str[1] = {(uint64_t)w_stride0 * 2};
    const uint32_t box[2] = {64, 128};
    if (const int st = make_map(&tm_w, tdt, 2, kv_down, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B)) return st;
  }
  {
    // token rows: box {64 hidden, n_tile tokens}; tokens past n read as zero
    const uint64_t dims[2] = {(uint64_t)hidden_dim, (uint64_t)n};
    const uint64_t str[1] = {(uint64_t)h_stride0 * 2};
    const uint32_t box[2] = {64, (uint32_t)dp.n_tile};
    if (const int st = make_map(&tm_x, tdt, 2, hidden, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B)) return st;
  }
  return launch_kv_down_write(tm_w, tm_x, dp, (cudaStream_t)stream);
}

int starkv_read_status(void* workspace, int32_t* host_status, int32_t reset, void* stream) {
  if (!workspace || !host_status) return STARKV_EINVAL;
  cudaStream_t s = (cudaStream_t)stream;
  if (cudaMemcpyAsync(host_status, workspace, sizeof(int32_t), cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return STARKV_ECUDA;
  if (cudaStreamSynchronize(s) != cudaSuccess) return STARKV_ECUDA;
  if (reset && cudaMemsetAsync(workspace, 0, sizeof(int32_t), s) != cudaSuccess) return STARKV_ECUDA;
  return STARKV_OK;
}

size_t starkv_status_offset(void) { return 0; }

int starkv_profile_begin(int32_t max_calls) {
  using namespace starkv;
  if (max_calls <= 0) return STARKV_EINVAL;
  if (g_prof.ev) {
    for (int i = 0; i < 5 * g_prof.max_calls; ++i) cudaEventDestroy(g_prof.ev[i]);
    delete[] g_prof.ev;
  }
  g_prof.ev = new cudaEvent_t[5 * max_calls];
  for (int i = 0; i < 5 * max_calls; ++i)
    if (cudaEventCreate(&g_prof.ev[i]) != cudaSuccess) return STARKV_ECUDA;
  g_prof.max_calls = max_calls;
  g_prof.calls = 0;
  g_prof.on = true;
  return STARKV_OK;
}

int starkv_profile_end(float* kernel_ms, int32_t* calls) {
  using namespace starkv;
  if (!kernel_ms || !calls) return STARKV_EINVAL;
  g_prof.on = false;
  for (int k = 0; k < 4; ++k) kernel_ms[k] = 0.f;
  for (int c = 0; c < g_prof.calls; ++c) {
    cudaEvent_t* e = g_prof.ev + 5 * c;
    if (cudaEventSynchronize(e[4]) != cudaSuccess) return STARKV_ECUDA;
    for (int k = 0; k < 4; ++k) {
      float ms = 0.f;
      if (cudaEventElapsedTime(&ms, e[k], e[k + 1]) != cudaSuccess) return STARKV_ECUDA;
      kernel_ms[k] += ms;
    }
  }
  *calls = g_prof.calls;
  return STARKV_OK;
}

size_t starkv_abi_sizeof(int32_t which) {
  switch (which) {
    case 0: return sizeof(StarKVDecodeArgs);
    case 1: return sizeof(StarKVPackArgs);
    case 2: return sizeof(StarKVCacheWriteArgs);
    default: return 0;
  }
}

const char* starkv_version(void) { return "starkv_b200 1.2 (abi 3, sm_100a)"; }

const char* starkv_strerror(int status) {
  switch (status) {
    case STARKV_OK: return "ok";
    case STARKV_EINVAL: return "invalid argument or unsupported shape";
    case STARKV_EALIGN: return "pointer or stride alignment not supported";
    case STARKV_EDTYPE: return "unsupported element type";
    case STARKV_EWORKSPACE: return "workspace missing or too small";
    case STARKV_ECUDA: return "CUDA call failed";
    case STARKV_ENODEV: return "current device is not sm_100";
    case STARKV_EBOUNDS: return "index out of range (recorded on device)";
    case STARKV_ETIMEOUT: return "pipeline wait expired on device";
    default: return "unknown status";
  }
}

}  // extern "C"
