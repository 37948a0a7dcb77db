// Internal launch interface between the C-ABI layer (api.cu) and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace starkv {

// Workspace layout of one decode call (offsets in bytes, 256-aligned).
struct Workspace {
  size_t status;     // int32 status word (+ padding)
  size_t ab;         // f16 [n, group, k_width, 128]   query folded into U (x scale)
  size_t cs;         // f16 [l_pad, 128]                rotary table rows 0..l_pad-1
  size_t e16;        // f16 [n, num_heads, l_pad]       exp(logit - tile max)
  size_t m_tile;     // f32 [n, num_heads, n_tiles]     tile max
  size_t l_seq;      // f32 [n, num_heads]              softmax denominator sum_t p_t
  size_t m_seq;      // f32 [n, num_heads]              sequence max
  size_t pv;         // f32 [n, num_heads, pv_stride]   sum_t p_t * V_t (unnormalised), zero padded
  int pv_stride;     // v_rank rounded up to 64
  size_t total;
  int l_pad, n_tiles;
};

Workspace workspace_layout(int n, int num_heads, int num_kv_heads, int k_width, int v_rank, int max_seq_len);

struct ScoresParams {
  const int32_t* seq_lens;
  const int32_t* block_table;
  int64_t bt_s0, bt_s1;
  int max_blocks;
  int n, num_heads, num_kv_heads, group, k_width, num_blocks, block_size, max_seq_len;
  int cache_dtype;
  const int32_t* k_ranks;
  const int32_t* k_head_offsets;
  const int32_t* tile_head;
  const int32_t* tile_nout;
  const int32_t* tile_last;
  int ks_off;                      // 3.2-bit: byte offset of the K scales in a row
  int code_pitch, tail_pitch;      // staged row pitch of a full / the last code window (bytes)
  int n_wins;                      // code windows per row
  int sc_pitch, sc_x0;             // 3.2-bit: staged scale window (pitch, 16-aligned byte start)
  int cp_rank, cp_world;           // context split: this rank decodes its share of each sequence's
                                   // 256-token tiles (rank r of w: tiles [T*r/w, T*(r+1)/w))
  __half* e16;
  float* m_tile;
  float* m_seq;
  int l_pad, n_tiles;
  int32_t* status;
};

struct PvParams {
  const int32_t* seq_lens;
  const int32_t* block_table;
  int64_t bt_s0, bt_s1;
  int max_blocks;
  int n, num_heads, k_width, v_rank, num_blocks, block_size, max_seq_len;
  int nh;                 // MMA N: num_heads rounded up to a multiple of 16
  int n_mtiles;           // 128-channel tiles over the V code (all ranges)
  int mt_per_range;       // tiles handled per work item (TMEM columns = mt_per_range * nh)
  int n_ranges;
  int cache_dtype;
  // 3.2-bit V layout (paged_quant.QuantRow)
  int v_nout, v_nbo, v_bytes, vq_off, vs_off, vx0;
  int v_pitch;            // 3.2-bit: staged row pitch of the V window [vx0, vq_off + v_bytes), odd x 16 B
  int cp_rank, cp_world;  // context split, as in ScoresParams (pages of the rank's 256-token tiles)
  int t_out;              // tiles over the outlier block (the rest cover inliers)
  // bf16 / f16 V tiles: v_rank / 64 whole 64-channel tiles come in one 4D box per page
  // (box_a tiles for every range but the last, box_b for the last one); a trailing
  // 32-channel tile (v_tail) comes in a 3D box of its own
  int v_full, box_a, box_b, v_tail;
  const __half* e16;
  const float* m_tile;
  const float* m_seq;
  float* l_seq;
  float* pv;
  int pv_stride;
  int l_pad, n_tiles;
  int32_t* status;
};

struct LiftParams {
  const float* pv;        // [n, H, pv_stride]
  int pv_stride;
  const float* l_seq;     // null: no normalisation (context-parallel partial output)
  const void* v_up; int64_t vu_s0, vu_s1, vu_s2; int v_up_dtype;   // [H, rv, Hd]
  void* out; int64_t o_s0, o_s1, o_s2; int out_dtype;              // [n, H, Hd]
  int n, num_heads, v_rank, head_dim;
};

struct FoldParams {
  const void* q; int64_t q_s0, q_s1, q_s2; int q_dtype;
  const void* k_up; int64_t ku_s0, ku_s1; int k_up_dtype;
  const int32_t* head_of_lane;     // 3.2-bit path (reference semantics: no rank mask)
  const int32_t* k_ranks;          // bf16 path: lanes past a head's rank get zero rows
  const int32_t* k_head_offsets;
  int n, num_heads, num_kv_heads, group, k_width, head_dim;
  float scale;
  __half* ab;                      // [n, group, W, 128], or the MMA image below when ab_image
  int ab_image;                    // 1: per (b, j, 128-lane chunk c, 64-lane half r) a 16 KB block
                                   //    [k half][64 lanes][128 B], 16-byte units XOR-swizzled by lane & 7
  // rotary table -> f16 copy
  const void* cs; int64_t cs_s0, cs_s1; int cs_dtype; int cs_rows;
  __half* cs16; int l_pad, max_seq_len;   // per 128-token tile a 32 KB block [k half][128 rows][128 B],
                                          // 16-byte units XOR-swizzled by row & 7
  // per-call initialisation
  float* m_seq; float* l_seq; int m_count;
  float* pv; int64_t pv_count;
  int32_t* status;
};

struct PrefillParams {
  const int32_t* cu_seqlens;       // [n_prompts + 1] token offsets of the prompts
  int n_prompts, num_tokens;
  int num_heads;                   // query heads (grid.y)
  int k_group, v_group;            // query heads per K head / per V head
  int dtype;                       // STARKV_BF16 or STARKV_F16 (q, k, v and out)
  float scale_log2;                // softmax scale * log2(e)
  void* out; int64_t o_s0, o_s1;   // [T, num_heads, 128], strides in elements
  int32_t* status;
};

struct DownWriteParams {
  int n, hidden, out_width;        // tokens, K, code channels (k_width + v_rank)
  int n_tile, stages, ctl_offset;  // tokens per launch column (multiple of 16, <= 256), K-block ring
  int dtype;                       // STARKV_BF16 or STARKV_F16 (hidden, kv_down and the cache)
  void* cache; int64_t c_s0, c_s1; int num_blocks, block_size;   // strides in elements
  const void* slot_mapping; int slot_dtype;
  int32_t* status;
};

size_t scores_smem_bytes(bool quant, int num_kv_heads, int n, int k_width, int code_pitch, int sc_pitch,
                         bool parts);
int code_pitch_bytes(int bytes);
int scores_window_bytes(bool quant);
size_t pv_smem_bytes(const PvParams& p);
int pv_page_stages(const PvParams& p);
size_t pvq_smem_bytes(const PvParams& p);
int pvq_page_stages(const PvParams& p);
int pvq_max_dequant_tasks();
int launch_pvq(const CUtensorMap& tm_v, const CUtensorMap& tm_e, const PvParams& p, int num_sms, cudaStream_t stream);

int launch_fold(const FoldParams& p, bool quant, cudaStream_t stream);
int launch_scores(bool quant, const CUtensorMap& tm_cs, const CUtensorMap& tm_ab, const CUtensorMap& tm_code,
                  const CUtensorMap& tm_tail, const CUtensorMap& tm_sc, const ScoresParams& p, int num_sms,
                  cudaStream_t stream);
int launch_pv(const CUtensorMap& tm_v, const CUtensorMap& tm_va, const CUtensorMap& tm_vb, const CUtensorMap& tm_e,
              const PvParams& p, int num_sms, cudaStream_t stream);
int launch_lift(const LiftParams& p, cudaStream_t stream);
int launch_lift_cluster(const LiftParams& p, cudaStream_t stream);   // -1: layout not taken
size_t kv_down_smem_bytes(int n_tile, int stages);
int kv_down_ctl_offset(int n_tile, int stages);
int kv_down_split();
int launch_kv_down_write(const CUtensorMap& tm_w, const CUtensorMap& tm_x, const DownWriteParams& p,
                         cudaStream_t stream);
int launch_prefill(const CUtensorMap& tm_q, const CUtensorMap& tm_k, const CUtensorMap& tm_v, const PrefillParams& p,
                   int q_tiles, cudaStream_t stream);

}  // namespace starkv
