/*
 * starkv_b200.h -- C ABI of the B200 (sm_100a) STAR-KV paged low-rank decode library.
 *
 * Plain pointers, sizes and element strides; no framework types. Every entry
 * point is asynchronous on the caller's CUDA stream, allocates nothing, never
 * synchronises the device and returns an int status (0 = ok, see
 * STARKV_E* below). Device-side bounds violations (a block id outside the
 * cache, a slot outside the cache) are recorded in a status word inside the
 * caller's workspace and read back with starkv_read_status (tests, debugging).
 *
 * Reference interfaces each entry point replaces (paths inside the
 * STAR-KV-Serve project):
 *   starkv_paged_decode_bf16   starkv_serve/kernels/paged_decode.py:150-226 (paged_starkv_decode)
 *   starkv_paged_decode_q32    starkv_serve/kernels/paged_quant.py:357-411  (paged_quant_decode)
 *   starkv_fold_q              starkv_serve/kernels/paged_quant.py:241-255  (fold_q)
 *   starkv_pack_kv_q32         starkv_serve/kernels/paged_quant.py:205-216  (pack_kv)
 *   starkv_cache_write_bf16    starkv_serve/attention.py:179-185            (bf16 cache write)
 *   starkv_decode_workspace_bytes   no reference counterpart: the reference
 *                              allocates its logits / segment buffers with
 *                              torch per call (paged_decode.py:179, 206;
 *                              paged_quant.py:251, 379, 401); here the caller
 *                              owns one reusable workspace, so calls can be
 *                              captured in CUDA graphs.
 */
#ifndef STARKV_B200_H
#define STARKV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* 3: adds starkv_prefill_attention and starkv_kv_down_cache_write (2: starkv_fold_q
 * takes a status word) */
#define STARKV_ABI_VERSION 3

#if defined(__GNUC__)
#define STARKV_API __attribute__((visibility("default")))
#else
#define STARKV_API
#endif

/* element types */
enum {
  STARKV_F16 = 0,
  STARKV_BF16 = 1,
  STARKV_F32 = 2,
  STARKV_U8 = 3,
  STARKV_I32 = 4,
  STARKV_I64 = 5
};

/* status codes */
enum {
  STARKV_OK = 0,
  STARKV_EINVAL = 22,     /* shape / argument not supported (reference: assert)      */
  STARKV_EALIGN = 100,    /* pointer or stride alignment not usable by TMA / vectors  */
  STARKV_EDTYPE = 101,    /* element type not supported                               */
  STARKV_EWORKSPACE = 102,/* workspace pointer null or smaller than required          */
  STARKV_ECUDA = 103,     /* a CUDA runtime / driver call failed                      */
  STARKV_ENODEV = 104,    /* current device is not sm_100                             */
  STARKV_EBOUNDS = 105,   /* device status word: index out of range (recorded, skipped)*/
  STARKV_ETIMEOUT = 106   /* device status word: a bounded pipeline wait expired      */
};

/*
 * Arguments of one decode call over one layer's paged cache.
 *
 * bf16 path (paged_decode.py:150-166): kv_cache is [num_blocks, block_size,
 * k_width + v_rank] in cache_dtype (bf16 or f16), strides in ELEMENTS.
 * 3.2-bit path (paged_quant.py:357-371): kv_cache is uint8 [num_blocks,
 * block_size, row_nbytes], strides in BYTES, with the QuantRow offsets below.
 *
 * Tensors: query [n, num_heads, head_dim] (RoPE applied); block_table
 * [n, max_blocks] int32; seq_lens [n] int32; k_up [k_width, head_dim];
 * k_ranks / k_head_offsets [num_kv_heads] int32 (device); v_up_by_q
 * [num_heads, v_rank, head_dim]; cos_sin_cache [cs_rows, head_dim] =
 * cat(cos, sin); out [n, num_heads, head_dim]. All pointers are device
 * pointers; all strides are element strides unless noted.
 */
typedef struct StarKVDecodeArgs {
  const void* query;          int64_t q_stride[3];    int32_t q_dtype;
  const void* kv_cache;       int64_t cache_stride[3]; int32_t cache_dtype;
  int32_t num_blocks;         int32_t block_size;
  const int32_t* block_table; int64_t bt_stride[2];   int32_t max_blocks;
  const int32_t* seq_lens;
  int32_t n;                  int32_t num_heads;      int32_t num_kv_heads; int32_t head_dim;
  int32_t max_seq_len;        /* host bound on seq_lens (max_model_len inside a CUDA graph) */
  const void* k_up;           int64_t k_up_stride[2]; int32_t k_up_dtype;
  const int32_t* k_ranks;     const int32_t* k_head_offsets;
  int32_t k_width;
  const void* v_up_by_q;      int64_t v_up_stride[3]; int32_t v_up_dtype;
  int32_t v_rank;
  const void* cos_sin_cache;  int64_t cs_stride[2];   int32_t cs_dtype; int32_t cs_rows;
  float scale;
  void* out;                  int64_t out_stride[3];  int32_t out_dtype;
  /* 3.2-bit path only (paged_quant.QuantRow, paged_quant.py:71-111; k_tables :114-131) */
  int32_t row_nbytes, ks_off, vs_off, vq_off, v_nout, v_nbo, v_bytes;
  const int32_t* head_of_lane;                      /* [k_width]                   */
  const int32_t* tile_head; const int32_t* tile_nout; const int32_t* tile_last; /* [k_width/16] */
} StarKVDecodeArgs;

/* Bytes of workspace a decode call with these sizes needs (both paths). */
STARKV_API size_t starkv_decode_workspace_bytes(int32_t n, int32_t num_heads, int32_t num_kv_heads,
                                     int32_t k_width, int32_t v_rank, int32_t max_seq_len);

/* paged_decode.py:150-226 -- bf16/f16 codes. */
STARKV_API int starkv_paged_decode_bf16(const StarKVDecodeArgs* args, void* workspace, size_t workspace_bytes,
                             void* stream);

/*
 * No counterpart in the reference. The bf16/f16 decode above for callers that
 * cannot allocate device memory (a host whose device memory is all handed out
 * at start-up, or a plug-in inside an engine that owns every allocation): it
 * takes no workspace and runs in a scratch array built into the library,
 * STARKV_NOALLOC_SCRATCH_BYTES on every GPU that loads the library, held until
 * the process exits. Calls needing more scratch than that
 * (starkv_decode_workspace_bytes) return STARKV_EWORKSPACE before any GPU work.
 * The first call on a device looks the array's address up (with that device
 * current) and should come before any stream capture. All calls share the
 * array: calls whose kernels overlap on the GPU race; keep them ordered on one
 * stream. Its device status word is cleared at the start of each call and read
 * with starkv_noalloc_read_status below. A failed first address lookup is
 * retried by the next call.
 */
#define STARKV_NOALLOC_SCRATCH_BYTES ((size_t)16 << 20)
STARKV_API int starkv_paged_decode_bf16_noalloc(const StarKVDecodeArgs* args, void* stream);

/*
 * No counterpart in the reference. Device status word of the built-in scratch
 * on the current device: what the last starkv_paged_decode_bf16_noalloc call's
 * kernels recorded (STARKV_EBOUNDS: a block id outside the cache was skipped;
 * STARKV_ETIMEOUT: a pipeline wait expired), 0 if nothing. Synchronises the
 * stream (tests, debugging); clears the word when reset != 0.
 */
STARKV_API int starkv_noalloc_read_status(int32_t* host_status, int32_t reset, void* stream);

/* paged_quant.py:357-411 -- 3.2-bit codes (MHA, head_dim 128). */
STARKV_API int starkv_paged_decode_q32(const StarKVDecodeArgs* args, void* workspace, size_t workspace_bytes,
                            void* stream);

/*
 * Context-parallel share of the two decodes above: the next step after
 * head sharding for multi-GPU decode (the reference has no multi-GPU path;
 * model.py:32-33 rejects tensor parallelism). Rank cp_rank of cp_world decodes,
 * for every head, its contiguous share of each sequence's 256-token tiles
 * (tiles [T*r/w, T*(r+1)/w) of T = ceil(seq_len/256)) and returns
 *   out   f32 [n, num_heads, 128] (args->out, out_dtype STARKV_F32):
 *         sum_t exp(logit_t - m) V_t . v_up_by_q, unnormalised;
 *   m_out f32 [n, num_heads]: that max m of the rank's logits (-inf if the rank
 *         holds no token of the sequence); l_out: sum_t exp(logit_t - m).
 * Ranks combine as out = sum_r exp(m_r - M) out_r / sum_r exp(m_r - M) l_r with
 * M = max_r m_r (starkv_b200.context_parallel). cp_world = 1 gives the whole
 * sequence. Errors as for the full decode.
 */
STARKV_API int starkv_paged_decode_bf16_partial(const StarKVDecodeArgs* args, int32_t cp_rank, int32_t cp_world,
                                                float* m_out, float* l_out, void* workspace, size_t workspace_bytes,
                                                void* stream);
STARKV_API int starkv_paged_decode_q32_partial(const StarKVDecodeArgs* args, int32_t cp_rank, int32_t cp_world,
                                               float* m_out, float* l_out, void* workspace, size_t workspace_bytes,
                                               void* stream);

/*
 * Self-test of the kernels' bounded pipeline waits (no counterpart in the
 * reference): one thread waits on a barrier that nothing completes. The wait gives
 * up after its poll limit (about a second) and records STARKV_ETIMEOUT in the
 * device status word `status` (caller-zeroed int32), as every pipeline wait in
 * the decode kernels does instead of hanging.
 */
STARKV_API int starkv_selftest_wait_timeout(int32_t* status, void* stream);

/*
 * Combine of context-parallel partials (no counterpart in the reference):
 * parts holds `world` packed partials one after the other, each
 *   out f32 [n, H, 128] | m f32 [n, H] | l f32 [n, H]   (n*H*130 floats)
 * as written by the *_partial calls into one buffer (starkv_b200.context_parallel
 * gathers them from the ranks). Writes the combined [n, H, 128] output (strides in
 * elements, bf16 / f16 / f32): sum_r exp(m_r - M) out_r / sum_r exp(m_r - M) l_r.
 */
STARKV_API int starkv_cp_combine(const float* parts, int32_t world, int32_t n, int32_t num_heads, void* out,
                                 const int64_t out_stride[3], int32_t out_dtype, void* stream);

/*
 * paged_quant.py:241-255 (fold_q): q [n, H, 128] (RoPE applied), k_up [W, 128],
 * head_of_lane [W] -> ab [n, W, 128] f16 (contiguous), the logit scale folded in:
 *   A[r,i] = (q_i U[r,i] + q_{i+64} U[r,i+64]) * scale
 *   B[r,i] = (q_{i+64} U[r,i] - q_i U[r,i+64]) * scale
 * q and k_up are bf16, f16 or f32 (else STARKV_EDTYPE); W is a multiple of 16.
 * A head_of_lane entry outside [0, H) gives a zero row and is recorded as
 * STARKV_EBOUNDS in *status (optional device int32; null: not recorded).
 */
STARKV_API int starkv_fold_q(const void* query, const int64_t q_stride[3], int32_t q_dtype,
                  const void* k_up, const int64_t k_up_stride[2], int32_t k_up_dtype,
                  const int32_t* head_of_lane, int32_t n, int32_t num_heads, int32_t k_width,
                  float scale, void* ab_out, int32_t* status, void* stream);

/*
 * attention.py:246-250 (flash_attn_varlen_func in _dense_prefill): causal attention
 * of whole prompts over their own keys. Prompt p holds tokens
 * cu_seqlens[p] .. cu_seqlens[p+1] (device int32, n_prompts + 1 entries) of
 *   q   [T, num_heads, 128]      rotated queries
 *   k   [T, num_k_heads, 128]    lifted, rotated keys (query head h reads K head
 *                                h / (num_heads / num_k_heads))
 *   v   [T, num_v_heads, 128]    lifted values (num_v_heads = num_heads: one V per
 *                                query head; = num_k_heads: per KV head)
 * -> out [T, num_heads, 128] = softmax(scale q k^T, key <= query) v.
 * Strides are in elements, {token, head}; the last dimension is contiguous and the
 * pointers and strides give 16-byte aligned rows. q, k, v and out share one dtype,
 * STARKV_BF16 or STARKV_F16 (else STARKV_EDTYPE); scale > 0. q_tiles = sum over prompts of
 * ceil(len / 128) (the grid; the kernel finds each tile's prompt in cu_seqlens).
 * A cu_seqlens entry outside [0, T] is recorded as STARKV_EBOUNDS in *status
 * (optional device int32).
 */
STARKV_API int starkv_prefill_attention(const void* q, const int64_t q_stride[2], const void* k,
                  const int64_t k_stride[2], const void* v, const int64_t v_stride[2], int32_t dtype,
                  int32_t num_tokens, int32_t num_heads, int32_t num_k_heads, int32_t num_v_heads,
                  const int32_t* cu_seqlens, int32_t n_prompts, int32_t q_tiles, float scale, void* out,
                  const int64_t o_stride[2], int32_t* status, void* stream);

/*
 * model.py:70 (codes = F.linear(hidden, kv_down)) fused with the cache write of
 * attention.py:179-185: cache[slot_t] row [0, out_width) = hidden_t . kv_down^T for
 * the n tokens, rounded once to the cache dtype, so the codes never go through
 * global memory. hidden [n, hidden_dim] (row stride h_stride0 elements), kv_down
 * [out_width, hidden_dim] (row stride w_stride0), both of `dtype` (STARKV_BF16 or
 * STARKV_F16, as the cache; else STARKV_EDTYPE), last dimensions contiguous, rows
 * 16-byte aligned; hidden_dim a multiple of 512; cache [num_blocks, block_size, >=
 * out_width] with strides cache_stride (elements) multiples of 8. slot_mapping int32
 * or int64 [n]; slot -1 (CUDA-graph padding) writes the reserved null slot 0, as
 * attention.py:181 clamps it; a slot past the cache is recorded as STARKV_EBOUNDS
 * in *status (optional device int32) and not written.
 */
STARKV_API int starkv_kv_down_cache_write(const void* hidden, int64_t h_stride0, const void* kv_down,
                  int64_t w_stride0, int32_t dtype, int32_t n, int32_t hidden_dim, int32_t out_width,
                  void* kv_cache, const int64_t cache_stride[2], int32_t num_blocks, int32_t block_size,
                  const void* slot_mapping, int32_t slot_dtype, int32_t* status, void* stream);

/* paged_quant.py:205-216 (pack_kv): quantize n tokens' codes into their slots. */
typedef struct StarKVPackArgs {
  const void* k_codes; int64_t k_stride0; int32_t k_dtype;   /* [n, k_width], unit inner stride */
  const void* v_codes; int64_t v_stride0; int32_t v_dtype;   /* [n, v_rank],  unit inner stride */
  void* cache; int64_t cache_stride[2];                      /* uint8, BYTE strides of dims 0, 1 */
  int32_t num_blocks, block_size;
  const void* slot_mapping; int32_t slot_dtype;              /* [n] int32 or int64; -1 -> slot 0 */
  int32_t n, num_kv_heads, k_width, v_rank;
  const int32_t* k_ranks; const int32_t* k_offsets; const int32_t* k_nouts; /* device [H] */
  int32_t ks_off, vs_off, vq_off, v_nout, v_nbo, v_bytes;
  int32_t* status;                                           /* optional device status word */
} StarKVPackArgs;
STARKV_API int starkv_pack_kv_q32(const StarKVPackArgs* args, void* stream);

/* attention.py:179-185: cache[slot // bs, slot % bs] = cat(key, value) (slot -1 -> 0). */
typedef struct StarKVCacheWriteArgs {
  const void* key; int64_t key_stride0; int32_t key_dtype;       /* [n, k_width] */
  const void* value; int64_t value_stride0; int32_t value_dtype; /* [n, v_rank]  */
  void* cache; int64_t cache_stride[3]; int32_t cache_dtype;     /* element strides */
  int32_t num_blocks, block_size;
  const void* slot_mapping; int32_t slot_dtype;
  int32_t n, k_width, v_rank;
  int32_t* status;
} StarKVCacheWriteArgs;
STARKV_API int starkv_cache_write_bf16(const StarKVCacheWriteArgs* args, void* stream);

/* Copy the device status word of a workspace to the host (synchronises the
 * stream; for tests and debugging, never on the decode path). Clears it when
 * reset != 0. */
STARKV_API int starkv_read_status(void* workspace, int32_t* host_status, int32_t reset, void* stream);

/* Offset of the status word inside a decode workspace (pack / cache-write
 * calls may point their `status` at it). */
STARKV_API size_t starkv_status_offset(void);

/* Per-kernel timing of decode calls, for benchmarking (no reference
 * counterpart). begin() creates events for up to max_calls decode calls and
 * makes each call record them on its stream around its 4 kernels (fold, scores,
 * pv, lift); end() waits for them and returns the summed milliseconds per
 * kernel over the recorded calls. Not thread-safe; not for production paths. */
STARKV_API int starkv_profile_begin(int32_t max_calls);
STARKV_API int starkv_profile_end(float* kernel_ms /* [4] */, int32_t* calls);

/* sizeof of the argument structs (0: StarKVDecodeArgs, 1: StarKVPackArgs,
 * 2: StarKVCacheWriteArgs), so a foreign-function binding can check its
 * struct layout against the library. No reference counterpart. */
STARKV_API size_t starkv_abi_sizeof(int32_t which);

STARKV_API const char* starkv_version(void);
STARKV_API const char* starkv_strerror(int status);

#ifdef __cplusplus
}
#endif
#endif /* STARKV_B200_H */
