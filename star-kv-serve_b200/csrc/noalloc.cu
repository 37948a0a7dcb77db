// Decode entry point for callers that cannot allocate device memory.
//
// Some hosts of this library cannot call cudaMalloc or any allocating runtime:
// an inference server whose memory pool is fixed at start-up (all device memory
// already handed to the KV cache), a process that runs under a strict allocator
// policy, or a plug-in loaded into an engine that owns every allocation. They
// can still pass input and output buffers, but cannot hand us a workspace.
// starkv_paged_decode_bf16_noalloc serves them: the decode scratch lives in the
// file-scope device array below, which the CUDA runtime places in device memory
// when it loads this library's module on a GPU and keeps there until the process
// exits (STARKV_NOALLOC_SCRATCH_BYTES on every GPU that loads the library).
//
// In host code `g_noalloc_scratch` only names a host-side stand-in for the
// array, never a device address; its device address is looked up with
// cudaGetSymbolAddress by the first call on each device (with that device
// current) and cached once the lookup succeeds. That first call should
// therefore happen before any stream capture. Device-side errors the kernels
// record in the array's status word are read with starkv_noalloc_read_status.
//
// All calls share the one array and it keeps the previous call's contents: the
// decode kernels initialise every accumulator they read (sequence max, softmax
// denominator, P.V sums) and this entry point clears the status word, so nothing
// leaks from call to call. Two calls whose kernels overlap on the GPU (different
// streams, no ordering between them) race on the array and give wrong results.
#include <cuda_runtime.h>

#include <mutex>

#include "starkv_common.cuh"

namespace {

constexpr size_t kScratchBytes = STARKV_NOALLOC_SCRATCH_BYTES;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

// Device address of the scratch array per device. Only a successful lookup is
// kept: a failed one (say, a first call made during stream capture) is retried
// by the next call instead of disabling the entry point for the process.
std::mutex g_scratch_mu;
void* g_scratch_of[64] = {};

// Device address of the scratch array on the current device.
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return STARKV_ECUDA;
  if (dev < 0 || dev >= 64) return STARKV_ENODEV;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_of[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();   // a failed lookup leaves no error behind for the caller's next CUDA call
      return STARKV_ECUDA;
    }
    g_scratch_of[dev] = p;
  }
  *out = g_scratch_of[dev];
  return STARKV_OK;
}

}  // namespace

extern "C" int starkv_paged_decode_bf16_noalloc(const StarKVDecodeArgs* args, void* stream) {
  if (!args) return STARKV_EINVAL;
  // Reject a call whose scratch would not fit before touching the GPU.
  const size_t need = starkv_decode_workspace_bytes(args->n, args->num_heads, args->num_kv_heads, args->k_width,
                                                    args->v_rank, args->max_seq_len);
  if (need == 0) return STARKV_EINVAL;
  if (need > kScratchBytes) return STARKV_EWORKSPACE;
  void* scratch = nullptr;
  const int st = scratch_address(&scratch);
  if (st != STARKV_OK) return st;
  // the device status word starts each call cleared (offset starkv_status_offset())
  if (cudaMemsetAsync(static_cast<uint8_t*>(scratch) + starkv_status_offset(), 0, sizeof(int32_t),
                      static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return STARKV_ECUDA;
  return starkv_paged_decode_bf16(args, scratch, kScratchBytes, stream);
}

// Status word of the built-in scratch on the current device: the device-side
// errors the decode kernels record there (STARKV_EBOUNDS for a block id outside
// the cache, STARKV_ETIMEOUT for an expired pipeline wait). Synchronises the
// stream; cleared when reset != 0 (each noalloc call also clears it on entry).
extern "C" int starkv_noalloc_read_status(int32_t* host_status, int32_t reset, void* stream) {
  if (!host_status) return STARKV_EINVAL;
  void* scratch = nullptr;
  const int st = scratch_address(&scratch);
  if (st != STARKV_OK) return st;
  return starkv_read_status(static_cast<uint8_t*>(scratch) + starkv_status_offset(), host_status, reset, stream);
}
