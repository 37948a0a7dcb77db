// Helpers shared by the P.V kernels (pv.cu: bf16 codes, pvq.cu: 3.2-bit codes):
// page-range bookkeeping of the work split, operand offsets, TMEM reads.
#pragma once

#include "starkv_common.cuh"
#include "starkv_kernels.h"

namespace starkv {
namespace pvc {

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

__device__ __forceinline__ bool next_sub(int& u, int u_end, int total_pages, const int* pprefix, const int* pbeg,
                                         int n, SubItem& si) {
  if (u >= u_end) return false;
  si.range = u / total_pages;
  const int pi = u % total_pages;
  si.b = find_le(pprefix, n, pi);
  si.page0 = pi - pprefix[si.b] + pbeg[si.b];   // absolute page of the sequence
  const int seq_end = si.range * total_pages + pprefix[si.b + 1];
  const int e = min(u_end, seq_end);
  si.npages = e - u;
  u = e;
  return true;
}


// Prefix of this rank's pages over the sequences (pprefix[n+1]) and the first page
// of each sequence's share (pbeg[n]): a rank of a context split owns the pages of
// its 256-token tiles [T r / w, T (r+1) / w).
__device__ __forceinline__ void page_ranges(const PvParams& p, int* pprefix, int* pbeg) {
  int acc = 0;
  for (int b = 0; b < p.n; ++b) {
    pprefix[b] = acc;
    const int L = min(max(p.seq_lens[b], 0), p.max_seq_len);
    const int T = (L + 255) >> 8;
    const int s0 = (int)((int64_t)T * p.cp_rank / p.cp_world), s1 = (int)((int64_t)T * (p.cp_rank + 1) / p.cp_world);
    const int pg0 = 16 * s0, pg1 = min(16 * s1, (L + 15) >> 4);
    pbeg[b] = pg0;
    acc += max(pg1 - pg0, 0);
  }
  pprefix[p.n] = acc;
}

}  // namespace pvc
}  // namespace starkv
