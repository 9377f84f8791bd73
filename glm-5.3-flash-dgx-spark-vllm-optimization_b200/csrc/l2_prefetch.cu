// L2 prefetch of the next layer's projection weights while the routed MoE runs (decode).
//
// The decode MoE is bound by the ALU work of the trellis decode and leaves most of the HBM bandwidth idle for
// hundreds of microseconds per layer; the projections that start the next layer (the KDA input projection, or the
// MLA query / key-value projections) are bandwidth-bound GEMVs.  This kernel issues bulk L2 prefetches
// (cp.async.bulk.prefetch.L2, 64 KB each, no completion to wait for) of up to four weight ranges and exits at once;
// the MoE's own trellis loads carry an evict-first L2 policy, so the prefetched lines outlive the stream and the
// next GEMV reads them from L2.  The role of the reference's FP8 "roof" L2-warming side stream
// (code/fork/fp8_roof.py:1-40), done here with the copy engine's prefetch instead of a warming kernel's loads.
#include <cstdint>
#include "launchers.h"

namespace g53 {

constexpr int64_t kPrefetchChunk = 64 << 10;

__global__ void __launch_bounds__(128) l2_prefetch_kernel(L2Ranges r) {
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int j = 0; j < r.count; ++j) {
    const int64_t n = r.bytes[j];
    const int64_t chunks = (n + kPrefetchChunk - 1) / kPrefetchChunk;
    for (int64_t c = tid; c < chunks; c += nth) {
      const int64_t off = c * kPrefetchChunk;
      const int64_t rem = n - off;
      const uint32_t sz = (uint32_t)((rem < kPrefetchChunk ? rem : kPrefetchChunk) & ~(int64_t)15);
      if (sz) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(r.ptr[j] + off), "r"(sz) : "memory");
    }
  }
}

}  // namespace g53

cudaError_t g53_l2_prefetch(const L2Ranges& r, cudaStream_t st) {
  if (r.count <= 0) return cudaSuccess;
  for (int j = 0; j < r.count; ++j)
    if (reinterpret_cast<uintptr_t>(r.ptr[j]) % 16 != 0) return cudaErrorInvalidValue;
  g53::l2_prefetch_kernel<<<4, 128, 0, st>>>(r);
  return cudaGetLastError();
}
