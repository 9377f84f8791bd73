// Allocation-free entry point of the MLA flash-decoding kernel.
//
// This entry point has no counterpart in the reference; it exists for callers of this library that cannot
// allocate device memory themselves -- for example code running inside a host allocator hook, a runtime that
// forbids cudaMalloc after start-up, or a plain C caller without a CUDA-aware allocator.  The regular entry point
// (g53_mla_decode) needs the caller to provide two scratch buffers for the per-split partial results; this one
// keeps them in a fixed-size array that lives in the library's device image, so the caller passes only inputs and
// outputs and nothing is allocated at call time.
//
// Limits and behaviour:
//   * the scratch array holds G53_MLA_NOALLOC_MAX_PARTIAL floats of partial outputs (R * splits * H * L) and
//     G53_MLA_NOALLOC_MAX_STATS floats of softmax statistics (R * splits * H * 2); larger problems are rejected
//     with G53_NOALLOC_ERR_TOO_LARGE before anything is launched.  Every GPU that loads the library keeps this
//     array (about 4.1 MB) for the life of the process.
//   * arguments are checked on the host before any launch: null inputs or outputs, a rope kernel (rope > 0)
//     without q_pe / kpe_cache, an (L, rope) pair other than (512, 0), (128, 0), (128, 32), splits outside
//     [1, 16] or max_sel < 1 return cudaErrorInvalidValue.  A row's sel_count is clamped to max_sel on the device.
//   * a failed device lookup returns its cudaError_t (for example cudaErrorInvalidDevice); only a failed symbol
//     lookup returns G53_NOALLOC_ERR_SYMBOL.
//   * nothing in the scratch has to start at zero: each call writes every partial it later reads.
//   * all calls on a device share the one array, so calls that can overlap on the GPU (different streams, or
//     different host threads, without ordering between them) race and corrupt each other's results; order them
//     on one stream or synchronise between them.
//   * the first call on a device looks up the device address of the array (cudaGetSymbolAddress) with that device
//     current; make that first call before starting any stream capture on that device.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define G53_MLA_NOALLOC_MAX_PARTIAL (1 << 20)
#define G53_MLA_NOALLOC_MAX_STATS (1 << 15)
#define G53_NOALLOC_ERR_TOO_LARGE 1001
#define G53_NOALLOC_ERR_SYMBOL 1002

#ifdef __cplusplus
extern "C" {
#endif

// Same arguments as MlaAttnArgs minus the two scratch buffers; returns 0 on success, a cudaError_t value, or one
// of the G53_NOALLOC_ERR_* codes.  `stream` is a cudaStream_t (0 = legacy default stream).
int g53_mla_decode_noalloc(const void* q_lat, const void* q_pe, int64_t q_pe_ld, int q_pe_hs, const void* kv_cache,
                           const float* kv_scale, const void* kpe_cache, const int* sel, const int* sel_count,
                           int max_sel, int R, int H, int L, int rope, float sm_scale, int splits, void* o_lat,
                           void* stream);

// Human-readable text of a return code of g53_mla_decode_noalloc.
const char* g53_mla_decode_noalloc_error(int code);

#ifdef __cplusplus
}
#endif
