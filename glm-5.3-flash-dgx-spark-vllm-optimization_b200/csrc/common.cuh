// Shared device helpers for the glm53 sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>
#include <cstdlib>

#define G53_CHECK_LAUNCH() do { cudaError_t e_ = cudaGetLastError(); if (e_ != cudaSuccess) return e_; } while (0)

// ---------------------------------------------------------------------------------------------------------------
// Bounds-checked debug build (GLM53_BOUNDS=1 compiles every source with -DG53_BOUNDS=1 into a second library).
// Indices that come from device data (token ids, cache slots from page tables and selections, state-pool slots,
// expert ids and row ids of the routing tables) are checked against the size of what they index.  An index out of
// range records (code, index, limit) in this source file's error record and the access is skipped (the kernel
// returns, skips the item, or reads a substitute in-range element); no assert and no trap, so the context stays
// usable.  The host reads and clears the records of every source file (bounds_status / bounds_reset).  In the
// regular build the checks compile to nothing.  A limit of 0 means "unknown" (not checked).
// Codes: 1 embedding row, 2 MLA cache slot written, 3 MLA cache slot read, 4 DSA cache slot / pool, 5 KDA state or
// conv slot, 6 MoE expert id, 7 MoE token row, 8 DSA tail-ring owner.
// ---------------------------------------------------------------------------------------------------------------
#ifndef G53_BOUNDS
#define G53_BOUNDS 0
#endif
struct G53BoundsRec {
  int count;
  int code;
  long long index;
  long long limit;
};
#ifdef __CUDACC__
#if G53_BOUNDS
static __device__ G53BoundsRec g53_bounds_rec;
#endif
__device__ __forceinline__ bool g53_in_bounds(long long i, long long n, int code) {
#if G53_BOUNDS
  if (n <= 0 || (i >= 0 && i < n)) return true;
  if (atomicAdd(&g53_bounds_rec.count, 1) == 0) {
    g53_bounds_rec.code = code;
    g53_bounds_rec.index = i;
    g53_bounds_rec.limit = n;
  }
  return false;
#else
  (void)i; (void)n; (void)code;
  return true;
#endif
}
// an index from device data, or `sub` (an in-range substitute, or -1 = masked) when it is out of range
__device__ __forceinline__ int g53_checked(int i, long long n, int code, int sub) {
  return g53_in_bounds(i, n, code) ? i : sub;
}
#if G53_BOUNDS && !defined(__CUDA_ARCH__)
// host pass: register this source file's record (its host-side symbol, for cudaMemcpyFromSymbol) at load time
void g53_bounds_register(const void* symbol);
namespace {
struct G53BoundsRegistrar {
  G53BoundsRegistrar() { g53_bounds_register(&g53_bounds_rec); }
};
G53BoundsRegistrar g53_bounds_registrar;
}  // namespace
#endif
#endif

// Programmatic dependent launch.  A kernel launched with the programmatic-stream-serialization attribute may start
// while the previous kernel of the stream still runs: it must call pdl_wait() before it reads anything that kernel
// writes (pdl_wait returns at once when the launch has no programmatic dependency).  pdl_trigger() lets the
// dependents of the calling kernel begin launching (they still wait for its completion in their own pdl_wait).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }
__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

// Host side: programmatic dependent launches are on unless GLM53_PDL=0.
inline bool g53_pdl_on() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("GLM53_PDL");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

// Launch `k` as a programmatic dependent of the previous kernel of the stream (optionally as clusters of
// cluster_z CTAs along z).  Only for kernels that call pdl_wait() before their first global write and before
// reading anything the previous kernels write.
template <typename... KArgs, typename... Args>
inline cudaError_t g53_launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                  int cluster_z, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (cluster_z > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = cluster_z;
    ++na;
  }
  if (g53_pdl_on()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, k, static_cast<Args&&>(args)...);
}

namespace g53 {

constexpr int kWarp = 32;

__device__ __forceinline__ int warp_sum_int(int v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Sum over groups of `width` lanes (width a power of two <= 32).
template <int W>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = W / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum; `red` must hold blockDim.x/32 floats. Result broadcast to every thread.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += red[i];   // fixed order: deterministic
  return t;
}

__device__ __forceinline__ float bf2f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ __nv_bfloat16 f2bf(float x) { return __float2bfloat16_rn(x); }
__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + __expf(-x)); }
__device__ __forceinline__ float siluf_(float x) { return x / (1.f + __expf(-x)); }

// two e4m3 bytes (low byte = element 0) -> f16x2 (exact)
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t v) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
  return r;
}

// two bf16 (packed) -> f16x2 (exact for |x| in f16's normal range)
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t v) {
  float lo = __uint_as_float(v << 16);
  float hi = __uint_as_float(v & 0xffff0000u);
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t f32x2_to_f16x2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// mma.sync m16n8k16, f16 inputs, fp32 accumulate: D = A*B + D
// (no `volatile` on the pure tensor-core / read-only load asm below: the scheduler may reorder and overlap them)
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

// L2 eviction-priority policy for data read once (streamed weights): such lines are replaced first, so data
// prefetched into L2 for a later kernel survives the stream
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint32_t ldg_nc_u32_ef(const void* p, uint64_t pol) {
  uint32_t r;
  asm("ld.global.nc.L1::no_allocate.L2::cache_hint.u32 %0, [%1], %2;" : "=r"(r) : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ uint32_t ldg_nc_u32(const void* p) {
  uint32_t r;
  asm("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}

// ---- cross-GPU signalling over peer memory (system scope) ----
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_sys_add(unsigned* p, unsigned v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Wait until *p - target >= 0 (wrap-around order).  Bounded: after ~2^22 polls (about a second with the back-off)
// the wait records `code` in *err and returns false, so a peer that never arrives cannot hang the GPU.
__device__ __forceinline__ bool wait_flag_geq(const unsigned* p, unsigned target, int* err, int code) {
  for (uint32_t n = 0;; ++n) {
    if ((int)(ld_acquire_sys(p) - target) >= 0) return true;
    if (n > (1u << 22)) {
      if (err) atomicExch(err, code);
      return false;
    }
    if (n > 32) __nanosleep(128);
  }
}

// In-warp orthonormal 128-point Walsh-Hadamard transform (Sylvester order). Lane l holds elements 4l..4l+3.
__device__ __forceinline__ void fwht128_warp(float (&v)[4]) {
  const int lane = threadIdx.x & 31;
  // in-lane stages (h = 1, 2)
  float a0 = v[0] + v[1], a1 = v[0] - v[1], a2 = v[2] + v[3], a3 = v[2] - v[3];
  v[0] = a0 + a2; v[2] = a0 - a2; v[1] = a1 + a3; v[3] = a1 - a3;
  // cross-lane stages (h = 4 .. 64 -> lane bit 1 .. 16)
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    const bool upper = (lane & m) != 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float p = __shfl_xor_sync(0xffffffffu, v[i], m);
      v[i] = upper ? (p - v[i]) : (v[i] + p);
    }
  }
  const float s = 0.08838834764831845f;   // 1/sqrt(128)
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] *= s;
}

// The same transform with each cross-lane butterfly as one FFMA (bit-identical results, fewer instructions, one
// more live register per stage): for kernels with registers to spare (the prefill MoE epilogue); the decode
// kernels, capped at 64 registers, keep the predicated form above.
__device__ __forceinline__ void fwht128_warp_fma(float (&v)[4]) {
  const int lane = threadIdx.x & 31;
  // in-lane stages (h = 1, 2)
  float a0 = v[0] + v[1], a1 = v[0] - v[1], a2 = v[2] + v[3], a3 = v[2] - v[3];
  v[0] = a0 + a2; v[2] = a0 - a2; v[1] = a1 + a3; v[3] = a1 - a3;
  // cross-lane stages (h = 4 .. 64 -> lane bit 1 .. 16)
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    // lower lane: v + p, upper lane: p - v, as one FFMA p + (+-1) v (the product is exact: same single rounding)
    const float sg = (lane & m) ? -1.f : 1.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float p = __shfl_xor_sync(0xffffffffu, v[i], m);
      v[i] = fmaf(sg, v[i], p);
    }
  }
  const float s = 0.08838834764831845f;   // 1/sqrt(128)
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] *= s;
}

// exclusive scan of an int over the block (blockDim multiple of 32, <= 1024); returns (prefix, total)
__device__ __forceinline__ int2 block_scan(int v, int* wsum) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) wsum[wid] = x;
  __syncthreads();
  if (wid == 0) {
    int t = lane < nw ? wsum[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    if (lane < nw) wsum[lane] = t;   // inclusive warp-total prefix
  }
  __syncthreads();
  const int before = wid > 0 ? wsum[wid - 1] : 0;
  const int total = wsum[nw - 1];
  return make_int2(before + x - v, total);
}

}  // namespace g53
