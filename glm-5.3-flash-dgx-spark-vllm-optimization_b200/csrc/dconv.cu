// Grouped dynamic convolution of the block drafter (the DFlash2 drafter's grouped conv; the reference replaces its
// ten eager bf16 elementwise ops with one kernel, code/fork/kernels/smallops.cu:6-7, and documents the op chain in
// code/fork/docs/DEC_SMALLOPS.md:24-27).
//
// For row t of a draft block (position p = t mod block_size in the block) and channel c:
//   c_k  = bf16(base[k][c] + delta[t][k][c / gs])                  the per-row kernel, one delta per channel group
//   o    = bf16(c_0 * x[t][c])
//   o    = bf16(o + bf16(bf16(c_k * x[t - k][c]) * (p >= k)))      k = 1 .. taps-1, x[t - k] = 0 before the first row
// Every step is rounded to bf16 where the eager op chain rounds, so the result equals that chain bit for bit.
// One thread per (row, two adjacent channels), bf16x2 loads.
#include "common.cuh"
#include "launchers.h"

namespace g53 {

__device__ __forceinline__ float rb(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__global__ void __launch_bounds__(128) dconv_kernel(DconvArgs a) {
  const int t = blockIdx.y;
  const int c = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (c >= a.H) return;
  const int p = t % a.block_size;
  const __nv_bfloat16* xt = a.x + (int64_t)t * a.ldx;
  const __nv_bfloat16* dt = a.delta + (int64_t)t * a.taps * a.G;
  const __nv_bfloat162 x2 = *reinterpret_cast<const __nv_bfloat162*>(xt + c);
  const __nv_bfloat162 b2 = *reinterpret_cast<const __nv_bfloat162*>(a.base + c);
  float o[2];
  const float xs0[2] = {__low2float(x2), __high2float(x2)};
  const float bs0[2] = {__low2float(b2), __high2float(b2)};
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const float ck = rb(bs0[e] + bf2f(dt[(c + e) / a.gs]));
    o[e] = rb(ck * xs0[e]);
  }
  for (int k = 1; k < a.taps; ++k) {
    float xk[2] = {0.f, 0.f};
    if (t >= k) {
      const __nv_bfloat162 s2 = *reinterpret_cast<const __nv_bfloat162*>(a.x + (int64_t)(t - k) * a.ldx + c);
      xk[0] = __low2float(s2);
      xk[1] = __high2float(s2);
    }
    const __nv_bfloat162 bk = *reinterpret_cast<const __nv_bfloat162*>(a.base + (int64_t)k * a.H + c);
    const float bks[2] = {__low2float(bk), __high2float(bk)};
    const float m = p >= k ? 1.f : 0.f;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float ck = rb(bks[e] + bf2f(dt[(int64_t)k * a.G + (c + e) / a.gs]));
      const float pr = rb(rb(ck * xk[e]) * m);
      o[e] = rb(o[e] + pr);
    }
  }
  *reinterpret_cast<__nv_bfloat162*>(a.out + (int64_t)t * a.H + c) = __floats2bfloat162_rn(o[0], o[1]);
}

}  // namespace g53

cudaError_t g53_dconv(const DconvArgs& a, cudaStream_t st) {
  if (a.H % 2 || a.gs < 1 || a.H % a.gs || a.taps < 1 || a.block_size < 1 || a.T < 1) return cudaErrorInvalidValue;
  dim3 grid((a.H / 2 + 127) / 128, a.T);
  g53::dconv_kernel<<<grid, 128, 0, st>>>(a);
  return cudaGetLastError();
}
