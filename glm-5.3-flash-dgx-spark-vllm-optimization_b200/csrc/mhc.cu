// Manifold-constrained hyper-connections (mHC) with S residual streams, embedding and norms.
//
// hc_post_pre = (optional) mHC post of the previous block fused with mHC pre of the next one:
//   partial  grid (D/256 column blocks, row groups): each thread owns one column d of every stream; with a branch
//            it first writes X_s[d] = bf16(post_s * bf16(branch[d]) + sum_j comb[j, s] X_j[d]); then it adds its
//            column's share of the n_mix mixing dots (fn rows held in registers, loaded once per CTA) and of the
//            sum of squares; per-CTA partials are reduced in a fixed warp order
//   finish   one CTA per row: partials summed in column-block order -> r = rsqrt(mean(X^2) + eps);
//            pre = sigmoid + eps, post = 2 sigmoid, comb = Sinkhorn(softmax + eps); collapsed = bf16(sum pre_s X_s);
//            normed = bf16(rmsnorm(collapsed) * w)
// Reference counterparts: code/fork/kernels/mhc_post_prenorm.cu:34 (prefill post+prenorm) and
// code/fork/kernels/smallops.cu:134 (decode mHC); math as code/fork/docs/ref/tf_glue.py:123-175.
#include <cstdlib>
#include "common.cuh"
#include "launchers.h"

namespace g53 {

constexpr int kDB = 64;      // columns per partial CTA (one per thread)
constexpr int kRB = 16;      // rows per partial CTA

template <int S>
__global__ void __launch_bounds__(kDB) hc_partial_kernel(HcArgs a) {
  pdl_trigger();                       // dependents (the next projection) may start prefetching
  constexpr int NM = 2 * S + S * S;
  const int d = blockIdx.x * kDB + threadIdx.x;
  const int NB = a.D / kDB;
  __shared__ float red[kDB][NM + 2];
  const bool pre = a.fn != nullptr;     // post only when no mixing weights are given
  float fnv[NM][S];
#pragma unroll
  for (int i = 0; i < NM; ++i)
#pragma unroll
    for (int s = 0; s < S; ++s) fnv[i][s] = pre ? bf2f(a.fn[(int64_t)i * S * a.D + s * a.D + d]) : 0.f;
  const int rb = (a.R + gridDim.y - 1) / gridDim.y;   // rows per CTA (1 for decode-sized launches)
  const int r0 = blockIdx.y * rb;
  if (a.gath) {
    // tensor-parallel partials pushed by every rank's producer: wait for all arrival flags of this parity
    if (threadIdx.x == 0) {
      const unsigned target = *reinterpret_cast<volatile unsigned*>(a.epoch) + 1u;
      for (int j = 0; j < a.world; ++j) wait_flag_geq(a.flags + j, target, a.err, 21);
    }
    __syncthreads();
  }
  for (int r = r0; r < min(r0 + rb, a.R); ++r) {
    __nv_bfloat16* xr = a.X + (int64_t)r * S * a.D;
    float x[S];
#pragma unroll
    for (int s = 0; s < S; ++s) x[s] = bf2f(xr[s * a.D + d]);
    if (a.branch || a.gath) {
      float bsum;
      if (a.gath) {
        bsum = 0.f;
        for (int j = 0; j < a.world; ++j) bsum += a.gath[(int64_t)j * a.gath_slot + (int64_t)r * a.D + d];
      } else {
        bsum = a.branch[(int64_t)r * a.D + d];
      }
      const float b = round_bf16(bsum);
      float nx[S];
#pragma unroll
      for (int s = 0; s < S; ++s) {
        float m = 0.f;
#pragma unroll
        for (int j = 0; j < S; ++j) m += a.comb[(r * S + j) * S + s] * x[j];
        nx[s] = round_bf16(a.post[r * S + s] * b + m);
      }
#pragma unroll
      for (int s = 0; s < S; ++s) { x[s] = nx[s]; xr[s * a.D + d] = f2bf(nx[s]); }
    }
    if (!pre) continue;
#pragma unroll
    for (int i = 0; i < NM; ++i) {
      float t = 0.f;
#pragma unroll
      for (int s = 0; s < S; ++s) t += fnv[i][s] * x[s];
      red[threadIdx.x][i] = t;
    }
    float ss = 0.f;
#pragma unroll
    for (int s = 0; s < S; ++s) ss += x[s] * x[s];
    red[threadIdx.x][NM] = ss;
    __syncthreads();
    {
      // 2 threads per output (columns c = h, h + 2, ...), 4 interleaved accumulators: fixed order, short chains
      const int i = threadIdx.x >> 1, h = threadIdx.x & 1;
      float t0 = 0.f, t1 = 0.f, t2 = 0.f, t3 = 0.f;
      if (i <= NM) {
#pragma unroll
        for (int c = h; c < kDB; c += 8) {
          t0 += red[c][i];
          t1 += red[c + 2][i];
          t2 += red[c + 4][i];
          t3 += red[c + 6][i];
        }
      }
      float t = (t0 + t1) + (t2 + t3);
      t += __shfl_xor_sync(0xffffffffu, t, 1);
      if (i <= NM && h == 0) a.part[((int64_t)r * NB + blockIdx.x) * 32 + i] = t;
    }
    __syncthreads();
  }
  if (a.gath) {
    // the last CTA marks this parity's receive buffer consumed (every CTA read the epoch before counting in)
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      const unsigned prev = atomicAdd(a.done, 1u);
      if (prev == gridDim.x * gridDim.y - 1) {
        *a.done = 0u;
        __threadfence();
        atomicAdd(a.epoch, 1u);
      }
    }
  }
}

// Sinkhorn on one warp: lane l < S*S holds comb[l / S][l % S]; rows reduce over the low log2(S) lane bits,
// columns over the next log2(S) bits
template <int S>
__device__ __forceinline__ float warp_row_sum(float v) {
#pragma unroll
  for (int o = 1; o < S; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
template <int S>
__device__ __forceinline__ float warp_row_max(float v) {
#pragma unroll
  for (int o = 1; o < S; o <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
template <int S>
__device__ __forceinline__ float warp_col_sum(float v) {
#pragma unroll
  for (int o = S; o < S * S; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int S>
__global__ void __launch_bounds__(512) hc_finish_kernel(HcArgs a) {
  pdl_trigger();                       // dependents (the next projection) may start prefetching
  constexpr int NM = 2 * S + S * S;
  const int r = blockIdx.x;
  const int NB = a.nb;
  __shared__ float mix[32];
  __shared__ float pre_s[S], post_s[S], comb_s[S * S];
  __shared__ float red[32];
  // partial sums over the column blocks: warp w reads blocks w, w + nw, ... (coalesced 32-wide rows), then the
  // per-warp sums are added in warp order (fixed order throughout)
  {
    __shared__ float wpart[16][33];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = min((int)(blockDim.x >> 5), 16);
    if (w < nw) {
      float t = 0.f;
      for (int b = w; b < NB; b += nw) t += a.part[((int64_t)r * NB + b) * 32 + lane];
      wpart[w][lane] = t;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      float t = 0.f;
      for (int j = 0; j < nw; ++j) t += wpart[j][threadIdx.x];
      mix[threadIdx.x] = t;
    }
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const float rinv = rsqrtf(mix[NM] / (float)(S * a.D) + a.eps);
    if (lane < S) {
      pre_s[lane] = sigmoidf_(mix[lane] * rinv * a.hscale[0] + a.base[lane]) + a.hc_eps;
      post_s[lane] = 2.f * sigmoidf_(mix[S + lane] * rinv * a.hscale[1] + a.base[S + lane]);
    }
    const int li = lane < S * S ? lane : 0;
    float c = mix[2 * S + li] * rinv * a.hscale[2] + a.base[2 * S + li];
    const float mx = warp_row_max<S>(c);
    c = __expf(c - mx);
    c = c / warp_row_sum<S>(c) + a.hc_eps;
    for (int it = 0; it < a.iters; ++it) {
      if (it > 0) c = c / (warp_row_sum<S>(c) + a.hc_eps);
      c = c / (warp_col_sum<S>(c) + a.hc_eps);
    }
    if (lane < S * S) comb_s[lane] = c;
  }
  __syncthreads();
  if (threadIdx.x < S) a.post_out[r * S + threadIdx.x] = post_s[threadIdx.x];
  if (threadIdx.x < S * S) a.comb_out[r * S * S + threadIdx.x] = comb_s[threadIdx.x];
  const __nv_bfloat16* xr = a.X + (int64_t)r * S * a.D;
  // 8 consecutive columns per thread and pass (16-byte loads of every stream issued together); D <= 8192
  constexpr int kPass = 2;
  float col[kPass][8];
  float ss = 0.f;
#pragma unroll
  for (int ps = 0; ps < kPass; ++ps) {
    const int d0 = (ps * blockDim.x + threadIdx.x) * 8;
    if (d0 >= a.D) continue;
    uint4 xs[S];
#pragma unroll
    for (int s = 0; s < S; ++s) xs[s] = *reinterpret_cast<const uint4*>(xr + (int64_t)s * a.D + d0);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float t = 0.f;
#pragma unroll
      for (int s = 0; s < S; ++s) t += pre_s[s] * bf2f(reinterpret_cast<const __nv_bfloat16*>(&xs[s])[e]);
      t = round_bf16(t);
      col[ps][e] = t;
      ss += t * t;
    }
  }
  ss = block_sum(ss, red);
  const float rinv = rsqrtf(ss / (float)a.D + a.eps);
#pragma unroll
  for (int ps = 0; ps < kPass; ++ps) {
    const int d0 = (ps * blockDim.x + threadIdx.x) * 8;
    if (d0 >= a.D) continue;
    const uint4 wv = *reinterpret_cast<const uint4*>(a.norm_w + d0);
    const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wv);
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      __nv_bfloat162 b2 = __floats2bfloat162_rn(col[ps][2 * e] * rinv * bf2f(wb[2 * e]),
                                                col[ps][2 * e + 1] * rinv * bf2f(wb[2 * e + 1]));
      o[e] = *reinterpret_cast<uint32_t*>(&b2);
    }
    *reinterpret_cast<uint4*>(a.normed + (int64_t)r * a.D + d0) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__global__ void embed_kernel(const int* ids, const __nv_bfloat16* table, int V, int D, int S, __nv_bfloat16* X) {
  const int r = blockIdx.y;
  const int d = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (d >= D) return;
  const int id = ids[r];
  if (!g53_in_bounds(id, V, 1)) return;
  const uint4 v = *reinterpret_cast<const uint4*>(table + (int64_t)id * D + d);
  for (int s = 0; s < S; ++s) *reinterpret_cast<uint4*>(X + ((int64_t)r * S + s) * D + d) = v;
}

__global__ void __launch_bounds__(512) stream_mean_norm_kernel(const __nv_bfloat16* X, int S, int D,
                                                               const __nv_bfloat16* w, float eps,
                                                               __nv_bfloat16* hidden, __nv_bfloat16* normed) {
  const int r = blockIdx.x;
  __shared__ float red[32];
  float col[16];
  float ss = 0.f;
  int n = 0;
  for (int d = threadIdx.x; d < D; d += blockDim.x, ++n) {
    float t = 0.f;
    for (int s = 0; s < S; ++s) t += bf2f(X[((int64_t)r * S + s) * D + d]);
    t = round_bf16(t / (float)S);
    if (hidden) hidden[(int64_t)r * D + d] = f2bf(t);
    col[n] = t;
    ss += t * t;
  }
  ss = block_sum(ss, red);
  const float rinv = rsqrtf(ss / (float)D + eps);
  n = 0;
  for (int d = threadIdx.x; d < D; d += blockDim.x, ++n) normed[(int64_t)r * D + d] = f2bf(col[n] * rinv * bf2f(w[d]));
}

__global__ void __launch_bounds__(256) rmsnorm_kernel(const __nv_bfloat16* x, int64_t ldx, const __nv_bfloat16* w,
                                                      int D, float eps, __nv_bfloat16* y, int64_t ldy) {
  const int r = blockIdx.x;
  __shared__ float red[32];
  float col[32];
  float ss = 0.f;
  int n = 0;
  for (int d = threadIdx.x; d < D; d += blockDim.x, ++n) {
    const float t = bf2f(x[(int64_t)r * ldx + d]);
    col[n] = t;
    ss += t * t;
  }
  ss = block_sum(ss, red);
  const float rinv = rsqrtf(ss / (float)D + eps);
  n = 0;
  for (int d = threadIdx.x; d < D; d += blockDim.x, ++n) y[(int64_t)r * ldy + d] = f2bf(col[n] * rinv * bf2f(w[d]));
}

}  // namespace g53

using namespace g53;

// decode windows take the one-kernel cluster form (mhc_decode.cu) unless GLM53_HC_FUSED=0
static bool hc_fused_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("GLM53_HC_FUSED");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

cudaError_t g53_hc_post_pre(const HcArgs& args, cudaStream_t st) {
  HcArgs a = args;
  if (a.D % kDB || a.D > 8192 || a.D % 8 || (a.S != 2 && a.S != 4)) return cudaErrorInvalidValue;
  if (hc_fused_enabled() && g53_hc_decode_ok(a)) return g53_hc_decode(a, st);
  // prefill-sized launches: post + mixing dots on the tensor cores (column blocks of 512), then the same finish
  if (a.use_tc && a.R >= 256 && a.S == 4 && a.fn && !a.gath && a.D % 512 == 0) {
    a.nb = a.D / 512;
    cudaError_t e = g53_hc_partial_tc(a, st);
    if (e != cudaSuccess) return e;
    hc_finish_kernel<4><<<a.R, 512, 0, st>>>(a);
    G53_CHECK_LAUNCH();
    return cudaSuccess;
  }
  a.nb = a.D / kDB;
  // decode-sized launches: one row per CTA (more CTAs in flight); prefill: kRB rows per CTA (fn reuse)
  dim3 g1(a.D / kDB, a.R <= kRB ? a.R : (a.R + kRB - 1) / kRB);
  if (a.S == 4) {
    hc_partial_kernel<4><<<g1, kDB, 0, st>>>(a);
    G53_CHECK_LAUNCH();
    if (a.fn) hc_finish_kernel<4><<<a.R, 512, 0, st>>>(a);
  } else {
    hc_partial_kernel<2><<<g1, kDB, 0, st>>>(a);
    G53_CHECK_LAUNCH();
    if (a.fn) hc_finish_kernel<2><<<a.R, 512, 0, st>>>(a);
  }
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}

cudaError_t g53_embed(const int* ids, const __nv_bfloat16* table, int V, int R, int D, int S, __nv_bfloat16* X,
                      cudaStream_t st) {
  if (D % 8) return cudaErrorInvalidValue;
  dim3 grid((D / 8 + 127) / 128, R);
  embed_kernel<<<grid, 128, 0, st>>>(ids, table, V, D, S, X);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}

cudaError_t g53_stream_mean_norm(const __nv_bfloat16* X, int R, int S, int D, const __nv_bfloat16* w, float eps,
                                 __nv_bfloat16* hidden, __nv_bfloat16* normed, cudaStream_t st) {
  if (D > 8192) return cudaErrorInvalidValue;
  stream_mean_norm_kernel<<<R, 512, 0, st>>>(X, S, D, w, eps, hidden, normed);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}

cudaError_t g53_rmsnorm(const __nv_bfloat16* x, int64_t ldx, const __nv_bfloat16* w, int R, int D, float eps,
                        __nv_bfloat16* y, int64_t ldy, cudaStream_t st) {
  if (D > 8192) return cudaErrorInvalidValue;
  rmsnorm_kernel<<<R, 256, 0, st>>>(x, ldx, w, D, eps, y, ldy);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}

// ---------------------------------------------------------------------------------------------------------------
// drafter helpers: RMSNorm of an fp32 residual row (bf16 out), and causal attention inside a block of <= 16 rows
// ---------------------------------------------------------------------------------------------------------------
namespace g53 {

__global__ void __launch_bounds__(256) rmsnorm_f32_kernel(const float* x, const __nv_bfloat16* w, int D, float eps,
                                                          __nv_bfloat16* y) {
  const int r = blockIdx.x;
  __shared__ float red[32];
  float ss = 0.f;
  for (int d = threadIdx.x; d < D; d += blockDim.x) { const float t = x[(int64_t)r * D + d]; ss += t * t; }
  ss = block_sum(ss, red);
  const float rinv = rsqrtf(ss / (float)D + eps);
  for (int d = threadIdx.x; d < D; d += blockDim.x)
    y[(int64_t)r * D + d] = f2bf(x[(int64_t)r * D + d] * rinv * bf2f(w[d]));
}

// qkv [R, 3, H, Dh] bf16 -> o [R, H, Dh] bf16; row i attends to rows 0..i of its block (blocks of `block` rows)
__global__ void block_attn_kernel(const __nv_bfloat16* qkv, int R, int H, int Dh, int block, float scale,
                                  __nv_bfloat16* o) {
  const int h = blockIdx.x, r = blockIdx.y;
  const int lane = threadIdx.x;      // one warp
  const int b0 = (r / block) * block;
  const int64_t rs = (int64_t)3 * H * Dh;
  float s[16];
  float mx = -INFINITY;
  for (int j = b0; j <= r; ++j) {
    float d = 0.f;
    for (int c = lane; c < Dh; c += 32)
      d += bf2f(qkv[r * rs + h * Dh + c]) * bf2f(qkv[j * rs + H * Dh + h * Dh + c]);
    d = warp_sum(d) * scale;
    s[j - b0] = d;
    mx = fmaxf(mx, d);
  }
  float den = 0.f;
  for (int j = b0; j <= r; ++j) { s[j - b0] = __expf(s[j - b0] - mx); den += s[j - b0]; }
  for (int c = lane; c < Dh; c += 32) {
    float acc = 0.f;
    for (int j = b0; j <= r; ++j) acc += s[j - b0] * bf2f(qkv[j * rs + 2 * H * Dh + h * Dh + c]);
    o[((int64_t)r * H + h) * Dh + c] = f2bf(acc / den);
  }
}

}  // namespace g53

cudaError_t g53_rmsnorm_f32(const float* x, const __nv_bfloat16* w, int R, int D, float eps, __nv_bfloat16* y,
                            cudaStream_t st) {
  g53::rmsnorm_f32_kernel<<<R, 256, 0, st>>>(x, w, D, eps, y);
  return cudaGetLastError();
}

cudaError_t g53_block_attn(const __nv_bfloat16* qkv, int R, int H, int Dh, int block, float scale, __nv_bfloat16* o,
                           cudaStream_t st) {
  if (block > 16 || block < 1) return cudaErrorInvalidValue;
  dim3 grid(H, R);
  g53::block_attn_kernel<<<grid, 32, 0, st>>>(qkv, R, H, Dh, block, scale, o);
  return cudaGetLastError();
}
