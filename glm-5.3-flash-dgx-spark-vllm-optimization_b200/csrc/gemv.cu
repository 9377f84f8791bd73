// Small-M GEMM ("GEMV") for decode: Y[M, N] = X[M, K] @ W[N, K]^T with M <= 16 activation rows.
//
// Weight-stationary, swap-AB on tensor cores: the weight tile is the 16-row A operand of mma.m16n8k16 and the
// (at most 16) activation rows are the 8-wide B operand, so every weight byte is loaded once, by one lane, with
// 16-byte loads, and the tensor core does the multiply (CUDA-core FMA would be compute-bound at M = 8).  The
// reduction dimension is permuted inside every 64-element chunk identically for A and B (a dot product does not
// depend on the order), which lets lane (g, q) read 16 contiguous bytes of weight rows g and g+8 and 16
// contiguous activations of token g for four consecutive mma steps.
//
// Weights: fp8 e4m3 with an fp32 scale per output row (converted exactly to f16 in registers; activations bf16
// converted to f16 -- exact in f16's normal range), or bf16 (router / indexer projections, bf16 mma).
// K is split across the warps of a CTA; the partial tiles are summed in a fixed order (deterministic).
//
// Reference counterparts: code/fork/kernels/fp8_gemv.cu:96 (Marlin-layout fp8 GEMV, M <= 64) and
// code/fork/kernels/gemv_bf16.cu:83 (router / small bf16 GEMM).
#include <algorithm>
#include <cstdlib>
#include <cooperative_groups.h>
#include "common.cuh"
#include "launchers.h"

namespace cg = cooperative_groups;

namespace g53 {

template <bool FP8, int KS, int NT, int CL>
__global__ void __launch_bounds__(256) gemv_kernel(GemvArgs p) {
  constexpr int CH = FP8 ? 64 : 32;            // k elements per lane-load chunk (16 bytes of weight)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int ks = warp % KS, tile = warp / KS;
  const int b = blockIdx.y;
  const int n0 = (blockIdx.x * NT + tile) * 16;
  const int nchunk_all = p.K / CH;
  // cluster split of K: CTA z of the cluster covers chunks [c_lo, c_hi)
  const int per = (nchunk_all + CL - 1) / CL;
  const int c_lo = (CL > 1 ? (int)blockIdx.z : 0) * per;
  const int nchunk = min(nchunk_all, c_lo + per);
  const bool two = p.M > 8;

  const uint8_t* wbase = reinterpret_cast<const uint8_t*>(p.w) + (int64_t)b * p.bsw * (FP8 ? 1 : 2);
  const __nv_bfloat16* xb = p.x + (int64_t)b * p.bsx;
  const int esz = FP8 ? 1 : 2;
  const bool rA = (n0 + g) < p.N, rB = (n0 + g + 8) < p.N;
  const uint8_t* wr0 = wbase + ((int64_t)(n0 + g) * p.K) * esz;
  const uint8_t* wr1 = wbase + ((int64_t)(n0 + g + 8) * p.K) * esz;
  const bool t0 = g < p.M, t1 = (g + 8) < p.M;
  const __nv_bfloat16* x0 = xb + (int64_t)g * p.ldx;
  const __nv_bfloat16* x1 = xb + (int64_t)(g + 8) * p.ldx;

  float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
  const uint4 z4 = make_uint4(0, 0, 0, 0);

  // the weights do not depend on the previous kernel: pull this warp's chunks towards L2 before waiting for it
  for (int c = c_lo + ks; c < nchunk; c += KS) {
    const int kb = c * CH + q * (CH / 4);
    if (rA) prefetch_l2(wr0 + (int64_t)kb * esz);
    if (rB) prefetch_l2(wr1 + (int64_t)kb * esz);
  }
  pdl_trigger();
  pdl_wait();

#pragma unroll 4
  for (int c = c_lo + ks; c < nchunk; c += KS) {
    const int kb = c * CH + q * (CH / 4);
    uint4 wa = rA ? ldg_nc_v4(wr0 + (int64_t)kb * esz) : z4;
    uint4 wb = rB ? ldg_nc_v4(wr1 + (int64_t)kb * esz) : z4;
    if constexpr (FP8) {
      // 16 activations per lane (two 16-byte loads), for tokens g and g+8
      uint4 xa0 = t0 ? *reinterpret_cast<const uint4*>(x0 + kb) : z4;
      uint4 xa1 = t0 ? *reinterpret_cast<const uint4*>(x0 + kb + 8) : z4;
      uint4 xc0 = z4, xc1 = z4;
      if (two && t1) {
        xc0 = *reinterpret_cast<const uint4*>(x1 + kb);
        xc1 = *reinterpret_cast<const uint4*>(x1 + kb + 8);
      }
      const uint32_t wav[4] = {wa.x, wa.y, wa.z, wa.w};
      const uint32_t wbv[4] = {wb.x, wb.y, wb.z, wb.w};
      const uint32_t xav[8] = {xa0.x, xa0.y, xa0.z, xa0.w, xa1.x, xa1.y, xa1.z, xa1.w};
      const uint32_t xcv[8] = {xc0.x, xc0.y, xc0.z, xc0.w, xc1.x, xc1.y, xc1.z, xc1.w};
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        uint32_t a[4];
        a[0] = e4m3x2_to_f16x2((uint16_t)(wav[s] & 0xffffu));
        a[1] = e4m3x2_to_f16x2((uint16_t)(wbv[s] & 0xffffu));
        a[2] = e4m3x2_to_f16x2((uint16_t)(wav[s] >> 16));
        a[3] = e4m3x2_to_f16x2((uint16_t)(wbv[s] >> 16));
        mma_f16_16816(acc0, a, bf16x2_to_f16x2(xav[2 * s]), bf16x2_to_f16x2(xav[2 * s + 1]));
        if (two) mma_f16_16816(acc1, a, bf16x2_to_f16x2(xcv[2 * s]), bf16x2_to_f16x2(xcv[2 * s + 1]));
      }
    } else {
      uint4 xa = t0 ? *reinterpret_cast<const uint4*>(x0 + kb) : z4;
      uint4 xc = (two && t1) ? *reinterpret_cast<const uint4*>(x1 + kb) : z4;
      const uint32_t wav[4] = {wa.x, wa.y, wa.z, wa.w};
      const uint32_t wbv[4] = {wb.x, wb.y, wb.z, wb.w};
      const uint32_t xav[4] = {xa.x, xa.y, xa.z, xa.w};
      const uint32_t xcv[4] = {xc.x, xc.y, xc.z, xc.w};
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        uint32_t a[4] = {wav[2 * s], wbv[2 * s], wav[2 * s + 1], wbv[2 * s + 1]};
        mma_bf16_16816(acc0, a, xav[2 * s], xav[2 * s + 1]);
        if (two) mma_bf16_16816(acc1, a, xcv[2 * s], xcv[2 * s + 1]);
      }
    }
  }

  // cross-warp (split-K) reduction in fixed order
  __shared__ float red[KS][NT][16][17];
  __shared__ float red2[KS][NT][16][17];
  red[ks][tile][g][2 * q] = acc0[0];
  red[ks][tile][g][2 * q + 1] = acc0[1];
  red[ks][tile][g + 8][2 * q] = acc0[2];
  red[ks][tile][g + 8][2 * q + 1] = acc0[3];
  if (two) {
    red2[ks][tile][g][2 * q] = acc1[0];
    red2[ks][tile][g][2 * q + 1] = acc1[1];
    red2[ks][tile][g + 8][2 * q] = acc1[2];
    red2[ks][tile][g + 8][2 * q + 1] = acc1[3];
  }
  __syncthreads();
  // tile sums (fixed warp order) -> tot[t][row][tok]
  __shared__ float tot[NT][16][17];
  for (int e = threadIdx.x; e < NT * 16 * 16; e += blockDim.x) {
    const int t = e / 256, r = (e / 16) % 16, tok = e % 16;
    float v = 0.f;
    if (tok < p.M) {
#pragma unroll
      for (int s2 = 0; s2 < KS; ++s2) v += tok < 8 ? red[s2][t][r][tok] : red2[s2][t][r][tok - 8];
    }
    tot[t][r][tok] = v;
  }
  if constexpr (CL > 1) {
    // cluster reduction over distributed shared memory, in rank order, by rank 0
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    if (cluster.block_rank() == 0) {
      for (int e = threadIdx.x; e < NT * 16 * 16; e += blockDim.x) {
        const int t = e / 256, r = (e / 16) % 16, tok = e % 16;
        float v = tot[t][r][tok];
        for (int q2 = 1; q2 < CL; ++q2) v += cluster.map_shared_rank(&tot[0][0][0], q2)[(t * 16 + r) * 17 + tok];
        tot[t][r][tok] = v;
      }
    }
    cluster.sync();
    if (cluster.block_rank() != 0) return;
  } else {
    __syncthreads();
  }
  const float* scale = p.scale ? p.scale + (int64_t)b * p.bss : nullptr;
  if (p.mode == GEMV_SWIGLU) {
    // rows 0..7 of every 16-row tile are gate rows j0..j0+7, rows 8..15 the matching up rows
    for (int e = threadIdx.x; e < NT * 8 * 16; e += blockDim.x) {
      const int t = e / (8 * 16), r = (e / 16) % 8, tok = e % 16;
      if (tok >= p.M) continue;
      const int nt0 = (blockIdx.x * NT + t) * 16;
      if (nt0 + r + 8 >= p.N) continue;
      float gv = tot[t][r][tok], uv = tot[t][r + 8][tok];
      if (scale) { gv *= scale[nt0 + r]; uv *= scale[nt0 + r + 8]; }
      // y stored as bf16 values of g and u first (the MLP output rounding points), then the activation
      gv = round_bf16(gv);
      uv = round_bf16(uv);
      gv = fminf(gv, p.limit);
      uv = fminf(fmaxf(uv, -p.limit), p.limit);
      const float act = siluf_(gv) * uv;
      __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(p.y) + (int64_t)b * p.bsy;
      y[(int64_t)tok * p.ldy + (nt0 >> 1) + r] = f2bf(act);
    }
    return;
  }
  for (int e = threadIdx.x; e < NT * 16 * 16; e += blockDim.x) {
    const int t = e / 256, r = (e / 16) % 16, tok = e % 16;
    const int n = (blockIdx.x * NT + t) * 16 + r;
    if (tok >= p.M || n >= p.N) continue;
    float v = tot[t][r][tok];
    if (scale) v *= scale[n];
    const int64_t off = (int64_t)b * p.bsy + (int64_t)tok * p.ldy + n;
    if (p.mode == GEMV_BF16) {
      reinterpret_cast<__nv_bfloat16*>(p.y)[off] = f2bf(v);
    } else {
      float* yf = reinterpret_cast<float*>(p.y);
      if (p.mode == GEMV_F32_ACC) v += yf[off];
      yf[off] = v;
      if (p.push_ptrs) {
        // this rank's partial into its slot of every rank's receive buffer (peer stores over NVLink)
        const int64_t so = (int64_t)p.push_rank * p.push_slot + off;
        for (int j = 0; j < p.push_world; ++j) p.push_ptrs[j][so] = v;
      }
    }
  }
  if (p.push_ptrs) {
    // the last CTA to finish raises this rank's arrival flag on every rank (release after all CTAs' stores)
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();
      const unsigned total = gridDim.x * gridDim.y;
      const unsigned prev = atomicAdd(p.push_done, 1u);
      if (prev == total - 1) {
        *p.push_done = 0u;
        __threadfence_system();
        for (int j = 0; j < p.push_world; ++j) red_release_sys_add(p.push_flags[j] + p.push_rank, 1u);
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Stream-K variant for large fp8 projections (decode).  The work is the list of units (16-row tile t, 64-wide k
// chunk c) in tile-major order; warp w of the grid takes the contiguous units [U w / W, U (w+1) / W), so every
// warp streams the same number of weight bytes (no tail wave) and keeps kSD units of weight loads in flight across
// tile boundaries.  A tile covered by one warp is finished by it; a tile split between warps w_lo..w_hi gets one
// fp32 partial per warp (slot: the warp's first or last tile), and the warp that arrives last (per-tile counter)
// adds the partials in warp order -- the result does not depend on arrival order -- and resets the counter.
// ---------------------------------------------------------------------------------------------------------------
constexpr int kSD = 12;                // units of weight loads in flight per warp

__device__ __forceinline__ int64_t stream_warp_of(int64_t x, int64_t U, int64_t W) { return ((x + 1) * W - 1) / U; }

template <bool TWO>
__device__ __forceinline__ void stream_store(const GemvArgs& p, int t, const float (&a0)[4], const float (&a1)[4]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const int n0 = t * 16;
  if (p.mode == GEMV_SWIGLU) {
    // rows 0..7 of the tile are gate rows, 8..15 the matching up rows
    if (n0 + g + 8 >= p.N) return;
    const float sg = p.scale ? p.scale[n0 + g] : 1.f, su = p.scale ? p.scale[n0 + g + 8] : 1.f;
    __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(p.y);
#pragma unroll
    for (int h = 0; h < (TWO ? 2 : 1); ++h)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int tok = h * 8 + 2 * q + e;
        if (tok >= p.M) continue;
        const float* a = h ? a1 : a0;
        float gv = round_bf16(a[e] * sg), uv = round_bf16(a[2 + e] * su);
        gv = fminf(gv, p.limit);
        uv = fminf(fmaxf(uv, -p.limit), p.limit);
        y[(int64_t)tok * p.ldy + (n0 >> 1) + g] = f2bf(siluf_(gv) * uv);
      }
    return;
  }
#pragma unroll
  for (int h = 0; h < (TWO ? 2 : 1); ++h)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int n = n0 + g + (i >= 2 ? 8 : 0), tok = h * 8 + 2 * q + (i & 1);
      if (n >= p.N || tok >= p.M) continue;
      float v = (h ? a1 : a0)[i];
      if (p.scale) v *= p.scale[n];
      const int64_t off = (int64_t)tok * p.ldy + n;
      if (p.mode == GEMV_BF16) {
        reinterpret_cast<__nv_bfloat16*>(p.y)[off] = f2bf(v);
      } else {
        float* yf = reinterpret_cast<float*>(p.y);
        if (p.mode == GEMV_F32_ACC) v += yf[off];
        yf[off] = v;
      }
    }
}

// a tile this warp finished only partly: publish the partial; the last of the tile's warps adds them in warp order
template <bool TWO>
__device__ __noinline__ void stream_partial(const GemvArgs& p, float* part, int* cnt, int t, int64_t wg, int64_t W,
                                            int64_t U, int C, float a0_0, float a0_1, float a0_2, float a0_3,
                                            float a1_0, float a1_1, float a1_2, float a1_3) {
  const int lane = threadIdx.x & 31;
  const int64_t first_u = U * wg / W;
  const int side = (first_u / C == t) ? 0 : 1;
  float* mine = part + ((wg * 2 + side) * 32 + lane) * 8;
  *reinterpret_cast<float4*>(mine) = make_float4(a0_0, a0_1, a0_2, a0_3);
  *reinterpret_cast<float4*>(mine + 4) = make_float4(a1_0, a1_1, a1_2, a1_3);
  __threadfence();
  __syncwarp();
  const int64_t w_lo = stream_warp_of((int64_t)t * C, U, W), w_hi = stream_warp_of((int64_t)t * C + C - 1, U, W);
  int last = 0;
  if (lane == 0) last = atomicAdd(&cnt[t], 1) == (int)(w_hi - w_lo);
  last = __shfl_sync(0xffffffffu, last, 0);
  if (!last) return;
  __threadfence();
  float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
  for (int64_t w = w_lo; w <= w_hi; ++w) {
    const int sd = ((U * w / W) / C == t) ? 0 : 1;
    const float* src = part + ((w * 2 + sd) * 32 + lane) * 8;
    const float4 v0 = __ldcg(reinterpret_cast<const float4*>(src));
    const float4 v1 = __ldcg(reinterpret_cast<const float4*>(src + 4));
    s0[0] += v0.x; s0[1] += v0.y; s0[2] += v0.z; s0[3] += v0.w;
    s1[0] += v1.x; s1[1] += v1.y; s1[2] += v1.z; s1[3] += v1.w;
  }
  if (lane == 0) cnt[t] = 0;
  stream_store<TWO>(p, t, s0, s1);
}

template <bool TWO>
__global__ void __launch_bounds__(256, 1) gemv_stream_kernel(GemvArgs p, float* part, int* cnt) {
  const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const int64_t W = (int64_t)gridDim.x * 8, wg = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int C = p.K / 64, T = (p.N + 15) / 16;
  const int64_t U = (int64_t)T * C;
  const int64_t u0 = U * wg / W, u1 = U * (wg + 1) / W;
  if (u0 >= u1) return;
  const uint8_t* wbase = reinterpret_cast<const uint8_t*>(p.w);
  const __nv_bfloat16* x0 = p.x + (int64_t)g * p.ldx + q * 16;
  const __nv_bfloat16* x1 = p.x + (int64_t)(g + 8) * p.ldx + q * 16;
  const bool t0 = g < p.M, t1 = TWO && (g + 8) < p.M;
  const uint4 z4 = make_uint4(0u, 0u, 0u, 0u);
  // prefetch cursor (tile, chunk) and the first kSD units
  int pt = (int)(u0 / C), pc = (int)(u0 % C);
  uint4 ra[kSD], rb[kSD];
#pragma unroll
  for (int j = 0; j < kSD; ++j) {
    ra[j] = rb[j] = z4;
    if (u0 + j < u1) {
      const int r = pt * 16 + g;
      const uint8_t* src = wbase + (int64_t)r * p.K + pc * 64 + q * 16;
      if (r < p.N) ra[j] = ldg_nc_v4(src);
      if (r + 8 < p.N) rb[j] = ldg_nc_v4(src + (int64_t)8 * p.K);
      if (++pc == C) { pc = 0; ++pt; }
    }
  }
  int t = (int)(u0 / C), c = (int)(u0 % C);
  bool whole = c == 0;                       // this warp started the current tile at its first chunk
  float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
  for (int64_t base = u0; base < u1; base += kSD) {
#pragma unroll
    for (int j = 0; j < kSD; ++j) {
      const int64_t uu = base + j;
      if (uu < u1) {
        const int kb = c * 64;
        const uint4 xa0 = t0 ? *reinterpret_cast<const uint4*>(x0 + kb) : z4;
        const uint4 xa1 = t0 ? *reinterpret_cast<const uint4*>(x0 + kb + 8) : z4;
        uint4 xc0 = z4, xc1 = z4;
        if (t1) {
          xc0 = *reinterpret_cast<const uint4*>(x1 + kb);
          xc1 = *reinterpret_cast<const uint4*>(x1 + kb + 8);
        }
        const uint32_t wav[4] = {ra[j].x, ra[j].y, ra[j].z, ra[j].w};
        const uint32_t wbv[4] = {rb[j].x, rb[j].y, rb[j].z, rb[j].w};
        const uint32_t xav[8] = {xa0.x, xa0.y, xa0.z, xa0.w, xa1.x, xa1.y, xa1.z, xa1.w};
        const uint32_t xcv[8] = {xc0.x, xc0.y, xc0.z, xc0.w, xc1.x, xc1.y, xc1.z, xc1.w};
        // refill this slot with unit uu + kSD
        ra[j] = rb[j] = z4;
        if (uu + kSD < u1) {
          const int r = pt * 16 + g;
          const uint8_t* src = wbase + (int64_t)r * p.K + pc * 64 + q * 16;
          if (r < p.N) ra[j] = ldg_nc_v4(src);
          if (r + 8 < p.N) rb[j] = ldg_nc_v4(src + (int64_t)8 * p.K);
          if (++pc == C) { pc = 0; ++pt; }
        }
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          uint32_t a[4];
          a[0] = e4m3x2_to_f16x2((uint16_t)(wav[s] & 0xffffu));
          a[1] = e4m3x2_to_f16x2((uint16_t)(wbv[s] & 0xffffu));
          a[2] = e4m3x2_to_f16x2((uint16_t)(wav[s] >> 16));
          a[3] = e4m3x2_to_f16x2((uint16_t)(wbv[s] >> 16));
          mma_f16_16816(acc0, a, bf16x2_to_f16x2(xav[2 * s]), bf16x2_to_f16x2(xav[2 * s + 1]));
          if (TWO) mma_f16_16816(acc1, a, bf16x2_to_f16x2(xcv[2 * s]), bf16x2_to_f16x2(xcv[2 * s + 1]));
        }
        const bool tile_end = c == C - 1;
        if (tile_end || uu == u1 - 1) {
          if (whole && tile_end) {
            stream_store<TWO>(p, t, acc0, acc1);
          } else {
            stream_partial<TWO>(p, part, cnt, t, wg, W, U, C, acc0[0], acc0[1], acc0[2], acc0[3], acc1[0], acc1[1],
                                acc1[2], acc1[3]);
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) acc0[i] = acc1[i] = 0.f;
          whole = true;
        }
        if (++c == C) { c = 0; ++t; }
      }
    }
  }
}

// launched as a programmatic dependent of the previous kernel (weights prefetched before pdl_wait) unless
// GLM53_PDL=0
static bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("GLM53_PDL");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

template <bool FP8, int KS, int NT>
static cudaError_t launch_cfg(const GemvArgs& p, dim3 grid, int cl, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  if (cl > 1) grid.z = cl;
  cfg.gridDim = grid;
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (cl > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = cl;
    ++na;
  }
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  if (cl <= 1) return cudaLaunchKernelEx(&cfg, gemv_kernel<FP8, KS, NT, 1>, p);
  switch (cl) {
    case 2: return cudaLaunchKernelEx(&cfg, gemv_kernel<FP8, KS, NT, 2>, p);
    case 4: return cudaLaunchKernelEx(&cfg, gemv_kernel<FP8, KS, NT, 4>, p);
    default: return cudaLaunchKernelEx(&cfg, gemv_kernel<FP8, KS, NT, 8>, p);
  }
}

// stream-K launch: one CTA of 8 warps per SM, at least 8 units per warp (part holds 16 warps per SM)
static cudaError_t launch_stream(const GemvArgs& p, float* part, int* cnt, int sms, cudaStream_t st) {
  const int64_t U = (int64_t)((p.N + 15) / 16) * (p.K / 64);
  const int64_t warps = std::min<int64_t>((int64_t)sms * 8, U / 8);
  const int grid = (int)std::max<int64_t>(1, warps / 8);
  if (p.M > 8) gemv_stream_kernel<true><<<grid, 256, 0, st>>>(p, part, cnt);
  else gemv_stream_kernel<false><<<grid, 256, 0, st>>>(p, part, cnt);
  return cudaGetLastError();
}

// large fp8 projections go through the bulk-copy kernel (GLM53_BULK_GEMV=0 disables it; GLM53_BULK_GEMV_MIN sets
// the weight size in bytes from which it is used).  Measured on B200 (L2 flushed, M = 8): 1.5x on the KDA input
// projection and the lm_head shard (0.89 of measured HBM), 1.1-1.3x on the 4096-row output projections, 1.2x on
// 8 MB shapes; for 9..16 rows with K > 4096 its 2 KB stages lose to the split-K kernel, which keeps those.
static bool bulk_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("GLM53_BULK_GEMV");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}
static int64_t bulk_min_bytes() {
  static int64_t v = -1;
  if (v < 0) {
    const char* e = std::getenv("GLM53_BULK_GEMV_MIN");
    v = e ? std::atoll(e) : (int64_t)4 << 20;
  }
  return v;
}

template <bool FP8>
static cudaError_t launch_gemv_t(const GemvArgs& p, cudaStream_t st) {
  const int CH = FP8 ? 64 : 32;
  if (p.K % CH != 0 || p.M < 1 || p.M > 16) return cudaErrorInvalidValue;
  if (FP8 && g53_gemv_bulk_ok(p) &&
      (p.force_ks == -1 || (p.force_ks == 0 && p.force_cl == 0 && bulk_enabled() && (p.M <= 8 || p.K <= 4096) &&
                            (int64_t)p.N * p.K >= bulk_min_bytes())))
    return g53_gemv_bulk(p, pdl_enabled(), st);
  if (FP8 && p.stream_part && p.force_ks == 0 && p.batch == 1 && p.push_ptrs == nullptr &&
      (int64_t)((p.N + 15) / 16) * (p.K / 64) >= (int64_t)p.stream_sms * 8 * 16 &&
      (p.N + 15) / 16 <= p.stream_tiles)
    return launch_stream(p, p.stream_part, p.stream_cnt, p.stream_sms, st);
  const int nchunk = p.K / CH;
  int ks = 8;
  while (ks > 1 && nchunk < ks * 2) ks >>= 1;
  if (p.force_ks == 1 || p.force_ks == 2 || p.force_ks == 4 || p.force_ks == 8) ks = p.force_ks;
  const int tiles = (p.N + 15) / 16;
  const int nt = 8 / ks;
  dim3 grid((tiles + nt - 1) / nt, p.batch);
  // too few CTAs to cover the SMs: split K across a cluster (DSMEM reduction)
  int cl = 1;
  const int ctas = grid.x * grid.y;
  while (cl < 8 && ctas * cl < 296 && nchunk >= ks * cl * 4) cl <<= 1;
  if (p.force_cl == 1 || p.force_cl == 2 || p.force_cl == 4 || p.force_cl == 8) cl = p.force_cl;
  if (nchunk < ks * cl) return cudaErrorInvalidValue;
  switch (ks) {
    case 8: return launch_cfg<FP8, 8, 1>(p, grid, cl, st);
    case 4: return launch_cfg<FP8, 4, 2>(p, grid, cl, st);
    case 2: return launch_cfg<FP8, 2, 4>(p, grid, cl, st);
    default: return launch_cfg<FP8, 1, 8>(p, grid, cl, st);
  }
}

}  // namespace g53

cudaError_t g53_gemv_fp8(const GemvArgs& p, cudaStream_t st) { return g53::launch_gemv_t<true>(p, st); }
cudaError_t g53_gemv_bf16(const GemvArgs& p, cudaStream_t st) { return g53::launch_gemv_t<false>(p, st); }
