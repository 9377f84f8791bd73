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
  // consecutive threads store consecutive output columns of one row (coalesced; for the tensor-parallel push these
  // are peer stores over NVLink, where scattered 4-byte stores cost a transaction each)
  for (int e = threadIdx.x; e < NT * 16 * 16; e += blockDim.x) {
    const int t = e / 256, r = e % 16, tok = (e / 16) % 16;
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
      const int t = e / (8 * 16), r = e % 8, tok = (e / 8) % 16;     // consecutive threads: consecutive columns
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
