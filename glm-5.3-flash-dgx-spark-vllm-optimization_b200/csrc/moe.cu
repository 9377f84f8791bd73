// Routed MoE for decode-sized batches: router top-k + grouping, and the EXL3 grouped expert GEMMs.
//
// EXL3 path (the trellis format is described in ops/exl3.py):
//   rot_in    xh[p] = f16(H128(x[token(p)] * suh[expert(p)]))                 (gate and up, per sorted pair)
//   gate_up   per (expert group, 128-column block): Z = xh @ W_q on tensor cores, the trellis decoded in
//             registers straight into mma.m16n8k16 B fragments (each lane decodes the 8 values of its fragment
//             from its own 32-bit word and its left neighbour's); epilogue in shared memory: H128 of the gate and
//             up rows, * svh, SwiGLU with clamp, * suh of the down projection, H128 -> f16 down input
//   down      same GEMM over the local expert width; epilogue H128, * svh, * routing weight -> fp32 per pair
//   combine   out[r] = sum over slots (fixed order) of the pair outputs
// One CTA owns one full 128-column Hadamard block of one expert, so both output rotations stay on chip.
// Reference counterparts: code/fork/kernels/exl3.cu:110 (grouped_kernel), :322 (rot_in), :371/:455 (epilogues),
// :529/:582 (route_prep / route_ids).
#include "common.cuh"
#include "launchers.h"

namespace g53 {

// ---------------------------------------------------------------------------------------------------------------
// trellis decode: lane l of a warp, 32-bit words of one 16x16 tile; returns the four f16x2 B-fragment registers
// (n-half 0: b0, b1; n-half 1: b2, b3).  Value j of lane l is the 16-bit state ending at stream bit 32l+4j+4.
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t mcg_x(uint32_t s) {
  uint32_t x = s * 0xCBAC1FEDu;
  return (x & 0x8FFF8FFFu) ^ 0x3B603B60u;
}

__device__ __forceinline__ uint32_t mcg_pair(uint32_t s0, uint32_t s1) {
  const uint32_t x0 = mcg_x(s0), x1 = mcg_x(s1);
  const uint32_t lo = __byte_perm(x0, x1, 0x5410);   // (x0.lo, x1.lo)
  const uint32_t hi = __byte_perm(x0, x1, 0x7632);   // (x0.hi, x1.hi)
  __half2 r = __hadd2(*reinterpret_cast<const __half2*>(&lo), *reinterpret_cast<const __half2*>(&hi));
  return *reinterpret_cast<uint32_t*>(&r);
}

__device__ __forceinline__ void trellis_frags(uint32_t cur, uint32_t prev, uint32_t (&b)[4]) {
  const uint32_t s0 = __funnelshift_r(cur, prev, 28) & 0xffffu;
  const uint32_t s1 = __funnelshift_r(cur, prev, 24) & 0xffffu;
  const uint32_t s2 = __funnelshift_r(cur, prev, 20) & 0xffffu;
  const uint32_t s3 = cur >> 16;
  const uint32_t s4 = (cur >> 12) & 0xffffu;
  const uint32_t s5 = (cur >> 8) & 0xffffu;
  const uint32_t s6 = (cur >> 4) & 0xffffu;
  const uint32_t s7 = cur & 0xffffu;
  b[0] = mcg_pair(s0, s1);
  b[1] = mcg_pair(s2, s3);
  b[2] = mcg_pair(s4, s5);
  b[3] = mcg_pair(s6, s7);
}

// ---------------------------------------------------------------------------------------------------------------
// routing: sigmoid scores, top-k of score + bias (ties -> lower id), normalised weights; then grouping of the
// R*top_k (row, slot) pairs by expert (ascending id; within an expert, ascending pair index).  One CTA.
// ---------------------------------------------------------------------------------------------------------------
constexpr int kMaxE = 512;
constexpr int kMaxPairs = 2048;

__global__ void __launch_bounds__(1024) moe_route_kernel(RouteArgs a) {
  __shared__ int cnt[kMaxE];
  __shared__ int start[kMaxE + 1];
  __shared__ int pe[kMaxPairs];
  __shared__ float red[32];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nw = blockDim.x >> 5;
  const int P = a.R * a.top_k;
  for (int e = tid; e < a.E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  // top-k per row: one warp per row; lane l holds candidates e = l + 32 i in registers
  constexpr int kPerLane = kMaxE / 32;
  for (int r = wid; r < a.R; r += nw) {
    const float* lg = a.logits + (int64_t)r * a.E;
    float cv[kPerLane];
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
      const int e = lane + 32 * i;
      cv[i] = e < a.E ? sigmoidf_(lg[e]) + a.bias[e] : -INFINITY;
    }
    float sel_sum = 0.f;
    int pick_l = 0;
    float wt_l = 0.f;
    for (int k = 0; k < a.top_k; ++k) {
      float best = -INFINITY;
      int bid = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < kPerLane; ++i) {
        const int e = lane + 32 * i;
        if (cv[i] > best) { best = cv[i]; bid = e; }      // ascending e within a lane: first max = lowest id
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bid, o);
        if (ob > best || (ob == best && oi < bid)) { best = ob; bid = oi; }
      }
      if ((bid & 31) == lane) {
#pragma unroll
        for (int i = 0; i < kPerLane; ++i)
          if (lane + 32 * i == bid) cv[i] = -INFINITY;
      }
      const float w = sigmoidf_(lg[bid]);
      sel_sum += w;
      if (lane == k) { pick_l = bid; wt_l = w; }
    }
    const float inv = a.norm ? 1.f / (sel_sum + 1e-20f) : 1.f;
    if (lane < a.top_k) {
      a.topk_ids[r * a.top_k + lane] = pick_l;
      a.topk_w[r * a.top_k + lane] = wt_l * inv * a.scale;
      pe[r * a.top_k + lane] = pick_l;
      atomicAdd(&cnt[pick_l], 1);
    }
  }
  __syncthreads();
  // exclusive scan of counts (serial per warp chunk; E <= 1024)
  if (tid == 0) {
    int s = 0, u = 0;
    for (int e = 0; e < a.E; ++e) {
      start[e] = s;
      if (cnt[e] > 0) {
        if (u < a.max_groups) { a.group_expert[u] = e; a.group_offset[u] = s; }
        ++u;
      }
      s += cnt[e];
    }
    start[a.E] = s;
    a.group_count[0] = u;
    for (int v = u; v <= a.max_groups; ++v) a.group_offset[v] = s;
  }
  __syncthreads();
  (void)red;
  // stable placement: rank of pair i among earlier pairs of the same expert
  for (int i = tid; i < P; i += blockDim.x) {
    const int e = pe[i];
    int rank = 0;
    for (int j = 0; j < i; ++j) rank += (pe[j] == e);
    const int pos = start[e] + rank;
    a.pair_of[i] = pos;
    a.pair_token[pos] = i / a.top_k;
    a.pair_expert[pos] = e;
    a.pair_w[pos] = a.topk_w[i];
  }
}

// ---------------------------------------------------------------------------------------------------------------
// rot_in: one warp per (sorted pair, 128-block); gate and up rotated inputs in f16
// ---------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(128) exl3_rot_in_kernel(Exl3Args a) {
  const int lane = threadIdx.x & 31;
  const int blk = blockIdx.y * 4 + (threadIdx.x >> 5);
  const int p = blockIdx.x;                      // pairs on grid.x (prefill chunks exceed 65535 pairs)
  if (blk * 128 >= a.K) return;
  const int r = a.pair_token[p], e = a.pair_expert[p];
  const int c0 = blk * 128 + lane * 4;
  const __nv_bfloat16* xr = a.x + (int64_t)r * a.ldx + c0;
  float xv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) xv[i] = bf2f(xr[i]);
  float g[4], u[4];
  const __half* sg = a.suh_g + (int64_t)e * a.K + c0;
  const __half* su = a.suh_u + (int64_t)e * a.K + c0;
#pragma unroll
  for (int i = 0; i < 4; ++i) { g[i] = xv[i] * __half2float(sg[i]); u[i] = xv[i] * __half2float(su[i]); }
  fwht128_warp(g);
  fwht128_warp(u);
  __half2* og = reinterpret_cast<__half2*>(a.xh_g + (int64_t)p * a.K + c0);
  __half2* ou = reinterpret_cast<__half2*>(a.xh_u + (int64_t)p * a.K + c0);
  og[0] = __floats2half2_rn(g[0], g[1]); og[1] = __floats2half2_rn(g[2], g[3]);
  ou[0] = __floats2half2_rn(u[0], u[1]); ou[1] = __floats2half2_rn(u[2], u[3]);
}

// A fragment (16 rows x 16 k, f16) of rotated inputs rows [row0, row0+16) at k-tile kt; rows >= nrows are zero
__device__ __forceinline__ void load_a_frag(const __half* xh, int64_t ld, int row0, int nrows, int kt,
                                            uint32_t (&a)[4]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const int k = kt * 16 + 2 * q;
  if (g < nrows) {
    const __half* r = xh + (int64_t)(row0 + g) * ld + k;
    a[0] = *reinterpret_cast<const uint32_t*>(r);
    a[2] = *reinterpret_cast<const uint32_t*>(r + 8);
  } else {
    a[0] = a[2] = 0u;
  }
  if (g + 8 < nrows) {
    const __half* r = xh + (int64_t)(row0 + g + 8) * ld + k;
    a[1] = *reinterpret_cast<const uint32_t*>(r);
    a[3] = *reinterpret_cast<const uint32_t*>(r + 8);
  } else {
    a[1] = a[3] = 0u;
  }
}

// ---------------------------------------------------------------------------------------------------------------
// gate + up: grid (N/128 column blocks, max_groups), 8 warps; warp w owns n-tile (block*8 + w)
// ---------------------------------------------------------------------------------------------------------------
constexpr int kPf = 4;   // k-tiles of trellis words prefetched per warp

__global__ void __launch_bounds__(256) exl3_gate_up_kernel(Exl3Args a) {
  const int u = blockIdx.y;
  if (u >= a.group_count[0] || u >= a.max_groups) return;
  __shared__ float zg[16][132];
  __shared__ float zu[16][132];
  const int e = a.group_expert[u];
  const int p0 = a.group_offset[u];
  const int np = a.group_offset[u + 1] - p0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const int nb = blockIdx.x;
  const int nt = nb * 8 + warp;
  const int KT = a.K / 16, NT = a.N / 16;
  const uint32_t* wg = reinterpret_cast<const uint32_t*>(a.tr_g) + ((int64_t)e * KT * NT + nt) * 32 + lane;
  const uint32_t* wu = reinterpret_cast<const uint32_t*>(a.tr_u) + ((int64_t)e * KT * NT + nt) * 32 + lane;
  const int64_t kstride = (int64_t)NT * 32;
  const int src = (lane + 31) & 31;

  for (int m0 = 0; m0 < np; m0 += 16) {
    const int nrows = min(16, np - m0);
    float ag[2][4] = {}, au[2][4] = {};
    uint32_t pg[kPf], pu[kPf];
#pragma unroll
    for (int i = 0; i < kPf; ++i) {
      pg[i] = i < KT ? ldg_nc_u32(wg + i * kstride) : 0u;
      pu[i] = i < KT ? ldg_nc_u32(wu + i * kstride) : 0u;
    }
    for (int kt0 = 0; kt0 < KT; kt0 += kPf) {
#pragma unroll
      for (int i = 0; i < kPf; ++i) {
        const int kt = kt0 + i;
        if (kt >= KT) break;
        const uint32_t cg = pg[i], cu = pu[i];
        const int nk = kt + kPf;
        pg[i] = nk < KT ? ldg_nc_u32(wg + nk * kstride) : 0u;
        pu[i] = nk < KT ? ldg_nc_u32(wu + nk * kstride) : 0u;
        uint32_t bg[4], bu[4], ax[4];
        trellis_frags(cg, __shfl_sync(0xffffffffu, cg, src), bg);
        trellis_frags(cu, __shfl_sync(0xffffffffu, cu, src), bu);
        load_a_frag(a.xh_g, a.K, p0 + m0, nrows, kt, ax);
        mma_f16_16816(ag[0], ax, bg[0], bg[1]);
        mma_f16_16816(ag[1], ax, bg[2], bg[3]);
        load_a_frag(a.xh_u, a.K, p0 + m0, nrows, kt, ax);
        mma_f16_16816(au[0], ax, bu[0], bu[1]);
        mma_f16_16816(au[1], ax, bu[2], bu[3]);
      }
    }
    // accumulators -> shared (row = pair, col = n within the 128-block)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c = warp * 16 + h * 8 + 2 * q;
      zg[g][c] = ag[h][0]; zg[g][c + 1] = ag[h][1]; zg[g + 8][c] = ag[h][2]; zg[g + 8][c + 1] = ag[h][3];
      zu[g][c] = au[h][0]; zu[g][c + 1] = au[h][1]; zu[g + 8][c] = au[h][2]; zu[g + 8][c + 1] = au[h][3];
    }
    __syncthreads();
    for (int r = warp; r < nrows; r += 8) {
      float vg[4], vu[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) { vg[i] = zg[r][lane * 4 + i]; vu[i] = zu[r][lane * 4 + i]; }
      fwht128_warp(vg);
      fwht128_warp(vu);
      const int col = nb * 128 + lane * 4;
      float act[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float gv = vg[i] * __half2float(a.svh_g[(int64_t)e * a.N + col + i]);
        float uv = vu[i] * __half2float(a.svh_u[(int64_t)e * a.N + col + i]);
        gv = fminf(gv, a.limit);
        uv = fminf(fmaxf(uv, -a.limit), a.limit);
        act[i] = siluf_(gv) * uv * __half2float(a.suh_d[(int64_t)e * a.N + col + i]);
      }
      fwht128_warp(act);
      __half2* o = reinterpret_cast<__half2*>(a.xd + (int64_t)(p0 + m0 + r) * a.N + col);
      o[0] = __floats2half2_rn(act[0], act[1]);
      o[1] = __floats2half2_rn(act[2], act[3]);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------------------------------------------
// down: grid (Dout/128, max_groups); epilogue H128, * svh, * routing weight -> yd[pair] fp32
// ---------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) exl3_down_kernel(Exl3Args a) {
  const int u = blockIdx.y;
  if (u >= a.group_count[0] || u >= a.max_groups) return;
  __shared__ float zd[16][132];
  const int e = a.group_expert[u];
  const int p0 = a.group_offset[u];
  const int np = a.group_offset[u + 1] - p0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const int nb = blockIdx.x;
  const int nt = nb * 8 + warp;
  const int KT = a.N / 16, NT = a.Dout / 16;
  const uint32_t* wd = reinterpret_cast<const uint32_t*>(a.tr_d) + ((int64_t)e * KT * NT + nt) * 32 + lane;
  const int64_t kstride = (int64_t)NT * 32;
  const int src = (lane + 31) & 31;

  for (int m0 = 0; m0 < np; m0 += 16) {
    const int nrows = min(16, np - m0);
    float ad[2][4] = {};
    uint32_t pd[kPf];
#pragma unroll
    for (int i = 0; i < kPf; ++i) pd[i] = i < KT ? ldg_nc_u32(wd + i * kstride) : 0u;
    for (int kt0 = 0; kt0 < KT; kt0 += kPf) {
#pragma unroll
      for (int i = 0; i < kPf; ++i) {
        const int kt = kt0 + i;
        if (kt >= KT) break;
        const uint32_t cd = pd[i];
        const int nk = kt + kPf;
        pd[i] = nk < KT ? ldg_nc_u32(wd + nk * kstride) : 0u;
        uint32_t bd[4], ax[4];
        trellis_frags(cd, __shfl_sync(0xffffffffu, cd, src), bd);
        load_a_frag(a.xd, a.N, p0 + m0, nrows, kt, ax);
        mma_f16_16816(ad[0], ax, bd[0], bd[1]);
        mma_f16_16816(ad[1], ax, bd[2], bd[3]);
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c = warp * 16 + h * 8 + 2 * q;
      zd[g][c] = ad[h][0]; zd[g][c + 1] = ad[h][1]; zd[g + 8][c] = ad[h][2]; zd[g + 8][c + 1] = ad[h][3];
    }
    __syncthreads();
    for (int r = warp; r < nrows; r += 8) {
      float v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = zd[r][lane * 4 + i];
      fwht128_warp(v);
      const int col = nb * 128 + lane * 4;
      const float w = a.pair_w[p0 + m0 + r];
      float4 o;
      o.x = v[0] * __half2float(a.svh_d[(int64_t)e * a.Dout + col + 0]) * w;
      o.y = v[1] * __half2float(a.svh_d[(int64_t)e * a.Dout + col + 1]) * w;
      o.z = v[2] * __half2float(a.svh_d[(int64_t)e * a.Dout + col + 2]) * w;
      o.w = v[3] * __half2float(a.svh_d[(int64_t)e * a.Dout + col + 3]) * w;
      *reinterpret_cast<float4*>(a.yd + (int64_t)(p0 + m0 + r) * a.Dout + col) = o;
    }
    __syncthreads();
  }
}

__global__ void moe_combine_kernel(const float* yd, const int* pair_of, int R, int top_k, int D, float* out,
                                   int accumulate) {
  const int r = blockIdx.y;
  const int d = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (d >= D) return;
  float4 acc = accumulate ? *reinterpret_cast<const float4*>(out + (int64_t)r * D + d) : make_float4(0, 0, 0, 0);
  for (int k = 0; k < top_k; ++k) {
    const float4 v = *reinterpret_cast<const float4*>(yd + (int64_t)pair_of[r * top_k + k] * D + d);
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
  *reinterpret_cast<float4*>(out + (int64_t)r * D + d) = acc;
}

__global__ void exl3_unpack_kernel(const int16_t* tr, int K, int N, __half* out) {
  const int lane = threadIdx.x & 31;
  const int tile = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int NT = N / 16;
  if (tile >= (K / 16) * NT) return;
  const int kt = tile / NT, nt = tile % NT;
  const uint32_t w = reinterpret_cast<const uint32_t*>(tr)[(int64_t)tile * 32 + lane];
  uint32_t b[4];
  trellis_frags(w, __shfl_sync(0xffffffffu, w, (lane + 31) & 31), b);
  const int g = lane >> 2, q = lane & 3;
  // value j of lane l sits at (row 2q + (j&1) + 8*((j>>1)&1), col g + 8*(j>>2))
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t reg = b[j >> 1];
    const uint16_t bits = (j & 1) ? (uint16_t)(reg >> 16) : (uint16_t)(reg & 0xffffu);
    const int row = 2 * q + (j & 1) + 8 * ((j >> 1) & 1);
    const int col = g + 8 * (j >> 2);
    out[(int64_t)(kt * 16 + row) * N + nt * 16 + col] = __ushort_as_half(bits);
  }
}

}  // namespace g53

using namespace g53;

cudaError_t g53_moe_route(const RouteArgs& a, cudaStream_t st) {
  if (a.E > kMaxE || a.R * a.top_k > kMaxPairs || a.top_k > 32) return cudaErrorInvalidValue;
  moe_route_kernel<<<1, 1024, 0, st>>>(a);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}

cudaError_t g53_exl3_rot_in(const Exl3Args& a, cudaStream_t st) {
  dim3 grid(a.pairs, (a.K / 128 + 3) / 4);
  exl3_rot_in_kernel<<<grid, 128, 0, st>>>(a);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}

cudaError_t g53_exl3_gate_up(const Exl3Args& a, cudaStream_t st) {
  if (a.K % 128 || a.N % 128) return cudaErrorInvalidValue;
  dim3 grid(a.N / 128, a.max_groups);
  exl3_gate_up_kernel<<<grid, 256, 0, st>>>(a);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}

cudaError_t g53_exl3_down(const Exl3Args& a, cudaStream_t st) {
  if (a.Dout % 128 || a.N % 16) return cudaErrorInvalidValue;
  dim3 grid(a.Dout / 128, a.max_groups);
  exl3_down_kernel<<<grid, 256, 0, st>>>(a);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}

cudaError_t g53_moe_combine(const float* yd, const int* pair_of, int R, int top_k, int D, float* out,
                            int accumulate, cudaStream_t st) {
  if (D % 4) return cudaErrorInvalidValue;
  dim3 grid((D / 4 + 255) / 256, R);
  moe_combine_kernel<<<grid, 256, 0, st>>>(yd, pair_of, R, top_k, D, out, accumulate);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}

cudaError_t g53_exl3_unpack(const int16_t* tr, int K, int N, __half* out, cudaStream_t st) {
  const int tiles = (K / 16) * (N / 16);
  exl3_unpack_kernel<<<(tiles + 7) / 8, 256, 0, st>>>(tr, K, N, out);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}

// ---------------------------------------------------------------------------------------------------------------
// routing for large row counts (prefill chunks): many CTAs
// ---------------------------------------------------------------------------------------------------------------
namespace g53 {

__global__ void __launch_bounds__(256) moe_topk_kernel(RouteArgs a, int* counts) {
  const int lane = threadIdx.x & 31;
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= a.R) return;
  constexpr int kPerLane = kMaxE / 32;
  const float* lg = a.logits + (int64_t)r * a.E;
  float cv[kPerLane];
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) {
    const int e = lane + 32 * i;
    cv[i] = e < a.E ? sigmoidf_(lg[e]) + a.bias[e] : -INFINITY;
  }
  float sel_sum = 0.f, wt_l = 0.f;
  int pick_l = 0;
  for (int k = 0; k < a.top_k; ++k) {
    float best = -INFINITY;
    int bid = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kPerLane; ++i)
      if (cv[i] > best) { best = cv[i]; bid = lane + 32 * i; }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bid, o);
      if (ob > best || (ob == best && oi < bid)) { best = ob; bid = oi; }
    }
    if ((bid & 31) == lane) {
#pragma unroll
      for (int i = 0; i < kPerLane; ++i)
        if (lane + 32 * i == bid) cv[i] = -INFINITY;
    }
    const float w = sigmoidf_(lg[bid]);
    sel_sum += w;
    if (lane == k) { pick_l = bid; wt_l = w; }
  }
  const float inv = a.norm ? 1.f / (sel_sum + 1e-20f) : 1.f;
  if (lane < a.top_k) {
    a.topk_ids[r * a.top_k + lane] = pick_l;
    a.topk_w[r * a.top_k + lane] = wt_l * inv * a.scale;
    atomicAdd(&counts[pick_l], 1);
  }
}

__global__ void __launch_bounds__(1024) moe_scan_kernel(RouteArgs a, int* counts, int* fill) {
  __shared__ int wsum[32];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  // E <= 1024: one element per thread, block-wide exclusive scan of counts and of the used flags
  const int c = tid < a.E ? counts[tid] : 0;
  const int used = c > 0;
  int xs = c, xu = used;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int ys = __shfl_up_sync(0xffffffffu, xs, o), yu = __shfl_up_sync(0xffffffffu, xu, o);
    if (lane >= o) { xs += ys; xu += yu; }
  }
  __shared__ int wu[32];
  if (lane == 31) { wsum[wid] = xs; wu[wid] = xu; }
  __syncthreads();
  if (wid == 0) {
    int ts = wsum[lane], tu = wu[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int ys = __shfl_up_sync(0xffffffffu, ts, o), yu = __shfl_up_sync(0xffffffffu, tu, o);
      if (lane >= o) { ts += ys; tu += yu; }
    }
    wsum[lane] = ts;
    wu[lane] = tu;
  }
  __syncthreads();
  const int start = (wid > 0 ? wsum[wid - 1] : 0) + xs - c;
  const int uidx = (wid > 0 ? wu[wid - 1] : 0) + xu - used;
  if (tid < a.E) {
    fill[tid] = start;
    if (used && uidx < a.max_groups) {
      a.group_expert[uidx] = tid;
      a.group_offset[uidx] = start;
    }
  }
  const int total_used = wu[31];
  const int total = wsum[31];
  if (tid == 0) a.group_count[0] = total_used;
  for (int v = total_used + tid; v <= a.max_groups; v += blockDim.x) a.group_offset[v] = total;
}

__global__ void moe_scatter_kernel(RouteArgs a, int* fill) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.R * a.top_k) return;
  const int e = a.topk_ids[i];
  const int pos = atomicAdd(&fill[e], 1);
  a.pair_of[i] = pos;
  a.pair_token[pos] = i / a.top_k;
  a.pair_expert[pos] = e;
  a.pair_w[pos] = a.topk_w[i];
}

}  // namespace g53

cudaError_t g53_moe_route_large(const RouteArgs& a, int* counts, int* fill, cudaStream_t st) {
  using namespace g53;
  if (a.E > 1024 || a.E > kMaxE || a.top_k > 32) return cudaErrorInvalidValue;
  cudaError_t e = cudaMemsetAsync(counts, 0, sizeof(int) * a.E, st);
  if (e != cudaSuccess) return e;
  moe_topk_kernel<<<(a.R + 7) / 8, 256, 0, st>>>(a, counts);
  G53_CHECK_LAUNCH();
  moe_scan_kernel<<<1, 1024, 0, st>>>(a, counts, fill);
  G53_CHECK_LAUNCH();
  const int P = a.R * a.top_k;
  moe_scatter_kernel<<<(P + 255) / 256, 256, 0, st>>>(a, fill);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}
