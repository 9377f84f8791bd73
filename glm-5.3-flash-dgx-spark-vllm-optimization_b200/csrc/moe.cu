// Routed MoE for decode-sized batches: router top-k + grouping, and the EXL3 grouped expert GEMMs.
//
// EXL3 path (the trellis format is described in ops/exl3.py):
//   rot_in    xh[p] = f16(H128(x[token(p)] * suh[expert(p)]))                 (gate and up, per sorted pair)
//   gate_up   per (expert group, 128-column block): Z = xh @ W_q on tensor cores, the trellis decoded in
//             registers straight into mma.m16n8k16 fragments (each lane decodes the 8 values of its fragment
//             from its own 32-bit word and its left neighbour's); the weight tile is the A operand (16 features)
//             and up to 8 tokens are the B operand; epilogue in shared memory: H128 of the gate and
//             up rows, * svh, SwiGLU with clamp, * suh of the down projection, H128 -> f16 down input
//   down      same GEMM over the local expert width; epilogue H128, * svh, * routing weight -> fp32 per pair
//   combine   out[r] = sum over slots (fixed order) of the pair outputs
// One CTA owns one full 128-column Hadamard block of one expert, so both output rotations stay on chip.
// Reference counterparts: code/fork/kernels/exl3.cu:110 (grouped_kernel), :322 (rot_in), :371/:455 (epilogues),
// :529/:582 (route_prep / route_ids).
#include <algorithm>
#include <cooperative_groups.h>
#include <cstdlib>
#include "common.cuh"
#include "launchers.h"

namespace cg = cooperative_groups;

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
  pdl_wait();                          // the router logits come from the previous kernel
  pdl_trigger();
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
    int pick_l = 0;
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
      if (lane == k) pick_l = bid;
    }
    // routing weights of the picks: one load per lane (in parallel), summed over the picks in pick order
    const float wt_l = lane < a.top_k ? sigmoidf_(lg[pick_l]) : 0.f;
    float sel_sum = 0.f;
    for (int k = 0; k < a.top_k; ++k) sel_sum += __shfl_sync(0xffffffffu, wt_l, k);
    const float inv = a.norm ? 1.f / (sel_sum + 1e-20f) : 1.f;
    if (lane < a.top_k) {
      a.topk_ids[r * a.top_k + lane] = pick_l;
      a.topk_w[r * a.top_k + lane] = wt_l * inv * a.scale;
      pe[r * a.top_k + lane] = pick_l;
      atomicAdd(&cnt[pick_l], 1);
    }
  }
  __syncthreads();
  // exclusive scans of the counts and of the non-empty flags (packed: count in bits 0-15, flag in bits 16-31)
  {
    __shared__ int wsum[32];
    const int c = tid < a.E ? cnt[tid] : 0;
    const int2 sc = block_scan(c | ((c > 0) << 16), wsum);
    const int s = sc.x & 0xffff, u = sc.x >> 16, total = sc.y & 0xffff, groups = sc.y >> 16;
    if (tid < a.E) {
      start[tid] = s;
      if (c > 0 && u < a.max_groups) { a.group_expert[u] = tid; a.group_offset[u] = s; }
    }
    if (tid == 0) { start[a.E] = total; a.group_count[0] = groups; }
    for (int v = groups + tid; v <= a.max_groups; v += blockDim.x) a.group_offset[v] = total;
  }
  __syncthreads();
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
// Decode-path trellis evaluation with split codebook halves.
//
// A codebook value is fp16(lo) + fp16(hi) of the masked product x = (s * 0xCBAC1FED & 0x8FFF8FFF) ^ 0x3B603B60.
// The decode kernels never add the halves on the CUDA cores: the 32-bit x is itself an f16x2 register holding
// (lo, hi), and it enters the tensor core as two consecutive k entries of the A operand, against the same input
// value duplicated in the B operand, so the MMA forms lo*x_k + hi*x_k in fp32.  Against the format's single fp16
// rounding of lo + hi this differs by at most half an fp16 ulp of the weight (the same order as the fp16 rounding
// of the rotated inputs) and it saves the packing and the fp16 add of every value: per state the CUDA cores do
// the window extraction, one IMAD and one LOP3.
//
// Per 16x16 tile, lane (g, q) holds states j = 0..7 at (k, n) = (2q + (j&1) + 8((j>>1)&1), g + 8(j>>2)).  The
// tile becomes two m16n8k16 steps with the weight as A (16 features x 16 virtual k) and 8 tokens as B; virtual k
// slots (q, q+4) of step t carry original k (2q + 8t, 2q + 1 + 8t):
//   step 0: A = {x0, x4, x1, x5}, B = {dup(in[2q]),     dup(in[2q+1])}
//   step 1: A = {x2, x6, x3, x7}, B = {dup(in[2q+8]),   dup(in[2q+9])}
// The rotated inputs (xh_g, xh_u, xd) of the decode path are stored as duplicated f16 pairs, one 32-bit word per
// element, ordered so that lane quad q finds the 4 words of each k-tile together and the 4 k-tiles of a 64-wide
// chunk next to each other: word(k) below.  A row of K elements takes 2K halves.
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ int dup_word(int k) {
  const int w = k & 63, t = w >> 4, kk = w & 15;
  const int q = (kk & 7) >> 1, i = (kk & 1) | ((kk >> 3) << 1);
  return (k & ~63) | (q << 4) | (t << 2) | i;
}

__device__ __forceinline__ uint32_t dup_half(float v) {
  const __half h = __float2half_rn(v);
  const uint32_t b = __half_as_ushort(h);
  return b | (b << 16);
}

// ---------------------------------------------------------------------------------------------------------------
// The 8 masked products of a lane's fragment, balanced over the two integer pipes.
//
// Measured on B200 (one warp instruction per SMSP per clock is issued): LOP3, PRMT, SHF and IMAD each retire 0.5
// warp instructions per clock (LOP3 / PRMT / SHF on the ALU pipe, IMAD on the FMA-heavy pipe), IMAD.HI 0.25.  The
// value of window b (stream bits [b, b + 16) counted from the LSB of the lane's word `cur`, with `prev` above it)
// is x_b = (s_b * C & M) ^ X.  Any 32-bit t with s_b in its low half gives s_b * C = t * C - (t >> 16) * (C << 16)
// (mod 2^32): the high half of t only adds (t >> 16) * C << 16 to the product.  And t >> 16 is itself the window
// 16 bits further up, which the tile needs anyway, so a pair of windows (b, b + 16) costs one word t_b, one
// extraction of s_{b+16} and three IMADs, instead of two extractions and two IMADs:
//   pair (0, 16):  t = cur (free),                   s16 = prmt(cur)
//   pair (8, 24):  t8 = prmt(cur, prev),              s24 = prmt(t8)
//   pair (4, 20):  t4 = shf(prev:cur, 4),             s20 = prmt(t4)
//   pair (12, 28): t12 = shf(prev:cur, 12),           s28 = prmt(t12)
// Per word: 7 ALU extractions + 8 LOP3 on the ALU pipe, 12 IMADs on the FMA-heavy pipe (the previous all-ALU
// extraction took 10 ALU operations plus two IMAD.HI).  Measured in isolation (decode + mma.sync, operands from
// shared memory): 18.1 values per clock per SM against 12.8, bit-identical products.
// Fragment order (value j = window b = 28 - 4j): a0 = {x0, x4, x1, x5}, a1 = {x2, x6, x3, x7}.
// ---------------------------------------------------------------------------------------------------------------
template <uint32_t SEL>
__device__ __forceinline__ uint32_t prmt_(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "n"(SEL));
  return r;
}

template <uint32_t SH>
__device__ __forceinline__ uint32_t shf_r_(uint32_t lo, uint32_t hi) {
  uint32_t r;
  asm("shf.r.wrap.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(lo), "r"(hi), "n"(SH));
  return r;
}

// (x & 0x8FFF8FFF) ^ 0x3B603B60 as one LOP3 (truth table 0x6a = (a & b) ^ c)
__device__ __forceinline__ uint32_t mcg_mask_(uint32_t x) {
  uint32_t r;
  asm("lop3.b32 %0, %1, 0x8FFF8FFF, 0x3B603B60, 0x6a;" : "=r"(r) : "r"(x));
  return r;
}

__device__ __forceinline__ void trellis_tile_mma(float (&c)[4], uint32_t cur, uint32_t prev, const uint4& b) {
  constexpr uint32_t C = 0xCBAC1FEDu, Cn = 0u - (C << 16);
  const uint32_t s16 = prmt_<0x4432>(cur, 0u);          // bits [16, 32)
  const uint32_t t8 = prmt_<0x4321>(cur, prev);         // bits [8, 40)
  const uint32_t s24 = prmt_<0x4432>(t8, 0u);           // bits [24, 40)
  const uint32_t t4 = shf_r_<4>(cur, prev);             // bits [4, 36)
  const uint32_t s20 = prmt_<0x4432>(t4, 0u);           // bits [20, 36)
  const uint32_t t12 = shf_r_<12>(cur, prev);           // bits [12, 44)
  const uint32_t s28 = prmt_<0x4432>(t12, 0u);          // bits [28, 44)
  uint32_t a0[4], a1[4];
  a0[0] = mcg_mask_(s28 * C);                           // x0
  a0[1] = mcg_mask_(t12 * C + s28 * Cn);                // x4
  a0[2] = mcg_mask_(s24 * C);                           // x1
  a0[3] = mcg_mask_(t8 * C + s24 * Cn);                 // x5
  mma_f16_16816(c, a0, b.x, b.y);
  a1[0] = mcg_mask_(s20 * C);                           // x2
  a1[1] = mcg_mask_(t4 * C + s20 * Cn);                 // x6
  a1[2] = mcg_mask_(s16 * C);                           // x3
  a1[3] = mcg_mask_(cur * C + s16 * Cn);                // x7
  mma_f16_16816(c, a1, b.z, b.w);
}

// ---------------------------------------------------------------------------------------------------------------
// rot_in: one warp per (sorted pair, 128-block); gate and up rotated inputs in f16
// ---------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(128) exl3_rot_in_kernel(Exl3Args a) {
  pdl_wait();                          // pairs from the routing kernel
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int blk = blockIdx.y * 4 + (threadIdx.x >> 5);
  if (blk * 128 >= a.K) return;
  const int np = a.pair_count ? min(*a.pair_count, a.pairs) : a.pairs;
  for (int p = blockIdx.x; p < np; p += gridDim.x) {   // pairs on grid.x (prefill chunks exceed 65535 pairs)
    const int r = a.pair_token[p], e = a.pair_expert[p];
    if (!g53_in_bounds(r, a.n_rows, 7) || !g53_in_bounds(e, a.n_experts, 6)) continue;   // warp-uniform
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
    if (a.decode_layout) {                         // duplicated words (see dup_word); (k, k+1) are adjacent words
      uint32_t* og = reinterpret_cast<uint32_t*>(a.xh_g) + (int64_t)p * a.K;
      uint32_t* ou = reinterpret_cast<uint32_t*>(a.xh_u) + (int64_t)p * a.K;
      const int w0 = dup_word(c0), w2 = dup_word(c0 + 2);
      *reinterpret_cast<uint2*>(og + w0) = make_uint2(dup_half(g[0]), dup_half(g[1]));
      *reinterpret_cast<uint2*>(og + w2) = make_uint2(dup_half(g[2]), dup_half(g[3]));
      *reinterpret_cast<uint2*>(ou + w0) = make_uint2(dup_half(u[0]), dup_half(u[1]));
      *reinterpret_cast<uint2*>(ou + w2) = make_uint2(dup_half(u[2]), dup_half(u[3]));
      continue;
    }
    __half2* og = reinterpret_cast<__half2*>(a.xh_g + (int64_t)p * a.K + c0);
    __half2* ou = reinterpret_cast<__half2*>(a.xh_u + (int64_t)p * a.K + c0);
    og[0] = __floats2half2_rn(g[0], g[1]); og[1] = __floats2half2_rn(g[2], g[3]);
    ou[0] = __floats2half2_rn(u[0], u[1]); ou[1] = __floats2half2_rn(u[2], u[3]);
  }
}

// Prefill layout (plain f16 rows), 16-byte accesses: a half-warp owns one 128-column block, a lane 8 consecutive
// columns; grid (pairs, K / 2048), 256 threads.  The butterflies are those of fwht128_warp in the same stage order
// (h = 1, 2, 4 inside the lane, then lane bits 0..3 for h = 8 .. 64), each stage's (a + b, a - b) computed with the
// same single roundings, so the output is bit-identical to exl3_rot_in_kernel's.
__device__ __forceinline__ void fwht128_half(float (&v)[8]) {
#pragma unroll
  for (int h = 1; h < 8; h <<= 1) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i & h) continue;
      const float x0 = v[i], x1 = v[i + h];
      v[i] = x0 + x1;
      v[i + h] = x0 - x1;
    }
  }
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int m = 1; m < 16; m <<= 1) {
    const float sg = (lane & m) ? -1.f : 1.f;         // lower lane: v + p, upper lane: p - v
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float pv = __shfl_xor_sync(0xffffffffu, v[i], m);
      v[i] = fmaf(sg, v[i], pv);
    }
  }
  const float s = 0.08838834764831845f;   // 1/sqrt(128)
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] *= s;
}

__global__ void __launch_bounds__(256) exl3_rot_in_wide_kernel(Exl3Args a) {
  pdl_wait();                          // pairs from the routing kernel
  pdl_trigger();
  const int blk = blockIdx.y * 16 + (threadIdx.x >> 4);
  if (blk * 128 >= a.K) return;        // whole warps: K is a multiple of 256
  const int c0 = blk * 128 + (threadIdx.x & 15) * 8;
  const int np = a.pair_count ? min(*a.pair_count, a.pairs) : a.pairs;
  for (int p = blockIdx.x; p < np; p += gridDim.x) {
    const int r = a.pair_token[p], e = a.pair_expert[p];
    if (!g53_in_bounds(r, a.n_rows, 7) || !g53_in_bounds(e, a.n_experts, 6)) continue;   // CTA-uniform
    const uint4 xw = *reinterpret_cast<const uint4*>(a.x + (int64_t)r * a.ldx + c0);
    const uint4 gw = *reinterpret_cast<const uint4*>(a.suh_g + (int64_t)e * a.K + c0);
    const uint4 uw = *reinterpret_cast<const uint4*>(a.suh_u + (int64_t)e * a.K + c0);
    const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&xw);
    const __half2* g2 = reinterpret_cast<const __half2*>(&gw);
    const __half2* u2 = reinterpret_cast<const __half2*>(&uw);
    float g[8], u[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 xf = __bfloat1622float2(x2[i]);
      const float2 gf = __half22float2(g2[i]), uf = __half22float2(u2[i]);
      g[2 * i] = xf.x * gf.x; g[2 * i + 1] = xf.y * gf.y;
      u[2 * i] = xf.x * uf.x; u[2 * i + 1] = xf.y * uf.y;
    }
    fwht128_half(g);
    fwht128_half(u);
    uint4 og, ou;
    __half2* og2 = reinterpret_cast<__half2*>(&og);
    __half2* ou2 = reinterpret_cast<__half2*>(&ou);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      og2[i] = __floats2half2_rn(g[2 * i], g[2 * i + 1]);
      ou2[i] = __floats2half2_rn(u[2 * i], u[2 * i + 1]);
    }
    *reinterpret_cast<uint4*>(a.xh_g + (int64_t)p * a.K + c0) = og;
    *reinterpret_cast<uint4*>(a.xh_u + (int64_t)p * a.K + c0) = ou;
  }
}

// accumulator (16 features x 8 tokens) of one warp's n-tile -> z[token][feature]
__device__ __forceinline__ void acc_to_smem(const float (&c)[4], int warp, float (*z)[132]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const int t = 2 * q, f = warp * 16 + g;
  z[t][f] = c[0];
  z[t + 1][f] = c[1];
  z[t][f + 8] = c[2];
  z[t + 1][f + 8] = c[3];
}

// split-K over a cluster along z: rank 0 adds the other ranks' partial tiles (fixed rank order) to its own
template <int KSPL>
__device__ __forceinline__ void cluster_reduce_tile(float (*z)[132], int nrows) {
  if constexpr (KSPL > 1) {
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    if (cluster.block_rank() == 0) {
      for (int i = threadIdx.x; i < 8 * 128; i += blockDim.x) {
        const int t = i >> 7, f = i & 127;
        if (t >= nrows) continue;
        float v = z[t][f];
#pragma unroll
        for (int r = 1; r < KSPL; ++r) v += cluster.map_shared_rank(&z[0][0], r)[t * 132 + f];
        z[t][f] = v;
      }
    }
  }
}

template <int KSPL>
__device__ __forceinline__ void cluster_release() {
  if constexpr (KSPL > 1) cg::this_cluster().sync();   // rank 0 has read every rank's tile
}

// ---------------------------------------------------------------------------------------------------------------
// gate + up: grid (N/128 column blocks, max_groups, KSPL), 8 warps; warp w owns n-tile (block*8 + w) of gate and
// up; the KSPL CTAs of a cluster split K and rank 0 reduces and runs the epilogue.
// Up to 8 tokens of the group per pass (one n8 block; a decode window of R <= 8 rows never has more per expert);
// larger groups decode the trellis again for every further 8 tokens.
// ---------------------------------------------------------------------------------------------------------------
// KS: the k-tile stride of the trellis in 32-bit words (N/16 tiles of 32 words), a compile-time constant for the
// model's shapes (0: read from the arguments).  With it, the four words of a chunk are one pointer plus immediate
// offsets and the walk over K is one pointer increment per chunk, instead of a 64-bit address product per load.
template <int KSPL, int KS>
__device__ __forceinline__ void gate_up_group(const Exl3Args& a, int u, float (*zg)[132], float (*zu)[132]) {
  const int e = a.group_expert[u];
  if (!g53_in_bounds(e, a.n_experts, 6)) return;       // uniform over the cluster (same group)
  const int p0 = a.group_offset[u];
  const int np = a.group_offset[u + 1] - p0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const int nb = blockIdx.x;
  const int nt = nb * 8 + warp;
  const int KT = a.K / 16, NT = a.N / 16;
  const int ks = KSPL > 1 ? (int)blockIdx.z : 0, cper = a.K / 64 / KSPL, c_lo = ks * cper, c_hi = c_lo + cper;
  const int kstride = KS > 0 ? KS : NT * 32;
  const uint32_t* wg = reinterpret_cast<const uint32_t*>(a.tr_g) + ((int64_t)e * KT * NT + nt) * 32 + lane +
                       (int64_t)4 * c_lo * kstride;
  const uint32_t* wu = reinterpret_cast<const uint32_t*>(a.tr_u) + ((int64_t)e * KT * NT + nt) * 32 + lane +
                       (int64_t)4 * c_lo * kstride;
  const int src = (lane + 31) & 31;
  const uint64_t pol = l2_evict_first_policy();     // the codes are read once per step: replace them first in L2

  for (int m0 = 0; m0 < np; m0 += 8) {
    const int nrows = min(8, np - m0);
    // token columns past the group read the group's first row: their MMA columns are never stored
    const int64_t r0 = (int64_t)(p0 + m0 + (g < nrows ? g : 0)) * 2 * a.K + q * 32;
    float cg[4] = {}, cu[4] = {};
    uint32_t pg[4], pu[4];
    const uint32_t* pgp = wg;
    const uint32_t* pup = wu;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      pg[i] = ldg_nc_u32_ef(pgp + i * kstride, pol);
      pu[i] = ldg_nc_u32_ef(pup + i * kstride, pol);
    }
    const uint4* bgp = reinterpret_cast<const uint4*>(a.xh_g + r0 + c_lo * 128);
    const uint4* bup = reinterpret_cast<const uint4*>(a.xh_u + r0 + c_lo * 128);
    for (int c = c_lo; c < c_hi; ++c) {
      uint32_t ng[4], nu[4];
      if (c + 1 < c_hi) { pgp += 4 * kstride; pup += 4 * kstride; }    // the last chunk reloads itself
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        ng[i] = ldg_nc_u32_ef(pgp + i * kstride, pol);
        nu[i] = ldg_nc_u32_ef(pup + i * kstride, pol);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 bg = bgp[i], bu = bup[i];
        trellis_tile_mma(cg, pg[i], __shfl_sync(0xffffffffu, pg[i], src), bg);
        trellis_tile_mma(cu, pu[i], __shfl_sync(0xffffffffu, pu[i], src), bu);
      }
      bgp += 16;                                    // 128 halves = 16 uint4 per 64-wide chunk
      bup += 16;
#pragma unroll
      for (int i = 0; i < 4; ++i) { pg[i] = ng[i]; pu[i] = nu[i]; }
    }
    acc_to_smem(cg, warp, zg);
    acc_to_smem(cu, warp, zu);
    __syncthreads();
    cluster_reduce_tile<KSPL>(zg, nrows);
    cluster_reduce_tile<KSPL>(zu, nrows);
    __syncthreads();
    for (int r = warp; r < nrows && ks == 0; r += 8) {
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
      uint32_t* o = reinterpret_cast<uint32_t*>(a.xd) + (int64_t)(p0 + m0 + r) * a.N;
      *reinterpret_cast<uint2*>(o + dup_word(col)) = make_uint2(dup_half(act[0]), dup_half(act[1]));
      *reinterpret_cast<uint2*>(o + dup_word(col + 2)) = make_uint2(dup_half(act[2]), dup_half(act[3]));
    }
    cluster_release<KSPL>();
    __syncthreads();
  }
}

// this CTA's share of the L2 prefetch: 64 KB chunks of the concatenated ranges, chunk i by CTA i mod grid size
__device__ __forceinline__ void l2_prefetch_share(const L2Ranges& r) {
  constexpr int64_t kChunk = 64 << 10;
  const int64_t cta = blockIdx.x + (int64_t)gridDim.x * (blockIdx.y + (int64_t)gridDim.y * blockIdx.z);
  const int64_t ncta = (int64_t)gridDim.x * gridDim.y * gridDim.z;
  int64_t base = 0;                              // chunk index of the first chunk of range j
  for (int j = 0; j < r.count; ++j) {
    const int64_t n = r.bytes[j], chunks = (n + kChunk - 1) / kChunk;
    for (int64_t c = ((cta - base) % ncta + ncta) % ncta; c < chunks; c += ncta) {
      const int64_t off = c * kChunk, rem = n - off;
      const uint32_t sz = (uint32_t)((rem < kChunk ? rem : kChunk) & ~(int64_t)15);
      if (sz) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(r.ptr[j] + off), "r"(sz) : "memory");
    }
    base += chunks;
  }
}

// CTAs loop over the groups (grid.y may be smaller than the group table: a decode window routes to few experts)
template <int KSPL, int KS>
__global__ void __launch_bounds__(256, 4) exl3_gate_up_kernel(Exl3Args a) {
  __shared__ float zg[8][132];
  __shared__ float zu[8][132];
  if (a.pf.count && threadIdx.x == 0) l2_prefetch_share(a.pf);
  pdl_wait();                          // rotated inputs and the group table from the previous kernels
  pdl_trigger();
  const int ng = min(a.group_count[0], a.max_groups);
  for (int u = blockIdx.y; u < ng; u += gridDim.y) gate_up_group<KSPL, KS>(a, u, zg, zu);
}

// expert parallelism: the last CTA of the down kernel (all pair rows stored into the sources' combine buffers and
// made visible system-wide) releases one flag on every source rank
__device__ __forceinline__ void ep_count_in(const Exl3Args& a) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned prev = atomicAdd(a.done, 1u);
    if (prev == gridDim.x * gridDim.y * gridDim.z - 1) {
      *a.done = 0u;
      __threadfence_system();
      for (int s = 0; s < a.push_world; ++s) red_release_sys_add(reinterpret_cast<unsigned*>(a.push_flags[s]), 1u);
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// down: grid (Dout/128, max_groups, KSPL) with K split over a cluster as in gate_up; epilogue H128, * svh,
// * routing weight -> yd[pair] fp32
// ---------------------------------------------------------------------------------------------------------------
template <int KSPL, int KS>
__device__ __forceinline__ void down_group(const Exl3Args& a, int u, float (*zd)[132]) {   // KSPL in {1, 2}
  const int e = a.group_expert[u];
  if (!g53_in_bounds(e, a.n_experts, 6)) return;       // uniform over the cluster (same group)
  const int p0 = a.group_offset[u];
  const int np = a.group_offset[u + 1] - p0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const int nb = blockIdx.x;
  const int nt = nb * 8 + warp;
  const int KT = a.N / 16, NT = a.Dout / 16;
  const int ks = KSPL > 1 ? (int)blockIdx.z : 0, cper = a.N / 64 / KSPL, c_lo = ks * cper, c_hi = c_lo + cper;
  const int kstride = KS > 0 ? KS : NT * 32;
  const uint32_t* wd = reinterpret_cast<const uint32_t*>(a.tr_d) + ((int64_t)e * KT * NT + nt) * 32 + lane +
                       (int64_t)4 * c_lo * kstride;
  const int src = (lane + 31) & 31;
  const uint64_t pol = l2_evict_first_policy();     // the codes are read once per step: replace them first in L2

  for (int m0 = 0; m0 < np; m0 += 8) {
    const int nrows = min(8, np - m0);
    // token columns past the group read the group's first row: their MMA columns are never stored
    const int64_t r0 = (int64_t)(p0 + m0 + (g < nrows ? g : 0)) * 2 * a.N + q * 32;
    float cd[4] = {};
    if ((c_hi - c_lo) % 2 == 0) {
      // two independent k-streams per warp (the two halves of the warp's chunk range, one chunk of each in flight
      // and one prefetched): twice the loads in flight of a single stream, which left the kernel waiting on memory
      const int half = (c_hi - c_lo) / 2;
      float ce[4] = {};
      uint32_t pd[4], pe[4];
      const uint32_t* pdp = wd;
      const uint32_t* pep = wd + (int64_t)4 * half * kstride;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        pd[i] = ldg_nc_u32_ef(pdp + i * kstride, pol);
        pe[i] = ldg_nc_u32_ef(pep + i * kstride, pol);
      }
      const uint4* bp = reinterpret_cast<const uint4*>(a.xd + r0 + c_lo * 128);
      const uint4* bq = bp + 16 * half;
      for (int c = 0; c < half; ++c) {
        uint32_t nd[4], ne[4];
        if (c + 1 < half) { pdp += 4 * kstride; pep += 4 * kstride; }    // the last chunk reloads itself
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          nd[i] = ldg_nc_u32_ef(pdp + i * kstride, pol);
          ne[i] = ldg_nc_u32_ef(pep + i * kstride, pol);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint4 b = bp[i], b2 = bq[i];
          trellis_tile_mma(cd, pd[i], __shfl_sync(0xffffffffu, pd[i], src), b);
          trellis_tile_mma(ce, pe[i], __shfl_sync(0xffffffffu, pe[i], src), b2);
        }
        bp += 16;
        bq += 16;
#pragma unroll
        for (int i = 0; i < 4; ++i) { pd[i] = nd[i]; pe[i] = ne[i]; }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) cd[i] += ce[i];
    } else {
      uint32_t pd[4];
      const uint32_t* pdp = wd;
#pragma unroll
      for (int i = 0; i < 4; ++i) pd[i] = ldg_nc_u32_ef(pdp + i * kstride, pol);
      const uint4* bp = reinterpret_cast<const uint4*>(a.xd + r0 + c_lo * 128);
      for (int c = c_lo; c < c_hi; ++c) {
        uint32_t nd[4];
        if (c + 1 < c_hi) pdp += 4 * kstride;        // the last chunk reloads itself
#pragma unroll
        for (int i = 0; i < 4; ++i) nd[i] = ldg_nc_u32_ef(pdp + i * kstride, pol);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint4 b = bp[i];
          trellis_tile_mma(cd, pd[i], __shfl_sync(0xffffffffu, pd[i], src), b);
        }
        bp += 16;
#pragma unroll
        for (int i = 0; i < 4; ++i) pd[i] = nd[i];
      }
    }
    acc_to_smem(cd, warp, zd);
    __syncthreads();
    cluster_reduce_tile<KSPL>(zd, nrows);
    __syncthreads();
    for (int r = warp; r < nrows && ks == 0; r += 8) {
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
      float* dst = a.out_ptrs ? reinterpret_cast<float*>(a.out_ptrs[p0 + m0 + r])     // the source's combine row
                              : a.yd + (int64_t)(p0 + m0 + r) * a.Dout;
      *reinterpret_cast<float4*>(dst + col) = o;
    }
    cluster_release<KSPL>();
    __syncthreads();
  }
}

template <int KSPL, int KS>
__global__ void __launch_bounds__(256) exl3_down_kernel(Exl3Args a) {
  __shared__ float zd[8][132];
  pdl_wait();                          // the gate/up kernel's activations
  pdl_trigger();
  const int ng = min(a.group_count[0], a.max_groups);
  for (int u = blockIdx.y; u < ng; u += gridDim.y) down_group<KSPL, KS>(a, u, zd);
  if (a.out_ptrs) ep_count_in(a);                   // expert parallelism: every CTA counts towards the release
}

__global__ void moe_combine_kernel(const float* yd, const int* pair_of, int R, int top_k, int D, float* out,
                                   int accumulate) {
  pdl_wait();                          // the down kernel's expert outputs
  pdl_trigger();                       // dependents (the next projection) may start prefetching
  const int r = blockIdx.y;
  const int d = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (d >= D) return;
  // accumulate 1: out + y_0 + y_1 + ...; 2: (y_0 + y_1 + ...) + out (the routed sum first, then the value in out)
  float4 acc = accumulate == 1 ? *reinterpret_cast<const float4*>(out + (int64_t)r * D + d) : make_float4(0, 0, 0, 0);
  for (int k = 0; k < top_k; ++k) {
    const float4 v = *reinterpret_cast<const float4*>(yd + (int64_t)pair_of[r * top_k + k] * D + d);
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
  if (accumulate == 2) {
    const float4 o = *reinterpret_cast<const float4*>(out + (int64_t)r * D + d);
    acc.x += o.x; acc.y += o.y; acc.z += o.z; acc.w += o.w;
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
  return g53_launch_pdl(moe_route_kernel, dim3(1), dim3(1024), 0, st, 1, a);
}

cudaError_t g53_exl3_rot_in(const Exl3Args& a, cudaStream_t st) {
  // device-side pair count (expert parallelism): a bounded grid strides over the rows that arrived
  const int gx = a.pair_count ? std::min(a.pairs, 1184) : a.pairs;
  const bool wide = !a.decode_layout && a.K % 256 == 0 && a.ldx % 8 == 0 &&
                    ((reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.suh_g) |
                      reinterpret_cast<uintptr_t>(a.suh_u) | reinterpret_cast<uintptr_t>(a.xh_g) |
                      reinterpret_cast<uintptr_t>(a.xh_u)) & 15) == 0;
  if (wide) return g53_launch_pdl(exl3_rot_in_wide_kernel, dim3(gx, (a.K + 2047) / 2048), dim3(256), 0, st, 1, a);
  return g53_launch_pdl(exl3_rot_in_kernel, dim3(gx, (a.K / 128 + 3) / 4), dim3(128), 0, st, 1, a);
}

// K split over a cluster of KSPL CTAs (more, smaller CTAs: the grid of a decode window is a couple of waves)
template <int KSPL>
static cudaError_t launch_split(void (*kern)(Exl3Args), dim3 grid, const Exl3Args& a, cudaStream_t st) {
  grid.z = KSPL;
  return g53_launch_pdl(kern, grid, dim3(256), 0, st, KSPL, a);
}

// the trellis k-tile stride (words) as a template constant for the model's expert shapes (hidden 4096 with expert
// width 2048 / TP for TP 1..8; the tiny proxy's 512 / 256), the generic kernel otherwise
template <int KSPL>
static cudaError_t gate_up_ks(const Exl3Args& a, dim3 grid, cudaStream_t st) {
  switch (a.N / 16 * 32) {
    case 4096: return launch_split<KSPL>(exl3_gate_up_kernel<KSPL, 4096>, grid, a, st);
    case 2048: return launch_split<KSPL>(exl3_gate_up_kernel<KSPL, 2048>, grid, a, st);
    case 1024: return launch_split<KSPL>(exl3_gate_up_kernel<KSPL, 1024>, grid, a, st);
    case 512: return launch_split<KSPL>(exl3_gate_up_kernel<KSPL, 512>, grid, a, st);
    default: return launch_split<KSPL>(exl3_gate_up_kernel<KSPL, 0>, grid, a, st);
  }
}

template <int KSPL>
static cudaError_t down_ks(const Exl3Args& a, dim3 grid, cudaStream_t st) {
  switch (a.Dout / 16 * 32) {
    case 8192: return launch_split<KSPL>(exl3_down_kernel<KSPL, 8192>, grid, a, st);
    case 1024: return launch_split<KSPL>(exl3_down_kernel<KSPL, 1024>, grid, a, st);
    default: return launch_split<KSPL>(exl3_down_kernel<KSPL, 0>, grid, a, st);
  }
}

cudaError_t g53_exl3_gate_up(const Exl3Args& a, cudaStream_t st) {
  if (a.K % 128 || a.N % 128 || !a.decode_layout) return cudaErrorInvalidValue;
  const dim3 grid(a.N / 128, a.launch_groups > 0 ? std::min(a.launch_groups, a.max_groups) : a.max_groups);
  // K split over a cluster: at least 2, then doubled up to 4 while the grid has fewer than 1024 CTAs.  Measured
  // per MoE layer at 8 tokens (kernel_bench moe --tp N, splits 1 / 2 / 4 / 8, us): TP1 349 / 341 / 356 / 395,
  // TP2 214 / 191 / 203 / 218, TP4 194 / 138 / 136 / 145, TP8 186 / 129 / 100 / 103
  const int kc = a.K / 64;
  int split = 1;
  while ((split < 2 || (split < 4 && (int64_t)grid.x * grid.y * split < 1024)) && kc % (2 * split) == 0 &&
         kc / (2 * split) >= 4)
    split *= 2;
  // GLM53_MOE_DECODE_SPLIT (1, 2, 4 or 8) overrides the choice, for tuning; the K range must divide
  static const int forced = [] {
    const char* e = std::getenv("GLM53_MOE_DECODE_SPLIT");
    return e ? std::atoi(e) : 0;
  }();
  if ((forced == 1 || forced == 2 || forced == 4 || forced == 8) && kc % forced == 0 && kc / forced >= 2)
    split = forced;
  switch (split) {
    case 8: return gate_up_ks<8>(a, grid, st);
    case 4: return gate_up_ks<4>(a, grid, st);
    case 2: return gate_up_ks<2>(a, grid, st);
    default: return gate_up_ks<1>(a, grid, st);
  }
}

cudaError_t g53_exl3_down(const Exl3Args& a, cudaStream_t st) {
  if (a.Dout % 128 || a.N % 64 || !a.decode_layout) return cudaErrorInvalidValue;
  const dim3 grid(a.Dout / 128, a.launch_groups > 0 ? std::min(a.launch_groups, a.max_groups) : a.max_groups);
  // the down grid is already Dout / 128 = 32 column blocks per group; its K (the local expert width) only shrinks
  // with tensor parallelism, so it is never split (two k-streams per warp give each warp its loads in flight)
  return down_ks<1>(a, grid, st);
}

cudaError_t g53_moe_combine(const float* yd, const int* pair_of, int R, int top_k, int D, float* out,
                            int accumulate, cudaStream_t st) {
  if (D % 4) return cudaErrorInvalidValue;
  dim3 grid((D / 4 + 255) / 256, R);
  return g53_launch_pdl(moe_combine_kernel, grid, dim3(256), 0, st, 1, yd, pair_of, R, top_k, D, out, accumulate);
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
