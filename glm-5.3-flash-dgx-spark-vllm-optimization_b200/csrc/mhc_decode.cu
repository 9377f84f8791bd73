// mHC post + pre for decode windows (R <= 16 rows) as ONE kernel: a cluster of 8 CTAs per row splits the columns,
// and the three row-wide reductions of the pre (the n_mix mixing dots with the sum of squares, then the norm of the
// collapsed stream) go through distributed shared memory instead of a second kernel.
//
// CTA (rank q of the row's cluster) owns columns [q D/8, (q+1) D/8), one thread per column pass:
//   post   X_s[d] = bf16(post_s * bf16(branch[d]) + sum_j comb[j, s] X_j[d])   (branch = the rank-ordered sum of
//          the tensor-parallel partials when they were pushed by the peers: bounded wait on their flags first)
//   dots   the column's share of the n_mix dots fn_i . X and of sum X^2 -> CTA sums (fixed warp order) -> every
//          CTA adds the 8 CTA sums in rank order -> pre = sigmoid + eps; rank 0's extra warp: post = 2 sigmoid,
//          comb = Sinkhorn, concurrently with the norm (the next block's mHC is their only reader)
//   norm   collapsed[d] = bf16(sum_s pre_s X_s[d]) from the registers, sum of squares -> all CTAs add the 8 partial
//          sums in rank order -> normed[d] = bf16(collapsed * rsqrt(mean + eps) * w[d])
// The unfused path (hc_partial + hc_finish, mhc.cu) computes the same quantities with another summation order.
// Reference counterpart: code/fork/kernels/smallops.cu:134 (decode mHC post + pre); math as
// code/fork/docs/ref/tf_glue.py:123-175.
#include <cooperative_groups.h>
#include "common.cuh"
#include "launchers.h"

namespace cg = cooperative_groups;

namespace g53 {
namespace hd {

constexpr int kCl = 8;           // CTAs per row
constexpr int kT = 512;          // threads per CTA (one column each at D = 4096)
constexpr int kMaxCols = 2;      // column passes per thread (D <= kCl * kT * kMaxCols = 8192)

template <int S>
__device__ __forceinline__ float row_sum(float v) {
#pragma unroll
  for (int o = 1; o < S; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
template <int S>
__device__ __forceinline__ float row_max(float v) {
#pragma unroll
  for (int o = 1; o < S; o <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
template <int S>
__device__ __forceinline__ float col_sum(float v) {
#pragma unroll
  for (int o = S; o < S * S; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// the kCl CTA partials of `n` values (each CTA's in its own `part`) summed in rank order
__device__ __forceinline__ float cluster_total(cg::cluster_group& cl, float* part, int i) {
  float t = 0.f;
#pragma unroll
  for (int q = 0; q < kCl; ++q) t += cl.map_shared_rank(part, q)[i];
  return t;
}

template <int S>
__global__ void __cluster_dims__(kCl, 1, 1) __launch_bounds__(kT + 32) hc_decode_kernel(HcArgs a) {
  constexpr int NM = 2 * S + S * S;
  cg::cluster_group cl = cg::this_cluster();
  pdl_trigger();
  const int q = (int)cl.block_rank(), r = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int span = a.D / kCl, c0 = q * span;
  __shared__ float wred[kT / 32][NM + 1];
  __shared__ float part[32];            // this CTA's sums: NM dots + sum of squares (then the norm's sum)
  __shared__ float part2[1];
  __shared__ float pre_s[S];
  // the mixing weights do not depend on the previous kernel: pull this CTA's slice towards L2 first
  for (int i = tid; i < NM * S; i += kT)
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a.fn + (int64_t)i * a.D + c0),
                 "r"((uint32_t)(span * 2) & ~15u) : "memory");
  pdl_wait();
  if (a.gath) {
    if (tid == 0) {
      const unsigned target = *reinterpret_cast<volatile unsigned*>(a.epoch) + 1u;
      for (int j = 0; j < a.world; ++j) wait_flag_geq(a.flags + j, target, a.err, 31);
    }
    __syncthreads();
  }
  __nv_bfloat16* xr = a.X + (int64_t)r * S * a.D;
  float x[kMaxCols][S];
  float t[NM + 1];
#pragma unroll
  for (int i = 0; i <= NM; ++i) t[i] = 0.f;
#pragma unroll
  for (int p = 0; p < kMaxCols; ++p) {
    const int d = c0 + p * kT + tid;
    if (p * kT + tid >= span) break;
#pragma unroll
    for (int s = 0; s < S; ++s) x[p][s] = bf2f(xr[s * a.D + d]);
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
        for (int j = 0; j < S; ++j) m += a.comb[(r * S + j) * S + s] * x[p][j];
        nx[s] = round_bf16(a.post[r * S + s] * b + m);
      }
#pragma unroll
      for (int s = 0; s < S; ++s) { x[p][s] = nx[s]; xr[s * a.D + d] = f2bf(nx[s]); }
    }
#pragma unroll
    for (int i = 0; i < NM; ++i) {
      float u = 0.f;
#pragma unroll
      for (int s = 0; s < S; ++s) u += bf2f(a.fn[(int64_t)i * S * a.D + s * a.D + d]) * x[p][s];
      t[i] += u;
    }
#pragma unroll
    for (int s = 0; s < S; ++s) t[NM] += x[p][s] * x[p][s];
  }
  // CTA sums in fixed order: warp trees, then warps in order
#pragma unroll
  for (int i = 0; i <= NM; ++i) {
    const float w = warp_sum(t[i]);
    if (lane == 0 && warp < kT / 32) wred[warp][i] = w;     // the extra warp holds no columns
  }
  __syncthreads();
  if (tid <= NM) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kT / 32; ++w) s += wred[w][tid];
    part[tid] = s;
  }
  cl.sync();                            // (1) every CTA's dot partials are visible
  // Every CTA forms the row totals itself (cluster_total adds the 8 partials in rank order: the same bits in every
  // CTA) and its pre weights, so the norm below waits for no other CTA's result.  The post weights and the Sinkhorn
  // mixing matrix are read only by the next block's mHC: rank 0's extra warp computes them while the column warps
  // run the norm, arriving at the next cluster barrier before its 20 iterations and waiting after them.
  if (warp == 0 || (warp == kT / 32 && q == 0)) {
    const float mix = lane <= NM ? cluster_total(cl, part, lane) : 0.f;
    const float sumsq = __shfl_sync(0xffffffffu, mix, NM);
    const float rinv = rsqrtf(sumsq / (float)(S * a.D) + a.eps);
    if (warp == 0) {
      const float m_pre = __shfl_sync(0xffffffffu, mix, lane < S ? lane : 0);
      if (lane < S) pre_s[lane] = sigmoidf_(m_pre * rinv * a.hscale[0] + a.base[lane]) + a.hc_eps;
    } else {
      const float m_post = __shfl_sync(0xffffffffu, mix, lane < S ? S + lane : 0);
      if (lane < S) a.post_out[r * S + lane] = 2.f * sigmoidf_(m_post * rinv * a.hscale[1] + a.base[S + lane]);
      const int li = lane < S * S ? lane : 0;
      const float m_c = __shfl_sync(0xffffffffu, mix, 2 * S + li);
      cluster_arrive();                 // (2) this warp's arrival: it reads no norm partial
      float c = m_c * rinv * a.hscale[2] + a.base[2 * S + li];
      const float mx = row_max<S>(c);
      c = __expf(c - mx);
      c = c / row_sum<S>(c) + a.hc_eps;
      for (int it = 0; it < a.iters; ++it) {
        if (it > 0) c = c / (row_sum<S>(c) + a.hc_eps);
        c = c / (col_sum<S>(c) + a.hc_eps);
      }
      if (lane < S * S) a.comb_out[r * S * S + lane] = c;
      cluster_wait();
    }
  }
  if (warp < kT / 32) {
    named_sync(1, kT);                  // pre_s of this CTA is visible to its column warps
    float pre[S];
#pragma unroll
    for (int s = 0; s < S; ++s) pre[s] = pre_s[s];
    // collapsed stream and its sum of squares
    float col[kMaxCols];
    float ss = 0.f;
#pragma unroll
    for (int p = 0; p < kMaxCols; ++p) {
      if (p * kT + tid >= span) break;
      float u = 0.f;
#pragma unroll
      for (int s = 0; s < S; ++s) u += pre[s] * x[p][s];
      col[p] = round_bf16(u);
      ss += col[p] * col[p];
    }
    ss = warp_sum(ss);
    if (lane == 0) wred[warp][0] = ss;
    named_sync(1, kT);
    if (tid == 0) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kT / 32; ++w) s += wred[w][0];
      part2[0] = s;
    }
    cl.sync();                          // (2) every CTA's norm partial is visible
    const float tot = cluster_total(cl, part2, 0);
    const float rinv = rsqrtf(tot / (float)a.D + a.eps);
#pragma unroll
    for (int p = 0; p < kMaxCols; ++p) {
      const int d = c0 + p * kT + tid;
      if (p * kT + tid >= span) break;
      a.normed[(int64_t)r * a.D + d] = f2bf(col[p] * rinv * bf2f(a.norm_w[d]));
    }
    if (a.gath) {
      // the last CTA marks this parity's receive buffer consumed (every CTA read the epoch before counting in)
      named_sync(1, kT);
      if (tid == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(a.done, 1u);
        if (prev == gridDim.x * gridDim.y - 1) {
          *a.done = 0u;
          __threadfence();
          atomicAdd(a.epoch, 1u);
        }
      }
    }
  } else if (q != 0) {
    cl.sync();                          // (2) the extra warp of ranks 1..7 has nothing to compute
  }
  cl.sync();                            // (3) no CTA leaves while a peer may still read its shared memory
}

}  // namespace hd
}  // namespace g53

bool g53_hc_decode_ok(const HcArgs& a) {
  return a.fn != nullptr && a.R >= 1 && a.R <= 16 && (a.S == 2 || a.S == 4) && a.D % (g53::hd::kCl * 8) == 0 &&
         a.D <= g53::hd::kCl * g53::hd::kT * g53::hd::kMaxCols;
}

cudaError_t g53_hc_decode(const HcArgs& a, cudaStream_t st) {
  if (!g53_hc_decode_ok(a)) return cudaErrorInvalidValue;
  dim3 grid(g53::hd::kCl, a.R);
  // kT column threads plus one warp for rank 0's post / Sinkhorn, which overlaps the norm
  if (a.S == 4) return g53_launch_pdl(g53::hd::hc_decode_kernel<4>, grid, dim3(g53::hd::kT + 32), 0, st, 1, a);
  return g53_launch_pdl(g53::hd::hc_decode_kernel<2>, grid, dim3(g53::hd::kT + 32), 0, st, 1, a);
}
