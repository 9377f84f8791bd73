// Sampling and speculative verification.
//
//   argmax_rows     per row (value, id) of the maximum logit (ties -> lower id), over this rank's vocabulary shard
//   greedy_verify   per request: accepted = length of the prefix of drafts that equal the target's greedy tokens;
//                   emitted tokens = accepted drafts + the target's token at the first mismatch (or the bonus row);
//                   `forced` accepts all K drafts (the fixed-acceptance benchmark mode)
//   rejection       probabilistic verification: standard (stop at the first rejection, resample from
//                   max(p - q, 0)) or block verification (Sun et al. 2024: the last row whose test passes wins);
//                   every draw is keyed by (seed, position, row) with a counter-based hash, and the residual resample
//                   uses a stream independent of the acceptance draws
//                   (reference behaviour: code/fork/docs/BLOCK_VERIFY.md:9-58,
//                    code/fork/overlay/patch_spec_resample_noise.py:2-33)
#include "common.cuh"
#include "launchers.h"

namespace g53 {

__global__ void __launch_bounds__(1024) argmax_rows_kernel(const float* logits, int V, int64_t ld, int vocab_offset,
                                                           float* best_val, int* best_id) {
  const int r = blockIdx.x;
  const float* row = logits + (int64_t)r * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = row[i];
    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) { sv[wid] = bv; si[wid] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
    best_val[r] = bv;
    best_id[r] = bi + vocab_offset;
  }
}

__global__ void greedy_verify_kernel(VerifyArgs a) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= a.B) return;
  const int* d = a.draft + (int64_t)b * a.K;
  const int* t = a.target_argmax + (int64_t)b * (a.K + 1);
  int n = 0;
  if (a.forced) {
    n = a.K;
  } else {
    while (n < a.K && d[n] == t[n]) ++n;
  }
  int* out = a.next_tokens + (int64_t)b * (a.K + 1);
  for (int i = 0; i < n; ++i) out[i] = d[i];
  out[n] = t[n];
  for (int i = n + 1; i <= a.K; ++i) out[i] = -1;
  a.accepted[b] = n;
}

// counter-based 64-bit hash (splitmix64 finaliser) -> uniform in [0, 1)
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__device__ __forceinline__ float uniform_key(uint64_t seed, int64_t pos, int row, int stream, int idx) {
  uint64_t h = mix64(seed ^ mix64((uint64_t)pos * 0x100000001B3ull + (uint64_t)row));
  h = mix64(h ^ ((uint64_t)stream << 40) ^ (uint64_t)(uint32_t)idx);
  return (float)(h >> 40) * (1.0f / 16777216.0f);
}

// one CTA per request; K <= 15
__global__ void __launch_bounds__(256) rejection_kernel(RejectArgs a) {
  const int b = blockIdx.x;
  const int K = a.K, V = a.V;
  const float* P = a.target_probs + (int64_t)b * (K + 1) * V;
  const float* Q = a.draft_probs + (int64_t)b * K * V;
  const int* d = a.draft + (int64_t)b * K;
  const int64_t pos0 = a.positions[b];
  __shared__ float ratio[16], hval[16], resid[16];
  __shared__ int acc_s;
  __shared__ float red[32];
  if (threadIdx.x < K) {
    const int i = threadIdx.x;
    const float p = P[(int64_t)i * V + d[i]], q = Q[(int64_t)i * V + d[i]];
    ratio[i] = q > 0.f ? p / q : (p > 0.f ? INFINITY : 0.f);
  }
  __syncthreads();
  // block verification: cumulative P_i = min(P_{i-1} * ratio_i, 1) and residual masses r_i
  if (a.block) {
    for (int i = 0; i < K; ++i) {
      // r_i = sum_x max(P_i * p_{i+1}(x) - q_{i+1}(x), 0) for i < K-1 (rows of the next position)
      float cum = 1.f;
      for (int j = 0; j <= i; ++j) cum = fminf(cum * ratio[j], 1.f);
      float rsum = 0.f;
      if (i < K - 1) {
        const float* pn = P + (int64_t)(i + 1) * V;
        const float* qn = Q + (int64_t)(i + 1) * V;
        for (int x = threadIdx.x; x < V; x += blockDim.x) rsum += fmaxf(cum * pn[x] - qn[x], 0.f);
        rsum = block_sum(rsum, red);
      }
      if (threadIdx.x == 0) {
        resid[i] = rsum;
        hval[i] = (i < K - 1) ? rsum / (rsum + 1.f - cum) : cum;
        if (!(hval[i] >= 0.f)) hval[i] = 0.f;
      }
      __syncthreads();
    }
    if (threadIdx.x == 0) {
      int n = 0;
      for (int i = 0; i < K; ++i)
        if (uniform_key(a.seed, pos0, i, 0, 0) <= hval[i]) n = i + 1;
      acc_s = n;
    }
  } else if (threadIdx.x == 0) {
    int n = 0;
    while (n < K && uniform_key(a.seed, pos0, n, 0, 0) < fminf(ratio[n], 1.f)) ++n;
    acc_s = n;
  }
  __syncthreads();
  const int n = acc_s;
  // resample row n: bonus (n == K) from p_K; otherwise residual
  const float* pr = P + (int64_t)n * V;
  const float* qr = n < K ? Q + (int64_t)n * V : nullptr;
  float cum = 1.f;
  if (a.block && n < K) for (int j = 0; j < n; ++j) cum = fminf(cum * ratio[j], 1.f);
  // Gumbel-max over the residual weights (independent stream 1)
  float bv = -INFINITY;
  int bi = 0;
  for (int x = threadIdx.x; x < V; x += blockDim.x) {
    float w = pr[x];
    if (qr) w = a.block ? fmaxf(cum * pr[x] - qr[x], 0.f) : fmaxf(pr[x] - qr[x], 0.f);
    if (w > 0.f) {
      const float u = fmaxf(uniform_key(a.seed, pos0, n, 1, x), 1e-12f);
      const float gsc = __logf(w) - __logf(-__logf(u));
      if (gsc > bv) { bv = gsc; bi = x; }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) { sv[wid] = bv; si[wid] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
    int* out = a.next_tokens + (int64_t)b * (K + 1);
    for (int i = 0; i < n; ++i) out[i] = d[i];
    out[n] = bi;
    for (int i = n + 1; i <= K; ++i) out[i] = -1;
    a.accepted[b] = n;
    if (a.scratch) for (int i = 0; i < K; ++i) a.scratch[(int64_t)b * (K + 1) + i] = hval[i];
  }
}

}  // namespace g53

using namespace g53;

cudaError_t g53_argmax_rows(const float* logits, int R, int V, int64_t ld, int vocab_offset, float* best_val,
                            int* best_id, cudaStream_t st) {
  argmax_rows_kernel<<<R, 1024, 0, st>>>(logits, V, ld, vocab_offset, best_val, best_id);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}

cudaError_t g53_greedy_verify(const VerifyArgs& a, cudaStream_t st) {
  greedy_verify_kernel<<<(a.B + 127) / 128, 128, 0, st>>>(a);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}

cudaError_t g53_rejection_sample(const RejectArgs& a, cudaStream_t st) {
  if (a.K > 15 || a.K < 1) return cudaErrorInvalidValue;
  rejection_kernel<<<a.B, 256, 0, st>>>(a);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}
