// Kimi delta attention (KDA): causal depthwise conv, the recurrent delta-rule step, the gated output norm.
//
// Recurrence per head (state S[v][k], fp32), for each row t in order (code/fork/glm53_kda_lazy.py:160-178):
//   q, k <- l2-normalised (q * Dh^-1/2); g = lower * sigmoid(exp(A_log) * (f + dt_bias)); S <- S * exp(g)[k]
//   v' = sigmoid(b) * (v - S k); S <- S + v' k^T; o = S q
// Window design for speculative verification: the kernel reads the committed state S_in and writes the state
// after its last row to S_out (the other buffer of a double buffer) and never writes S_in, so a verify window of
// R rows needs no per-row state stores; committing fewer rows (keep < R) re-runs the kernel on the first `keep`
// rows (their conv outputs stay in the layer's qkv scratch) into S_out.  This is the reference's "lazy commit"
// (code/fork/glm53_kda_lazy.py:1-30) built into the kernel contract.
//
// Mapping: CTA = (head, 32 value rows); thread (vr, kq) owns S[vr][kq*Dh/4 .. +Dh/4); dot products over k are
// reduced over the 4 threads of a row group.
#include "common.cuh"
#include "launchers.h"

namespace g53 {

constexpr int kConvRB = 64;   // rows per conv thread

// grid (channel blocks, row blocks, sequences)
__global__ void kda_conv_kernel(KdaArgs a) {
  const int C = 3 * a.H * a.Dh;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.z;
  if (c >= C) return;
  const int base = a.row0[b], n = a.nrows[b];
  const int t0 = blockIdx.y * kConvRB;
  if (t0 >= n) return;
  const int t1 = min(t0 + kConvRB, n);
  const int T = a.taps;   // <= 8
  const __nv_bfloat16* win = a.conv_pool + (int64_t)a.conv_slot[b] * (T - 1) * C;
  float w[8], hist[8];
  for (int i = 0; i < T; ++i) w[i] = a.conv_w[(int64_t)c * T + i];
  for (int i = 0; i < T - 1; ++i) {
    const int t = t0 - (T - 1) + i;
    hist[i] = t < 0 ? bf2f(win[(int64_t)(T - 1 + t) * C + c]) : bf2f(a.proj[(int64_t)(base + t) * a.ldp + c]);
  }
  for (int t = t0; t < t1; ++t) {
    hist[T - 1] = bf2f(a.proj[(int64_t)(base + t) * a.ldp + c]);
    float s = 0.f;
    for (int i = 0; i < T; ++i) s += w[i] * hist[i];
    a.qkv[(int64_t)(base + t) * C + c] = f2bf(siluf_(s));
    for (int i = 0; i < T - 1; ++i) hist[i] = hist[i + 1];
  }
}

// grid (channel blocks, sequences): window <- last taps-1 rows of [window ; proj rows 0..nrows-1]
__global__ void kda_conv_commit_kernel(KdaArgs a) {
  const int C = 3 * a.H * a.Dh;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.y;
  if (c >= C) return;
  const int T = a.taps;
  const int base = a.row0[b], keep = a.nrows[b];
  __nv_bfloat16* win = a.conv_pool + (int64_t)a.conv_slot[b] * (T - 1) * C;
  float rows[8];
  for (int i = 0; i < T - 1; ++i) {
    const int idx = keep + i;
    rows[i] = idx < T - 1 ? bf2f(win[(int64_t)idx * C + c]) : bf2f(a.proj[(int64_t)(base + idx - (T - 1)) * a.ldp + c]);
  }
  for (int i = 0; i < T - 1; ++i) win[(int64_t)i * C + c] = f2bf(rows[i]);
}

// grid (H, Dh/32, sequences)
template <int DH>
__global__ void __launch_bounds__(128) kda_recurrent_kernel(KdaArgs a) {
  constexpr int KP = DH / 4;
  const int h = blockIdx.x, b = blockIdx.z;
  const int vr = threadIdx.x >> 2, kq = threadIdx.x & 3;
  const int v = blockIdx.y * 32 + vr;
  const int k0 = kq * KP;
  const int HD = a.H * DH;
  const int base = a.row0[b], n = a.nrows[b];
  const int64_t sstride = (int64_t)a.H * DH * DH;
  float S[KP];
  const float* sin = a.S_pool + a.s_in[b] * sstride + ((int64_t)h * DH + v) * DH + k0;
#pragma unroll
  for (int j = 0; j < KP; j += 4) {
    const float4 t = *reinterpret_cast<const float4*>(sin + j);
    S[j] = t.x; S[j + 1] = t.y; S[j + 2] = t.z; S[j + 3] = t.w;
  }
  const float ea = __expf(a.a_log[h]);
  float dtb[KP];
#pragma unroll
  for (int j = 0; j < KP; ++j) dtb[j] = a.dt_bias[h * DH + k0 + j];
  for (int tt = 0; tt < n; ++tt) {
    const int t = base + tt;
    const __nv_bfloat16* row = a.qkv + (int64_t)t * 3 * HD;
    float q[KP], k[KP];
    float sq = 0.f, sk = 0.f;
#pragma unroll
    for (int j = 0; j < KP; ++j) {
      q[j] = bf2f(row[h * DH + k0 + j]);
      k[j] = bf2f(row[HD + h * DH + k0 + j]);
      sq += q[j] * q[j];
      sk += k[j] * k[j];
    }
    sq = group_sum<4>(sq);
    sk = group_sum<4>(sk);
    const float qn = rsqrtf(sq + 1e-6f) * rsqrtf((float)DH);
    const float kn = rsqrtf(sk + 1e-6f);
    const float vv = bf2f(row[2 * HD + h * DH + v]);
    const float beta = sigmoidf_(bf2f(a.proj[(int64_t)t * a.ldp + a.b_off + h]));
    const __nv_bfloat16* fr = a.f + (int64_t)t * HD + h * DH + k0;
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < KP; ++j) {
      const float g = a.lower * sigmoidf_(ea * (bf2f(fr[j]) + dtb[j]));
      S[j] *= __expf(g);
      k[j] *= kn;
      q[j] *= qn;
      dot += S[j] * k[j];
    }
    dot = group_sum<4>(dot);
    const float vn = beta * (vv - dot);
    float o = 0.f;
#pragma unroll
    for (int j = 0; j < KP; ++j) {
      S[j] += vn * k[j];
      o += S[j] * q[j];
    }
    o = group_sum<4>(o);
    if (a.o_raw && kq == 0) a.o_raw[(int64_t)t * HD + h * DH + v] = o;
  }
  float* sout = a.S_pool + a.s_out[b] * sstride + ((int64_t)h * DH + v) * DH + k0;
#pragma unroll
  for (int j = 0; j < KP; j += 4) *reinterpret_cast<float4*>(sout + j) = make_float4(S[j], S[j + 1], S[j + 2], S[j + 3]);
}

// one warp per (row, head)
__global__ void kda_gated_norm_kernel(KdaArgs a) {
  const int lane = threadIdx.x & 31;
  const int idx = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (idx >= a.R * a.H) return;
  const int t = idx / a.H, h = idx % a.H;
  const int HD = a.H * a.Dh;
  const float* o = a.o_raw + (int64_t)t * HD + h * a.Dh;
  float ss = 0.f;
  for (int i = lane; i < a.Dh; i += 32) ss += o[i] * o[i];
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)a.Dh + a.eps);
  const __nv_bfloat16* gt = a.gate + (int64_t)t * HD + h * a.Dh;
  for (int i = lane; i < a.Dh; i += 32)
    a.out[(int64_t)t * HD + h * a.Dh + i] = f2bf(o[i] * r * bf2f(a.o_norm[i]) * sigmoidf_(bf2f(gt[i])));
}

}  // namespace g53

using namespace g53;

cudaError_t g53_kda_conv(const KdaArgs& a, cudaStream_t st) {
  if (a.taps > 8 || a.taps < 2) return cudaErrorInvalidValue;
  const int C = 3 * a.H * a.Dh;
  dim3 grid((C + 255) / 256, (a.max_rows + kConvRB - 1) / kConvRB, a.B);
  kda_conv_kernel<<<grid, 256, 0, st>>>(a);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}

cudaError_t g53_kda_conv_commit(const KdaArgs& a, cudaStream_t st) {
  if (a.taps > 8 || a.taps < 2) return cudaErrorInvalidValue;
  const int C = 3 * a.H * a.Dh;
  dim3 grid((C + 255) / 256, a.B);
  kda_conv_commit_kernel<<<grid, 256, 0, st>>>(a);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}

cudaError_t g53_kda_recurrent(const KdaArgs& a, cudaStream_t st) {
  dim3 grid(a.H, a.Dh / 32, a.B);
  if (a.Dh == 128) kda_recurrent_kernel<128><<<grid, 128, 0, st>>>(a);
  else if (a.Dh == 64) kda_recurrent_kernel<64><<<grid, 128, 0, st>>>(a);
  else return cudaErrorInvalidValue;
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}

cudaError_t g53_kda_gated_norm(const KdaArgs& a, cudaStream_t st) {
  const int warps = a.R * a.H;
  kda_gated_norm_kernel<<<(warps + 7) / 8, 256, 0, st>>>(a);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}

// ---------------------------------------------------------------------------------------------------------------
// Chunked KDA for prefill (same contract as kda_recurrent: reads S_pool[s_in], writes S_pool[s_out] and o_raw).
//
// Within a chunk of C rows starting from state S0 (G_t = cumulative log-decay, g <= 0 per channel):
//   S_t = S0 diag(e^{G_t}) + sum_{s<=t} v'_s (k_s * e^{G_t - G_s})^T
//   v'_t = beta_t (v_t - S0 (k_t e^{G_t}) - sum_{s<t} M_ts v'_s),  M_ts = sum_c k_t k_s e^{G_t - G_s}
//   o_t  = S0 (q_t e^{G_t}) + sum_{s<=t} P_ts v'_s,                  P_ts = sum_c q_t k_s e^{G_t - G_s}
//   S_C  = S0 diag(e^{G_C}) + sum_s v'_s (k_s e^{G_C - G_s})^T
// M and P use a reference row r (start of t's 16-row sub-chunk): e^{G_t - G_s} = e^{G_t - G_r} e^{G_r - G_s}, so
// both factors are bounded (|g| <= |lower| per step keeps e^{G_r - G_s} <= e^{15 |lower|}) and each inner product
// is a plain dot product of pre-scaled rows.  v' comes from forward substitution over the chunk.
// CTA = (head, 32 value rows, sequence); thread (vr, kc) keeps S[vr][kc + 8j] (j < DH/8) in registers (strided
// channels: the 8 kc threads of a row read 8 consecutive shared-memory words, no bank conflicts).  The CTAs of
// one head form a thread-block cluster: M and P do not depend on the value rows, so CTA rank j computes the rows
// of sub-chunk j (j, j+4, ... for fewer CTAs) and every CTA gathers the others' rows over distributed shared
// memory.
// ---------------------------------------------------------------------------------------------------------------
#include <cooperative_groups.h>
namespace cg = cooperative_groups;

namespace g53 {

constexpr int kCh = 64;      // chunk rows
constexpr int kSub = 16;     // sub-chunk rows (reference points)

template <int DH>
__global__ void __launch_bounds__(256, 1) kda_chunk_kernel(KdaArgs a) {
  constexpr int KPT = DH / 8;                 // state channels per thread
  constexpr int P1 = DH + 1;
  extern __shared__ float sm[];
  float* sK = sm;                             // [kCh][P1] normalised keys      (later: k * e^{G})
  float* sQ = sK + kCh * P1;                  // [kCh][P1] normalised, scaled queries (later: q * e^{G})
  float* sG = sQ + kCh * P1;                  // [kCh][P1] cumulative log-decay
  float* sX = sG + kCh * P1;                  // [kCh][P1] scratch: B~ rows, then k * e^{G_C - G_s}
  float* sA = sX + kCh * P1;                  // [kSub][P1] A~ (keys of the sub-chunk, ref-scaled)
  float* sQt = sA + kSub * P1;                // [kSub][P1] Q~
  float* sM = sQt + kSub * P1;                // [kCh][kCh+1]
  float* sP = sM + kCh * (kCh + 1);           // [kCh][kCh+1]
  float* sU = sP + kCh * (kCh + 1);           // [kCh][33] u_t then v'_t (this CTA's 32 value rows)
  float* sB = sU + kCh * 33;                  // [kCh] beta
  float* sV = sB + kCh;                       // [kCh][33] raw v

  const int h = blockIdx.x, b = blockIdx.z;
  const int v0 = blockIdx.y * 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int vr = tid >> 3, kc = tid & 7;
  const int HD = a.H * DH;
  const int base = a.row0[b], n_all = a.nrows[b];
  const int64_t sstride = (int64_t)a.H * DH * DH;
  const float ea = __expf(a.a_log[h]);

  float S[KPT];
  {
    const float* sin = a.S_pool + a.s_in[b] * sstride + ((int64_t)h * DH + v0 + vr) * DH + kc;
#pragma unroll
    for (int j = 0; j < KPT; ++j) S[j] = sin[8 * j];
  }

  for (int c0 = 0; c0 < n_all; c0 += kCh) {
    const int n = min(kCh, n_all - c0);
    // 1. rows: normalised q, k; raw g; beta; v of this CTA's rows
    for (int t = warp; t < kCh; t += 8) {
      const int row = base + c0 + t;
      constexpr int PL = DH / 32;
      float q[PL], k[PL], g[PL];
      float sq = 0.f, sk = 0.f;
#pragma unroll
      for (int i = 0; i < PL; ++i) {
        const int c = lane + 32 * i;
        if (t < n) {
          const __nv_bfloat16* rp = a.qkv + (int64_t)row * 3 * HD;
          q[i] = bf2f(rp[h * DH + c]);
          k[i] = bf2f(rp[HD + h * DH + c]);
          g[i] = a.lower * sigmoidf_(ea * (bf2f(a.f[(int64_t)row * HD + h * DH + c]) + a.dt_bias[h * DH + c]));
        } else {
          q[i] = k[i] = g[i] = 0.f;
        }
        sq += q[i] * q[i];
        sk += k[i] * k[i];
      }
      sq = warp_sum(sq);
      sk = warp_sum(sk);
      const float qn = rsqrtf(sq + 1e-6f) * rsqrtf((float)DH), kn = rsqrtf(sk + 1e-6f);
#pragma unroll
      for (int i = 0; i < PL; ++i) {
        const int c = lane + 32 * i;
        sQ[t * P1 + c] = q[i] * qn;
        sK[t * P1 + c] = k[i] * kn;
        sG[t * P1 + c] = g[i];
      }
      if (lane == 0) sB[t] = t < n ? sigmoidf_(bf2f(a.proj[(int64_t)row * a.ldp + a.b_off + h])) : 0.f;
      if (t < n) sV[t * 33 + lane] = bf2f(a.qkv[(int64_t)row * 3 * HD + 2 * HD + h * DH + v0 + lane]);
      else sV[t * 33 + lane] = 0.f;
    }
    __syncthreads();
    // 2. cumulative log-decay per channel (rows past n keep the last value)
    for (int c = tid; c < DH; c += blockDim.x) {
      float acc = 0.f;
      for (int t = 0; t < kCh; ++t) {
        acc += sG[t * P1 + c];
        sG[t * P1 + c] = acc;
      }
    }
    __syncthreads();
    // 3. M (strictly lower) and P (lower incl. diagonal) for this CTA's 16-row sub-chunks of t; every thread a
    //    strip of 4 s columns of one row t
    cg::cluster_group cluster = cg::this_cluster();
    const int crank = (int)cluster.block_rank(), csize = (int)cluster.num_blocks();
    for (int j = crank; j < kCh / kSub; j += csize) {
      const int r = j * kSub;
      const int ns = r + kSub;                          // s ranges over [0, ns)
      for (int e = tid; e < kSub * DH; e += blockDim.x) {
        const int t = e / DH, c = e % DH;
        const float f = __expf(sG[(r + t) * P1 + c] - sG[r * P1 + c]);
        sA[t * P1 + c] = sK[(r + t) * P1 + c] * f;
        sQt[t * P1 + c] = sQ[(r + t) * P1 + c] * f;
      }
      for (int e = tid; e < ns * DH; e += blockDim.x) {
        const int s = e / DH, c = e % DH;
        sX[s * P1 + c] = sK[s * P1 + c] * __expf(sG[r * P1 + c] - sG[s * P1 + c]);
      }
      __syncthreads();
      const int strips = ns / 4;
      for (int e = tid; e < kSub * strips; e += blockDim.x) {
        const int t = e / strips, s0 = (e % strips) * 4;
        const int tt = r + t;
        float m[4] = {0.f, 0.f, 0.f, 0.f}, pp[4] = {0.f, 0.f, 0.f, 0.f};
        if (s0 <= tt) {
#pragma unroll 4
          for (int c = 0; c < DH; ++c) {
            const float av = sA[t * P1 + c], qv = sQt[t * P1 + c];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float bs = sX[(s0 + i) * P1 + c];
              m[i] += av * bs;
              pp[i] += qv * bs;
            }
          }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int s = s0 + i;
          sM[tt * (kCh + 1) + s] = s < tt ? m[i] : 0.f;
          sP[tt * (kCh + 1) + s] = s <= tt ? pp[i] : 0.f;
        }
      }
      __syncthreads();
    }
    // gather the other CTAs' sub-chunk rows of M and P
    cluster.sync();
    for (int j = 0; j < kCh / kSub; ++j) {
      const int owner = j % csize;
      if (owner == crank) continue;
      const float* rM = cluster.map_shared_rank(sM, owner);
      const float* rP = cluster.map_shared_rank(sP, owner);
      for (int e = tid; e < kSub * (kCh + 1); e += blockDim.x) {
        const int idx = j * kSub * (kCh + 1) + e;
        sM[idx] = rM[idx];
        sP[idx] = rP[idx];
      }
    }
    cluster.sync();
    // 4. scaled rows for the chunk-start state: K e^{G}, Q e^{G}; and k_s e^{G_C - G_s} for the state update
    const int last = n - 1;
    for (int e = tid; e < kCh * DH; e += blockDim.x) {
      const int t = e / DH, c = e % DH;
      const float G = sG[t * P1 + c];
      sX[t * P1 + c] = t < n ? sK[t * P1 + c] * __expf(sG[last * P1 + c] - G) : 0.f;
      const float d = __expf(G);
      sK[t * P1 + c] *= d;
      sQ[t * P1 + c] *= d;
    }
    __syncthreads();
    // 5. u_t = v_t - S0 Ke_t and o0_t = S0 Qe_t  (row vr, partial over this thread's channels, reduced over kc)
    for (int t = 0; t < kCh; ++t) {
      float du = 0.f, dq = 0.f;
#pragma unroll
      for (int j = 0; j < KPT; ++j) {
        du += S[j] * sK[t * P1 + kc + 8 * j];
        dq += S[j] * sQ[t * P1 + kc + 8 * j];
      }
      du = group_sum<8>(du);
      dq = group_sum<8>(dq);
      if (kc == 0) {
        sU[t * 33 + vr] = sV[t * 33 + vr] - du;
        sV[t * 33 + vr] = dq;                          // reuse: o0_t for row vr
      }
    }
    __syncthreads();
    // 6. forward substitution: v'_t = beta_t (u_t - sum_{s<t} M_ts v'_s); thread (vr, kc) sums s = kc (mod 8)
    for (int t = 0; t < n; ++t) {
      float acc = 0.f;
      for (int s = kc; s < t; s += 8) acc += sM[t * (kCh + 1) + s] * sU[s * 33 + vr];
      acc = group_sum<8>(acc);
      if (kc == 0) sU[t * 33 + vr] = sB[t] * (sU[t * 33 + vr] - acc);
      __syncthreads();
    }
    // 7. outputs o_t = o0_t + sum_{s<=t} P_ts v'_s
    for (int t = 0; t < n; ++t) {
      float acc = 0.f;
      for (int s = kc; s <= t; s += 8) acc += sP[t * (kCh + 1) + s] * sU[s * 33 + vr];
      acc = group_sum<8>(acc);
      if (kc == 0) a.o_raw[(int64_t)(base + c0 + t) * HD + h * DH + v0 + vr] = sV[t * 33 + vr] + acc;
    }
    // 8. state: S <- S diag(e^{G_C}) + sum_s v'_s (k_s e^{G_C - G_s})^T
#pragma unroll
    for (int j = 0; j < KPT; ++j) {
      const int c = kc + 8 * j;
      float acc = S[j] * __expf(sG[last * P1 + c]);
      for (int s = 0; s < n; ++s) acc += sU[s * 33 + vr] * sX[s * P1 + c];
      S[j] = acc;
    }
    __syncthreads();
  }
  float* sout = a.S_pool + a.s_out[b] * sstride + ((int64_t)h * DH + v0 + vr) * DH + kc;
#pragma unroll
  for (int j = 0; j < KPT; ++j) sout[8 * j] = S[j];
}

}  // namespace g53

cudaError_t g53_kda_chunk(const KdaArgs& a, cudaStream_t st) {
  using namespace g53;
  const int DH = a.Dh;
  const int P1 = DH + 1;
  const size_t smem = sizeof(float) * ((size_t)4 * kCh * P1 + 2 * kSub * P1 + 2 * kCh * (kCh + 1) + kCh * 33 +
                                       kCh + kCh * 33);
  dim3 grid(a.H, DH / 32, a.B);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = DH / 32;               // the value blocks of one head
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  if (DH == 128) {
    e = cudaFuncSetAttribute(kda_chunk_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    e = cudaLaunchKernelEx(&cfg, kda_chunk_kernel<128>, a);
  } else if (DH == 64) {
    e = cudaFuncSetAttribute(kda_chunk_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    e = cudaLaunchKernelEx(&cfg, kda_chunk_kernel<64>, a);
  } else {
    return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}
