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
// Mapping: CTA = (head, 32 value rows); thread (vr, kq) owns S[vr][kq + 4j] (j < Dh/4); dot products over k are
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
  if (c >= C || !g53_in_bounds(a.conv_slot[b], a.n_conv, 5)) return;
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

// vectorised form for a compile-time tap count: a thread owns 8 consecutive channels (16-byte loads and stores)
// of kConvRB consecutive rows; the taps and the history stay in registers
template <int T>
__global__ void __launch_bounds__(256) kda_conv_vec_kernel(KdaArgs a) {
  pdl_trigger();                       // dependents (the next projection) may start prefetching
  const int C = 3 * a.H * a.Dh;
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  const int b = blockIdx.z;
  if (c >= C || !g53_in_bounds(a.conv_slot[b], a.n_conv, 5)) return;
  const int base = a.row0[b], n = a.nrows[b];
  const int t0 = blockIdx.y * kConvRB;
  if (t0 >= n) return;
  const int t1 = min(t0 + kConvRB, n);
  const __nv_bfloat16* win = a.conv_pool + (int64_t)a.conv_slot[b] * (T - 1) * C;
  float w[T][8], hist[T][8];
#pragma unroll
  for (int e = 0; e < 8; ++e)
#pragma unroll
    for (int i = 0; i < T; ++i) w[i][e] = a.conv_w[(int64_t)(c + e) * T + i];
  auto load8 = [&](const __nv_bfloat16* p, float (&o)[8]) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    const uint32_t ws[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      o[2 * e] = __uint_as_float(ws[e] << 16);
      o[2 * e + 1] = __uint_as_float(ws[e] & 0xffff0000u);
    }
  };
#pragma unroll
  for (int i = 0; i < T - 1; ++i) {
    const int t = t0 - (T - 1) + i;
    load8(t < 0 ? win + (int64_t)(T - 1 + t) * C + c : a.proj + (int64_t)(base + t) * a.ldp + c, hist[i]);
  }
  // rows in groups of kGrp: the group's loads are issued together (read-only path) before any of its rows is
  // convolved, so a thread keeps kGrp 16-byte loads in flight instead of one
  constexpr int kGrp = 4;
  for (int tg = t0; tg < t1; tg += kGrp) {
    uint4 raw[kGrp];
#pragma unroll
    for (int j = 0; j < kGrp; ++j)
      raw[j] = tg + j < t1 ? ldg_nc_v4(a.proj + (int64_t)(base + tg + j) * a.ldp + c) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int j = 0; j < kGrp; ++j) {
      const int t = tg + j;
      if (t >= t1) break;
      const uint32_t ws[4] = {raw[j].x, raw[j].y, raw[j].z, raw[j].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        hist[T - 1][2 * e] = __uint_as_float(ws[e] << 16);
        hist[T - 1][2 * e + 1] = __uint_as_float(ws[e] & 0xffff0000u);
      }
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int i = 0; i < T; ++i) { s0 += w[i][e] * hist[i][e]; s1 += w[i][e + 1] * hist[i][e + 1]; }
        __nv_bfloat162 p2 = __floats2bfloat162_rn(siluf_(s0), siluf_(s1));
        o[e >> 1] = *reinterpret_cast<uint32_t*>(&p2);
      }
      *reinterpret_cast<uint4*>(a.qkv + (int64_t)(base + t) * C + c) = make_uint4(o[0], o[1], o[2], o[3]);
#pragma unroll
      for (int i = 0; i < T - 1; ++i)
#pragma unroll
        for (int e = 0; e < 8; ++e) hist[i][e] = hist[i + 1][e];
    }
  }
}

// grid (channel blocks, sequences): window <- last taps-1 rows of [window ; proj rows 0..nrows-1]
__global__ void kda_conv_commit_kernel(KdaArgs a) {
  const int C = 3 * a.H * a.Dh;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.y;
  if (c >= C || !g53_in_bounds(a.conv_slot[b], a.n_conv, 5)) return;
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

// grid (H, Dh/32, sequences).  Rows are staged 8 at a time in shared memory (normalised q, k, the decay g,
// this CTA's 32 values of v, beta) by all 128 threads with coalesced loads, so the sequential recurrence only reads
// shared memory; the state stays in registers.
constexpr int kRecRows = 8;
template <int DH>
__global__ void __launch_bounds__(128) kda_recurrent_kernel(KdaArgs a) {
  pdl_trigger();                       // dependents (the next projection) may start prefetching
  constexpr int KP = DH / 4;
  __shared__ float sq[kRecRows][DH], sk[kRecRows][DH], sg[kRecRows][DH], sv[kRecRows][32], sb[kRecRows];
  const int h = blockIdx.x, b = blockIdx.z;
  if (!g53_in_bounds(a.s_in[b], a.n_states, 5) || !g53_in_bounds(a.s_out[b], a.n_states, 5)) return;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int vr = tid >> 2, kq = tid & 3;
  const int v0 = blockIdx.y * 32, v = v0 + vr;
  // thread (vr, kq) owns state channels kq + 4 j (interleaved: the 4 threads of a row read 4 banks)
  const int HD = a.H * DH;
  const int base = a.row0[b], n = a.nrows[b];
  const int64_t sstride = (int64_t)a.H * DH * DH;
  float S[KP];
  const float* sin = a.S_pool + a.s_in[b] * sstride + ((int64_t)h * DH + v) * DH + kq;
#pragma unroll
  for (int j = 0; j < KP; ++j) S[j] = sin[4 * j];
  const float ea = __expf(a.a_log[h]);
  for (int r0 = 0; r0 < n; r0 += kRecRows) {
    const int nr = min(kRecRows, n - r0);
    // stage: warp w normalises rows w, w + 4 (q and k: one row per warp, DH/32 elements per lane)
    for (int rr = warp; rr < nr; rr += 4) {
      const int t = base + r0 + rr;
      const __nv_bfloat16* row = a.qkv + (int64_t)t * 3 * HD;
      constexpr int PL = DH / 32;
      float q[PL], k[PL];
      float qq = 0.f, kk = 0.f;
#pragma unroll
      for (int i = 0; i < PL; ++i) {
        const int c = lane + 32 * i;
        q[i] = bf2f(row[h * DH + c]);
        k[i] = bf2f(row[HD + h * DH + c]);
        qq += q[i] * q[i];
        kk += k[i] * k[i];
        sg[rr][c] = a.lower * sigmoidf_(ea * (bf2f(a.f[(int64_t)t * HD + h * DH + c]) + a.dt_bias[h * DH + c]));
      }
      qq = warp_sum(qq);
      kk = warp_sum(kk);
      const float qn = rsqrtf(qq + 1e-6f) * rsqrtf((float)DH), kn = rsqrtf(kk + 1e-6f);
#pragma unroll
      for (int i = 0; i < PL; ++i) {
        sq[rr][lane + 32 * i] = q[i] * qn;
        sk[rr][lane + 32 * i] = k[i] * kn;
      }
      sv[rr][lane] = bf2f(row[2 * HD + h * DH + v0 + lane]);
      if (lane == 0) sb[rr] = sigmoidf_(bf2f(a.proj[(int64_t)t * a.ldp + a.b_off + h]));
    }
    __syncthreads();
    for (int rr = 0; rr < nr; ++rr) {
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < KP; ++j) {
        S[j] *= __expf(sg[rr][kq + 4 * j]);
        dot += S[j] * sk[rr][kq + 4 * j];
      }
      dot = group_sum<4>(dot);
      const float vn = sb[rr] * (sv[rr][vr] - dot);
      float o = 0.f;
#pragma unroll
      for (int j = 0; j < KP; ++j) {
        S[j] += vn * sk[rr][kq + 4 * j];
        o += S[j] * sq[rr][kq + 4 * j];
      }
      o = group_sum<4>(o);
      if (a.o_raw && kq == 0) a.o_raw[(int64_t)(base + r0 + rr) * HD + h * DH + v] = o;
    }
    __syncthreads();
  }
  float* sout = a.S_pool + a.s_out[b] * sstride + ((int64_t)h * DH + v) * DH + kq;
#pragma unroll
  for (int j = 0; j < KP; ++j) sout[4 * j] = S[j];
}

// one warp per (row, head)
__global__ void kda_gated_norm_kernel(KdaArgs a) {
  pdl_trigger();                       // dependents (the next projection) may start prefetching
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
  // 16-byte rows: the vectorised kernel (4 taps: the model's short convolution)
  if (a.taps == 4 && C % 8 == 0 && a.ldp % 8 == 0 && (reinterpret_cast<uintptr_t>(a.proj) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(a.qkv) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.conv_pool) & 15) == 0) {
    dim3 grid((C / 8 + 255) / 256, (a.max_rows + kConvRB - 1) / kConvRB, a.B);
    kda_conv_vec_kernel<4><<<grid, 256, 0, st>>>(a);
    G53_CHECK_LAUNCH();
    return cudaSuccess;
  }
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
