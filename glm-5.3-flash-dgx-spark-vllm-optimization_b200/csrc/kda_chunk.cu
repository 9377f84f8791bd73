// Chunked KDA for prefill in two kernels (same contract as kda_recurrent: reads S_pool[s_in], writes S_pool[s_out]
// and o_raw).  Per head, a chunk of C = 64 rows starting from state S0 (G_t = cumulative log-decay, g <= 0 per
// channel):
//   S_t  = S0 diag(e^{G_t}) + sum_{s<=t} v'_s (k_s e^{G_t - G_s})^T
//   v'   = T (V - K~ S0^T),   T = (I + diag(beta) M)^{-1} diag(beta),   M_ts = sum_c k_t k_s e^{G_t - G_s} (s < t)
//   o    = Q~ S0^T + P v',    P_ts = sum_c q_t k_s e^{G_t - G_s} (s <= t)
//   S_C  = S0 diag(e^{G_C}) + v'^T K^ ,   K~_t = k_t e^{G_t},  Q~_t = q_t e^{G_t},  K^_s = k_s e^{G_C - G_s}
//
// kda_prep_kernel   one CTA per (chunk, head, sequence), all chunks in parallel: normalised rows, cumulative
//                   decay, M and P (fp32, with 16-row sub-chunk reference points so every exponential factor stays
//                   bounded), the unit lower-triangular inverse by forward substitution, T, and the scaled rows
//                   Q~, K~, K^ and e^{G_C}; written to a per-(chunk, head) scratch.
// kda_scan_kernel   one CTA per (head, 32 value rows, sequence), sequential over the chunks: the four chunk
//                   products (K~ S0^T, T Z, Q~ S0^T + P v', v'^T K^) on the tensor cores (mma.sync m16n8k8 tf32,
//                   fp32 accumulate) with the state S kept in fp32 in shared memory.
// The state-independent work (about 60 % of the FLOPs and all of the triangular solve) leaves the sequential
// chain, which is what bounds a chunked scan on a GPU with 148 SMs and only 64 heads x 4 value blocks of work.
// Reference counterpart: FlashKDA chunked prefill (code/fork/overlay/glm53_flashkda.py:136), fp32 state.
#include "common.cuh"
#include "launchers.h"

namespace g53 {

constexpr int kC = 64;       // chunk rows
constexpr int kSubR = 16;    // sub-chunk rows (reference points)

__host__ __device__ constexpr int64_t kda_scr_per_head(int dh) { return 3LL * kC * dh + 2LL * kC * kC + dh; }

__device__ __forceinline__ int chunk_slot(int row0, int b, int c) { return row0 / kC + b + c; }

// ---------------------------------------------------------------------------------------------------------------
// prep: grid (max chunks, H, B), 256 threads
// ---------------------------------------------------------------------------------------------------------------
template <int DH>
__global__ void __launch_bounds__(256, 1) kda_prep_kernel(KdaArgs a) {
  constexpr int P1 = DH + 1;
  extern __shared__ float sm[];
  float* sK = sm;                       // [kC][P1] normalised k
  float* sQ = sK + kC * P1;             // [kC][P1] normalised, scaled q
  float* sG = sQ + kC * P1;             // [kC][P1] raw g, then cumulative G
  float* sX = sG + kC * P1;             // [kC][P1] scratch: k_s e^{G_r - G_s}, then K^
  float* sA = sX + kC * P1;             // [kSubR][P1] k_t e^{G_t - G_r}
  float* sQt = sA + kSubR * P1;         // [kSubR][P1] q_t e^{G_t - G_r}
  float* sM = sQt + kSubR * P1;         // [kC][kC+1]
  float* sP = sM + kC * (kC + 1);       // [kC][kC+1]
  float* sI = sP + kC * (kC + 1);       // [kC][kC+1] (I + diag(beta) M)^{-1}
  float* sB = sI + kC * (kC + 1);       // [kC] beta

  const int ci = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int base = a.row0[b], n_all = a.nrows[b];
  const int c0 = ci * kC;
  if (c0 >= n_all) return;
  const int n = min(kC, n_all - c0);
  const int slot = chunk_slot(base, b, ci);
  if (slot >= a.scr_slots) return;                 // the launcher sizes the scratch; never reached
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int HD = a.H * DH;
  const float ea = __expf(a.a_log[h]);

  // 1. rows: normalised q, k; raw g; beta
  for (int t = warp; t < kC; t += 8) {
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
  }
  __syncthreads();
  // 2. cumulative log-decay per channel (rows past n add 0 and keep the last value)
  for (int c = tid; c < DH; c += blockDim.x) {
    float acc = 0.f;
    for (int t = 0; t < kC; ++t) {
      acc += sG[t * P1 + c];
      sG[t * P1 + c] = acc;
    }
  }
  __syncthreads();
  // 3. M (strictly lower) and P (lower incl. diagonal), one 16-row sub-chunk of t at a time; reference row r
  for (int j = 0; j < kC / kSubR; ++j) {
    const int r = j * kSubR;
    const int ns = r + kSubR;                      // s ranges over [0, ns)
    for (int e = tid; e < kSubR * DH; e += blockDim.x) {
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
    for (int e = tid; e < kSubR * strips; e += blockDim.x) {
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
        sM[tt * (kC + 1) + s] = s < tt ? m[i] : 0.f;
        sP[tt * (kC + 1) + s] = s <= tt ? pp[i] : 0.f;
      }
    }
    __syncthreads();
  }
  // zero the upper parts of M and P (columns >= ns of each sub-chunk were not written)
  for (int e = tid; e < kC * kC; e += blockDim.x) {
    const int t = e / kC, s = e % kC;
    if (s >= (t / kSubR + 1) * kSubR) { sM[t * (kC + 1) + s] = 0.f; sP[t * (kC + 1) + s] = 0.f; }
  }
  __syncthreads();
  // 4. X = (I + diag(beta) M)^{-1}, unit lower triangular, by rows: X_t = e_t - beta_t sum_{s<t} M_ts X_s.
  //    4 threads per column j split the sum over s (fixed order, shuffle-reduced)
  {
    const int j = tid >> 2, part = tid & 3;
    for (int e = tid; e < kC * kC; e += blockDim.x) sI[(e / kC) * (kC + 1) + e % kC] = (e / kC == e % kC) ? 1.f : 0.f;
    __syncthreads();
    for (int t = 1; t < kC; ++t) {
      float acc = 0.f;
      if (j < t)
        for (int s = j + part; s < t; s += 4) acc += sM[t * (kC + 1) + s] * sI[s * (kC + 1) + j];
      acc = group_sum<4>(acc);
      if (j < t && part == 0) sI[t * (kC + 1) + j] = -sB[t] * acc;
      __syncthreads();
    }
  }
  // 5. scaled rows: Q~ = q e^{G}, K~ = k e^{G} (in place), K^ = k e^{G_C - G} (rows past n: 0)
  const int last = n - 1;
  for (int e = tid; e < kC * DH; e += blockDim.x) {
    const int t = e / DH, c = e % DH;
    const float G = sG[t * P1 + c];
    sX[t * P1 + c] = t < n ? sK[t * P1 + c] * __expf(sG[last * P1 + c] - G) : 0.f;
    const float d = __expf(G);
    sK[t * P1 + c] *= d;
    sQ[t * P1 + c] *= d;
  }
  __syncthreads();
  // 6. write the chunk record: Q~, K~, K^ [kC][DH], T = X diag(beta) [kC][kC], P [kC][kC], e^{G_C} [DH]
  float* out = a.scr + ((int64_t)slot * a.H + h) * kda_scr_per_head(DH);
  float* oQ = out;
  float* oK = oQ + kC * DH;
  float* oKb = oK + kC * DH;
  float* oT = oKb + kC * DH;
  float* oP = oT + kC * kC;
  float* oE = oP + kC * kC;
  for (int e = tid; e < kC * DH; e += blockDim.x) {
    const int t = e / DH, c = e % DH;
    oQ[e] = sQ[t * P1 + c];
    oK[e] = sK[t * P1 + c];
    oKb[e] = sX[t * P1 + c];
  }
  for (int e = tid; e < kC * kC; e += blockDim.x) {
    const int t = e / kC, s = e % kC;
    oT[e] = sI[t * (kC + 1) + s] * sB[s];
    oP[e] = sP[t * (kC + 1) + s];
  }
  for (int c = tid; c < DH; c += blockDim.x) oE[c] = __expf(sG[last * P1 + c]);
}

// ---------------------------------------------------------------------------------------------------------------
// scan: grid (H, DH/32, B), 256 threads (8 warps)
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// A fragment (16 x 8) of a row-major matrix: element (m, k) at p[m * ld + k]
__device__ __forceinline__ void frag_a_row(const float* p, int ld, uint32_t (&f)[4]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  f[0] = to_tf32(p[g * ld + q]);
  f[1] = to_tf32(p[(g + 8) * ld + q]);
  f[2] = to_tf32(p[g * ld + q + 4]);
  f[3] = to_tf32(p[(g + 8) * ld + q + 4]);
}
// A fragment of a transposed store: element (m, k) at p[k * ld + m]
__device__ __forceinline__ void frag_a_col(const float* p, int ld, uint32_t (&f)[4]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  f[0] = to_tf32(p[q * ld + g]);
  f[1] = to_tf32(p[q * ld + g + 8]);
  f[2] = to_tf32(p[(q + 4) * ld + g]);
  f[3] = to_tf32(p[(q + 4) * ld + g + 8]);
}
// B fragment (8 x 8) with element (k, n) at p[n * ld + k]
__device__ __forceinline__ void frag_b_nk(const float* p, int ld, uint32_t& b0, uint32_t& b1) {
  const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  b0 = to_tf32(p[g * ld + q]);
  b1 = to_tf32(p[g * ld + q + 4]);
}
// B fragment with element (k, n) at p[k * ld + n]
__device__ __forceinline__ void frag_b_kn(const float* p, int ld, uint32_t& b0, uint32_t& b1) {
  const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  b0 = to_tf32(p[q * ld + g]);
  b1 = to_tf32(p[(q + 4) * ld + g]);
}

template <int DH>
__global__ void __launch_bounds__(256, 1) kda_scan_kernel(KdaArgs a) {
  constexpr int LD = DH + 4;       // row pitch of the [kC][DH] and [32][DH] tiles (conflict-free fragments)
  constexpr int LT = kC + 4;       // row pitch of T and P
  constexpr int LV = 36;           // row pitch of the [kC][32] value tiles
  extern __shared__ float sm[];
  float* sQ = sm;                  // [kC][LD]  Q~
  float* sKt = sQ + kC * LD;       // [kC][LD]  K~
  float* sKb = sKt + kC * LD;      // [kC][LD]  K^
  float* sT = sKb + kC * LD;       // [kC][LT]
  float* sP = sT + kC * LT;        // [kC][LT]
  float* sS = sP + kC * LT;        // [32][LD]  state rows v0..v0+31 (v-major), fp32
  float* sZ = sS + 32 * LD;        // [kC][LV]  V, then V - K~ S0^T
  float* sV = sZ + kC * LV;        // [kC][LV]  v'
  float* sE = sV + kC * LV;        // [DH]      e^{G_C}

  const int h = blockIdx.x, b = blockIdx.z;
  const int v0 = blockIdx.y * 32;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, q = lane & 3;
  const int HD = a.H * DH;
  const int base = a.row0[b], n_all = a.nrows[b];
  const int64_t sstride = (int64_t)a.H * DH * DH;

  {
    const float* sin = a.S_pool + a.s_in[b] * sstride + ((int64_t)h * DH + v0) * DH;
    for (int e = tid; e < 32 * DH / 4; e += blockDim.x) {
      const int v = e / (DH / 4), c = (e % (DH / 4)) * 4;
      *reinterpret_cast<float4*>(sS + v * LD + c) = *reinterpret_cast<const float4*>(sin + v * DH + c);
    }
  }
  // warp tiles: [kC x 32] outputs -> m-tile mt (16 rows), n-tiles 2 nh, 2 nh + 1 (8 columns each)
  const int mt = warp >> 1, nh = warp & 1;
  for (int ci = 0; ci * kC < n_all; ++ci) {
    const int c0 = ci * kC;
    const int n = min(kC, n_all - c0);
    const int slot = chunk_slot(base, b, ci);
    if (slot >= a.scr_slots) break;
    const float* rec = a.scr + ((int64_t)slot * a.H + h) * kda_scr_per_head(DH);
    __syncthreads();
    // load the chunk record and the value slice
    for (int e = tid; e < kC * DH / 4; e += blockDim.x) {
      const int t = e / (DH / 4), c = (e % (DH / 4)) * 4;
      *reinterpret_cast<float4*>(sQ + t * LD + c) = *reinterpret_cast<const float4*>(rec + t * DH + c);
      *reinterpret_cast<float4*>(sKt + t * LD + c) = *reinterpret_cast<const float4*>(rec + kC * DH + t * DH + c);
      *reinterpret_cast<float4*>(sKb + t * LD + c) =
          *reinterpret_cast<const float4*>(rec + 2 * kC * DH + t * DH + c);
    }
    for (int e = tid; e < kC * kC / 4; e += blockDim.x) {
      const int t = e / (kC / 4), s = (e % (kC / 4)) * 4;
      *reinterpret_cast<float4*>(sT + t * LT + s) = *reinterpret_cast<const float4*>(rec + 3 * kC * DH + t * kC + s);
      *reinterpret_cast<float4*>(sP + t * LT + s) =
          *reinterpret_cast<const float4*>(rec + 3 * kC * DH + kC * kC + t * kC + s);
    }
    for (int c = tid; c < DH; c += blockDim.x) sE[c] = rec[3 * kC * DH + 2 * kC * kC + c];
    for (int e = tid; e < kC * 32; e += blockDim.x) {
      const int t = e >> 5, v = e & 31;
      sZ[t * LV + v] = t < n ? bf2f(a.qkv[(int64_t)(base + c0 + t) * 3 * HD + 2 * HD + h * DH + v0 + v]) : 0.f;
    }
    __syncthreads();
    // (1) Z = V - K~ S0^T
    {
      float acc[2][4] = {};
      for (int k0 = 0; k0 < DH; k0 += 8) {
        uint32_t fa[4];
        frag_a_row(sKt + mt * 16 * LD + k0, LD, fa);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          uint32_t b0, b1;
          frag_b_nk(sS + (nh * 16 + j * 8) * LD + k0, LD, b0, b1);
          mma_tf32(acc[j], fa, b0, b1);
        }
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int r = mt * 16 + g, cidx = nh * 16 + j * 8 + 2 * q;
        sZ[r * LV + cidx] -= acc[j][0];
        sZ[r * LV + cidx + 1] -= acc[j][1];
        sZ[(r + 8) * LV + cidx] -= acc[j][2];
        sZ[(r + 8) * LV + cidx + 1] -= acc[j][3];
      }
    }
    __syncthreads();
    // (2) v' = T Z  (T lower triangular: columns past the m-tile's last row are zero)
    {
      float acc[2][4] = {};
      for (int k0 = 0; k0 < (mt + 1) * 16; k0 += 8) {
        uint32_t fa[4];
        frag_a_row(sT + mt * 16 * LT + k0, LT, fa);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          uint32_t b0, b1;
          frag_b_kn(sZ + k0 * LV + nh * 16 + j * 8, LV, b0, b1);
          mma_tf32(acc[j], fa, b0, b1);
        }
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int r = mt * 16 + g, cidx = nh * 16 + j * 8 + 2 * q;
        sV[r * LV + cidx] = acc[j][0];
        sV[r * LV + cidx + 1] = acc[j][1];
        sV[(r + 8) * LV + cidx] = acc[j][2];
        sV[(r + 8) * LV + cidx + 1] = acc[j][3];
      }
    }
    __syncthreads();
    // (3) o = Q~ S0^T + P v'
    {
      float acc[2][4] = {};
      for (int k0 = 0; k0 < DH; k0 += 8) {
        uint32_t fa[4];
        frag_a_row(sQ + mt * 16 * LD + k0, LD, fa);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          uint32_t b0, b1;
          frag_b_nk(sS + (nh * 16 + j * 8) * LD + k0, LD, b0, b1);
          mma_tf32(acc[j], fa, b0, b1);
        }
      }
      for (int k0 = 0; k0 < (mt + 1) * 16; k0 += 8) {
        uint32_t fa[4];
        frag_a_row(sP + mt * 16 * LT + k0, LT, fa);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          uint32_t b0, b1;
          frag_b_kn(sV + k0 * LV + nh * 16 + j * 8, LV, b0, b1);
          mma_tf32(acc[j], fa, b0, b1);
        }
      }
      if (a.o_raw) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int r = mt * 16 + g, cidx = v0 + nh * 16 + j * 8 + 2 * q;
          if (r < n)
            *reinterpret_cast<float2*>(a.o_raw + (int64_t)(base + c0 + r) * HD + h * DH + cidx) =
                make_float2(acc[j][0], acc[j][1]);
          if (r + 8 < n)
            *reinterpret_cast<float2*>(a.o_raw + (int64_t)(base + c0 + r + 8) * HD + h * DH + cidx) =
                make_float2(acc[j][2], acc[j][3]);
        }
      }
    }
    __syncthreads();
    // (4) S = S diag(e^{G_C}) + v'^T K^   ([32 x DH] outputs: m-tile (warp & 1), DH/32 n-tiles per warp)
    {
      constexpr int NTW = DH / 32;
      const int mv = warp & 1, nb0 = (warp >> 1) * NTW;
      float acc[NTW][4];
#pragma unroll
      for (int j = 0; j < NTW; ++j) {
        const int r = mv * 16 + g, c = (nb0 + j) * 8 + 2 * q;
        acc[j][0] = sS[r * LD + c] * sE[c];
        acc[j][1] = sS[r * LD + c + 1] * sE[c + 1];
        acc[j][2] = sS[(r + 8) * LD + c] * sE[c];
        acc[j][3] = sS[(r + 8) * LD + c + 1] * sE[c + 1];
      }
      for (int k0 = 0; k0 < kC; k0 += 8) {
        uint32_t fa[4];
        frag_a_col(sV + k0 * LV + mv * 16, LV, fa);
#pragma unroll
        for (int j = 0; j < NTW; ++j) {
          uint32_t b0, b1;
          frag_b_kn(sKb + k0 * LD + (nb0 + j) * 8, LD, b0, b1);
          mma_tf32(acc[j], fa, b0, b1);
        }
      }
#pragma unroll
      for (int j = 0; j < NTW; ++j) {
        const int r = mv * 16 + g, c = (nb0 + j) * 8 + 2 * q;
        sS[r * LD + c] = acc[j][0];
        sS[r * LD + c + 1] = acc[j][1];
        sS[(r + 8) * LD + c] = acc[j][2];
        sS[(r + 8) * LD + c + 1] = acc[j][3];
      }
    }
  }
  __syncthreads();
  float* sout = a.S_pool + a.s_out[b] * sstride + ((int64_t)h * DH + v0) * DH;
  for (int e = tid; e < 32 * DH / 4; e += blockDim.x) {
    const int v = e / (DH / 4), c = (e % (DH / 4)) * 4;
    *reinterpret_cast<float4*>(sout + v * DH + c) = *reinterpret_cast<const float4*>(sS + v * LD + c);
  }
}

template <int DH>
cudaError_t launch_chunk(const KdaArgs& a, cudaStream_t st) {
  constexpr int P1 = DH + 1;
  const size_t smem_prep =
      sizeof(float) * ((size_t)4 * kC * P1 + 2 * kSubR * P1 + 3 * kC * (kC + 1) + kC);
  const size_t smem_scan =
      sizeof(float) * ((size_t)3 * kC * (DH + 4) + 2 * kC * (kC + 4) + 32 * (DH + 4) + 2 * kC * 36 + DH);
  cudaError_t e = cudaFuncSetAttribute(kda_prep_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem_prep);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(kda_scan_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_scan);
  if (e != cudaSuccess) return e;
  const dim3 gp((a.R + kC - 1) / kC, a.H, a.B);     // chunks past a sequence's rows exit at once
  kda_prep_kernel<DH><<<gp, 256, smem_prep, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const dim3 gs(a.H, DH / 32, a.B);
  kda_scan_kernel<DH><<<gs, 256, smem_scan, st>>>(a);
  return cudaGetLastError();
}

}  // namespace g53

int64_t g53_kda_chunk_scratch_floats(int max_rows, int max_seqs, int H, int Dh) {
  return ((int64_t)(max_rows + g53::kC - 1) / g53::kC + max_seqs + 1) * H * g53::kda_scr_per_head(Dh);
}

cudaError_t g53_kda_chunk(const KdaArgs& a, cudaStream_t st) {
  if (!a.scr || a.scr_slots <= 0) return cudaErrorInvalidValue;
  // the scratch must hold every chunk slot of this launch
  if ((int64_t)(a.R + g53::kC - 1) / g53::kC + a.B + 1 > a.scr_slots) return cudaErrorInvalidValue;
  if (a.Dh == 128) return g53::launch_chunk<128>(a, st);
  if (a.Dh == 64) return g53::launch_chunk<64>(a, st);
  return cudaErrorInvalidValue;
}
