// Chunked KDA for prefill in two kernels (same contract as kda_recurrent: reads S_pool[s_in], writes S_pool[s_out]
// and o_raw).  Per head, a chunk of C = 64 rows starting from state S0 (G_t = cumulative log-decay, g <= 0 per
// channel):
//   S_t  = S0 diag(e^{G_t}) + sum_{s<=t} v'_s (k_s e^{G_t - G_s})^T
//   v'   = T (V - K~ S0^T),   T = (I + diag(beta) M)^{-1} diag(beta),   M_ts = sum_c k_t k_s e^{G_t - G_s} (s < t)
//   o    = Q~ S0^T + P v',    P_ts = sum_c q_t k_s e^{G_t - G_s} (s <= t)
//   S_C  = S0 diag(e^{G_C}) + v'^T K^ ,   K~_t = k_t e^{G_t},  Q~_t = q_t e^{G_t},  K^_s = k_s e^{G_C - G_s}
//
// kda_prep_kernel   one CTA per (chunk, head, sequence), two per SM, all chunks in parallel, over 64-channel
//                   blocks: normalised rows, cumulative decay, M and P (3xTF32 tensor-core products with fp32
//                   accumulation, 16-row sub-chunk reference points so every exponential factor stays bounded),
//                   the unit lower-triangular inverse by forward substitution, T, and the scaled rows Q~, K~, K^
//                   and e^{G_C}; written to a per-(chunk, head) scratch.
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

// record per (chunk slot, head), in floats: Q~, K~, K^ as fp16 [kC][dh] each (exact for the tf32 products; every
// value is a unit-normalised row times a decay factor <= 1), T and P as fp16 [kC][kC] (the scan feeds them to tf32
// products: fp16 keeps the same 10 explicit significand bits; T's columns are those of a product of delta-rule
// contractions and P's entries are decayed dot products of normalised rows, far inside the fp16 range), e^{G_C}
// fp32 [dh]
__host__ __device__ constexpr int64_t kda_scr_per_head(int dh) { return 3LL * kC * dh / 2 + 1LL * kC * kC + dh; }

__device__ __forceinline__ int chunk_slot(int row0, int b, int c) { return row0 / kC + b + c; }

// ---------------------------------------------------------------------------------------------------------------
// tf32 tensor-core helpers (both kernels)
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

// x = hi + lo with hi and lo both tf32 (3xTF32: hi*hi + hi*lo + lo*hi keeps about fp32 accuracy)
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
  hi = to_tf32(x);
  lo = to_tf32(x - __uint_as_float(hi));
}

// ---------------------------------------------------------------------------------------------------------------
// prep: grid (max chunks, H, B), 256 threads, two CTAs per SM.
// The channels are taken in blocks of kCB = 64 (DH / 64 blocks): a block's rows, cumulative decay and scaled rows
// need only its own channels, and M / P are sums over channels, so each block adds its part to M and P and writes
// its columns of Q~, K~, K^ and e^{G_C} to the record; the unit lower-triangular inverse runs once at the end.
// The M / P products (16 rows of t x up to 64 keys s x 64 channels per sub-chunk) run on the tensor cores as
// 3xTF32 m16n8k8 products.
// ---------------------------------------------------------------------------------------------------------------
constexpr int kCB = 64;                 // channels per block
constexpr int kPH = kCB + 4;            // row pitch of the block tiles: the mma fragment loads hit 32 banks
constexpr int kPM = kC + 1;             // row pitch of the 64 x 64 chunk matrices

__host__ __device__ constexpr int prep_smem_floats() { return 4 * kC * kPH + 2 * kSubR * kPH + 2 * kC * kPM + kC; }

template <int DH>
__global__ void __launch_bounds__(256, 2) kda_prep_kernel(KdaArgs a) {
  constexpr int NB = DH / kCB;          // channel blocks
  constexpr int PL = DH / 32;           // channels per lane of a full row
  extern __shared__ float sm[];
  float* sK = sm;                       // [kC][kPH] normalised k of the block's channels
  float* sQ = sK + kC * kPH;            // [kC][kPH] normalised, scaled q
  float* sG = sQ + kC * kPH;            // [kC][kPH] raw g, then cumulative G
  float* sX = sG + kC * kPH;            // [kC][kPH] k_s e^{G_r - G_s}
  float* sA = sX + kC * kPH;            // [kSubR][kPH] k_t e^{G_t - G_r}
  float* sQt = sA + kSubR * kPH;        // [kSubR][kPH] q_t e^{G_t - G_r}
  float* sM = sQt + kSubR * kPH;        // [kC][kPM] M (summed over the channel blocks)
  float* sP = sM + kC * kPM;            // [kC][kPM] P
  float* sB = sP + kC * kPM;            // [kC] beta
  float* sI = sm;                       // [kC][kPM] (I + diag(beta) M)^{-1}: after the blocks, over sK / sQ
  float* sW = sm + kC * kPM;            // W blocks of one distance (step 4)

  const int ci = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int base = a.row0[b], n_all = a.nrows[b];
  const int c0 = ci * kC;
  if (c0 >= n_all) return;
  const int n = min(kC, n_all - c0);
  const int slot = chunk_slot(base, b, ci);
  if (slot >= a.scr_slots) return;                 // the launcher sizes the scratch; never reached
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g8 = lane >> 2, q4 = lane & 3;
  const int HD = a.H * DH;
  const float ea = __expf(a.a_log[h]);
  const int last = n - 1;

  float* out = a.scr + ((int64_t)slot * a.H + h) * kda_scr_per_head(DH);
  __half* oQ = reinterpret_cast<__half*>(out);
  __half* oK = oQ + kC * DH;
  __half* oKb = oK + kC * DH;
  __half* oT = reinterpret_cast<__half*>(out + 3 * kC * DH / 2);
  __half* oP = oT + kC * kC;
  float* oE = out + 3 * kC * DH / 2 + kC * kC;

  for (int e = tid; e < 2 * kC * kPM; e += blockDim.x) sM[e] = 0.f;     // sM and sP are adjacent

  for (int hb = 0; hb < NB; ++hb) {
    const int cb = hb * kCB;
    if (hb > 0) __syncthreads();                  // the previous block's tiles are consumed
    // 1. rows: normalised q, k (norms over all DH channels), this block's raw g, beta.  A warp owns rows warp,
    //    warp + 8, ...; the loads of 4 rows are issued together before any of them is reduced
    for (int t0 = warp; t0 < kC; t0 += 32) {
      __nv_bfloat16 rq[4][PL], rk[4][PL], rf[4][2], rb[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int t = t0 + 8 * u, row = base + c0 + t;
        const bool on = t < n;
        const __nv_bfloat16* rp = a.qkv + (int64_t)(on ? row : base) * 3 * HD;
        const __nv_bfloat16* fp = a.f + (int64_t)(on ? row : base) * HD + h * DH + cb;
#pragma unroll
        for (int i = 0; i < PL; ++i) {
          const int c = lane + 32 * i;
          rq[u][i] = rp[h * DH + c];
          rk[u][i] = rp[HD + h * DH + c];
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) rf[u][i] = fp[lane + 32 * i];
        rb[u] = a.proj[(int64_t)(on ? row : base) * a.ldp + a.b_off + h];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int t = t0 + 8 * u;
        const bool on = t < n;
        float q[PL], k[PL];
        float sq = 0.f, sk = 0.f;
#pragma unroll
        for (int i = 0; i < PL; ++i) {
          q[i] = on ? bf2f(rq[u][i]) : 0.f;
          k[i] = on ? bf2f(rk[u][i]) : 0.f;
          sq += q[i] * q[i];
          sk += k[i] * k[i];
        }
        sq = warp_sum(sq);
        sk = warp_sum(sk);
        const float qn = rsqrtf(sq + 1e-6f) * rsqrtf((float)DH), kn = rsqrtf(sk + 1e-6f);
#pragma unroll
        for (int i = 0; i < PL; ++i) {               // the lane's channels of this block: i / 2 == hb
          if ((i >> 1) != hb) continue;
          const int cl = lane + 32 * (i & 1), c = cb + cl;
          sQ[t * kPH + cl] = q[i] * qn;
          sK[t * kPH + cl] = k[i] * kn;
          sG[t * kPH + cl] = on ? a.lower * sigmoidf_(ea * (bf2f(rf[u][i & 1]) + a.dt_bias[h * DH + c])) : 0.f;
        }
        if (hb == 0 && lane == 0) sB[t] = on ? sigmoidf_(bf2f(rb[u])) : 0.f;
      }
    }
    __syncthreads();
    // 2. cumulative log-decay per channel (rows past n add 0 and keep the last value): four 16-row segments per
    //    channel summed in parallel, one per thread, then each segment adds the totals of the segments before it
    {
      const int c = tid % kCB, sb = tid / kCB;
      float acc = 0.f;
#pragma unroll 4
      for (int t = 0; t < 16; ++t) {
        const int r = sb * 16 + t;
        acc += sG[r * kPH + c];
        sG[r * kPH + c] = acc;
      }
      __syncthreads();
      const float tot0 = sG[15 * kPH + c], tot1 = sG[31 * kPH + c], tot2 = sG[47 * kPH + c];
      __syncthreads();
      if (sb > 0) {
        const float add = sb == 1 ? tot0 : (sb == 2 ? tot0 + tot1 : (tot0 + tot1) + tot2);
#pragma unroll 4
        for (int t = 0; t < 16; ++t) sG[(sb * 16 + t) * kPH + c] += add;
      }
    }
    __syncthreads();
    // 3. this block's part of M (strictly lower) and P (lower incl. diagonal), one 16-row sub-chunk of t at a time
    //    with reference row r (every exponential factor stays bounded); warp jobs = (matrix, 8-key tile)
    for (int j = 0; j < kC / kSubR; ++j) {
      const int r = j * kSubR;
      const int ns = r + kSubR;                    // s ranges over [0, ns)
      for (int e = tid; e < kSubR * kCB; e += blockDim.x) {
        const int t = e / kCB, c = e % kCB;
        const float f = __expf(sG[(r + t) * kPH + c] - sG[r * kPH + c]);
        sA[t * kPH + c] = sK[(r + t) * kPH + c] * f;
        sQt[t * kPH + c] = sQ[(r + t) * kPH + c] * f;
      }
      for (int e = tid; e < ns * kCB; e += blockDim.x) {
        const int s = e / kCB, c = e % kCB;
        sX[s * kPH + c] = sK[s * kPH + c] * __expf(sG[r * kPH + c] - sG[s * kPH + c]);
      }
      __syncthreads();
      const int jobs = 2 * (ns / 8);
      for (int jb = warp; jb < jobs; jb += 8) {
        const int mm = jb & 1, nt = jb >> 1;
        const float* As = mm ? sQt : sA;
        const float* Bs = sX + (nt * 8 + g8) * kPH;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 2
        for (int k0 = 0; k0 < kCB; k0 += 8) {
          uint32_t ah[4], al[4], bh[2], bl[2];
          split_tf32(As[g8 * kPH + k0 + q4], ah[0], al[0]);
          split_tf32(As[(g8 + 8) * kPH + k0 + q4], ah[1], al[1]);
          split_tf32(As[g8 * kPH + k0 + q4 + 4], ah[2], al[2]);
          split_tf32(As[(g8 + 8) * kPH + k0 + q4 + 4], ah[3], al[3]);
          split_tf32(Bs[k0 + q4], bh[0], bl[0]);
          split_tf32(Bs[k0 + q4 + 4], bh[1], bl[1]);
          mma_tf32(acc, al, bh[0], bh[1]);
          mma_tf32(acc, ah, bl[0], bl[1]);
          mma_tf32(acc, ah, bh[0], bh[1]);
        }
        // accumulator (t = r + g8 (+8), s = nt*8 + 2 q4 (+1)); each element has one owner: plain adds
        float* dst = mm ? sP : sM;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int tt = r + g8 + (i >> 1) * 8, s = nt * 8 + 2 * q4 + (i & 1);
          const bool keep = mm ? s <= tt : s < tt;
          if (keep) dst[tt * kPM + s] += acc[i];
        }
      }
      __syncthreads();
    }
    // 5. this block's scaled rows into the record: Q~ = q e^{G}, K~ = k e^{G}, K^ = k e^{G_C - G} (rows past n: 0),
    //    and e^{G_C}
    for (int e = tid; e < kC * kCB / 2; e += blockDim.x) {
      const int t = (2 * e) / kCB, c = (2 * e) % kCB;
      float vq[2], vk[2], vb[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const float G = sG[t * kPH + c + i];
        const float d = __expf(G);
        vq[i] = sQ[t * kPH + c + i] * d;
        vk[i] = sK[t * kPH + c + i] * d;
        vb[i] = t < n ? sK[t * kPH + c + i] * __expf(sG[last * kPH + c + i] - G) : 0.f;
      }
      const int64_t o = (int64_t)t * DH + cb + c;
      *reinterpret_cast<__half2*>(oQ + o) = __floats2half2_rn(vq[0], vq[1]);
      *reinterpret_cast<__half2*>(oK + o) = __floats2half2_rn(vk[0], vk[1]);
      *reinterpret_cast<__half2*>(oKb + o) = __floats2half2_rn(vb[0], vb[1]);
    }
    for (int c = tid; c < kCB; c += blockDim.x) oE[cb + c] = __expf(sG[last * kPH + c]);
  }
  __syncthreads();
  // 4. X = (I + diag(beta) M)^{-1} (unit lower triangular) in 16 x 16 blocks: the four diagonal blocks by forward
  //    substitution, one warp each with a column per lane held in registers (no block-wide barriers), then the
  //    blocks below the diagonal by distance d = i - j: X_ij = -X_ii sum_{k=j}^{i-1} (diag(beta) M)_ik X_kj
  {
    for (int e = tid; e < kC * kC; e += blockDim.x) sI[(e / kC) * kPM + e % kC] = 0.f;
    __syncthreads();
    if (warp < 4 && lane < kSubR) {
      const int o = warp * kSubR, jc = lane;
      float x[kSubR];
#pragma unroll
      for (int t = 0; t < kSubR; ++t) x[t] = t == jc ? 1.f : 0.f;
#pragma unroll
      for (int t = 1; t < kSubR; ++t) {
        float acc = 0.f;
#pragma unroll
        for (int s2 = 0; s2 < t; ++s2) acc += sM[(o + t) * kPM + o + s2] * x[s2];
        if (t > jc) x[t] = -sB[o + t] * acc;
      }
#pragma unroll
      for (int t = 0; t < kSubR; ++t) sI[(o + t) * kPM + o + jc] = x[t];
    }
    __syncthreads();
    for (int d = 1; d < kC / kSubR; ++d) {
      const int nblk = kC / kSubR - d;
      for (int e = tid; e < nblk * kSubR * kSubR; e += blockDim.x) {
        const int jb = e / (kSubR * kSubR), rr = (e / kSubR) % kSubR, col = e % kSubR, ib = jb + d;
        float w = 0.f;
        for (int kb = jb; kb < ib; ++kb)
#pragma unroll 4
          for (int m = 0; m < kSubR; ++m)
            w += sM[(kSubR * ib + rr) * kPM + kSubR * kb + m] * sI[(kSubR * kb + m) * kPM + kSubR * jb + col];
        sW[e] = w * sB[kSubR * ib + rr];
      }
      __syncthreads();
      for (int e = tid; e < nblk * kSubR * kSubR; e += blockDim.x) {
        const int jb = e / (kSubR * kSubR), rr = (e / kSubR) % kSubR, col = e % kSubR, ib = jb + d;
        float x = 0.f;
#pragma unroll 4
        for (int m = 0; m < kSubR; ++m)
          x += sI[(kSubR * ib + rr) * kPM + kSubR * ib + m] * sW[jb * kSubR * kSubR + m * kSubR + col];
        sI[(kSubR * ib + rr) * kPM + kSubR * jb + col] = -x;
      }
      __syncthreads();
    }
  }
  // 6. T = X diag(beta) and P into the record
  for (int e = tid; e < kC * kC; e += blockDim.x) {
    const int t = e / kC, s = e % kC;
    oT[e] = __float2half_rn(sI[t * kPM + s] * sB[s]);
    oP[e] = __float2half_rn(sP[t * kPM + s]);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// scan: grid (H, DH/32, B), 256 threads (8 warps)
// ---------------------------------------------------------------------------------------------------------------
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

// fp16 tile element -> tf32 operand (exact: fp16 has the tf32 mantissa width)
__device__ __forceinline__ uint32_t h2tf(const __half* p) { return __float_as_uint(__half2float(*p)); }
__device__ __forceinline__ void frag_a_row_h(const __half* p, int ld, uint32_t (&f)[4]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  f[0] = h2tf(p + g * ld + q);
  f[1] = h2tf(p + (g + 8) * ld + q);
  f[2] = h2tf(p + g * ld + q + 4);
  f[3] = h2tf(p + (g + 8) * ld + q + 4);
}
__device__ __forceinline__ void frag_b_kn_h(const __half* p, int ld, uint32_t& b0, uint32_t& b1) {
  const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  b0 = h2tf(p + q * ld + g);
  b1 = h2tf(p + (q + 4) * ld + g);
}
__device__ __forceinline__ void cp16(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src), "r"(bytes) : "memory");
}

// shared-memory layout of one record buffer (floats): fp16 Q~ / K~ / K^ tiles, T, P, e^{G_C}, raw bf16 V slice
template <int DH>
struct ScanBuf {
  static constexpr int LH = DH + 8;                        // row pitch (halves) of the fp16 tiles
  static constexpr int LT = kC + 8;                        // row pitch (halves) of T and P
  static constexpr int H3 = 3 * kC * LH / 2;               // floats of the three fp16 tiles
  static constexpr int T_OFF = H3, P_OFF = H3 + kC * LT / 2, E_OFF = H3 + kC * LT, V_OFF = E_OFF + DH;
  static constexpr int FLOATS = V_OFF + kC * 32 / 2;        // + [kC][32] bf16 value slice
};

// DB: two record buffers, one CTA per SM (the next chunk's record loads during this chunk); otherwise one
// buffer and two CTAs per SM (used when the grid has more CTAs than SMs: all of them run in one round, each
// CTA's record load overlapping the other CTA's products)
template <int DH, bool DB>
__global__ void __launch_bounds__(256, DB ? 1 : 2) kda_scan_kernel(KdaArgs a) {
  using B = ScanBuf<DH>;
  constexpr int LH = B::LH, LT = B::LT;
  constexpr int LD = DH + 4;       // row pitch of the fp32 state tile
  constexpr int LV = 36;           // row pitch of the [kC][32] value tiles
  extern __shared__ float sm[];
  float* buf0 = sm;                // record buffers (DB: chunk ci uses buffer ci % 2; ci + 1 loads meanwhile)
  float* sS = sm + (DB ? 2 : 1) * B::FLOATS;   // [32][LD]  state rows v0..v0+31 (v-major), fp32
  float* sZ = sS + 32 * LD;        // [kC][LV]  V, then V - K~ S0^T
  float* sV = sZ + kC * LV;        // [kC][LV]  v'

  const int h = blockIdx.x, b = blockIdx.z;
  if (!g53_in_bounds(a.s_in[b], a.n_states, 5) || !g53_in_bounds(a.s_out[b], a.n_states, 5)) return;
  const int v0 = blockIdx.y * 32;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, q = lane & 3;
  const int HD = a.H * DH;
  const int base = a.row0[b], n_all = a.nrows[b];
  const int64_t sstride = (int64_t)a.H * DH * DH;
  const int nchunks = (n_all + kC - 1) / kC;

  // asynchronous copy of chunk ci's record and value slice into buffer bi (every thread issues its share)
  auto issue = [&](int ci, int bi) {
    const int slot = chunk_slot(base, b, ci);
    if (slot >= a.scr_slots) return;
    const float* rec = a.scr + ((int64_t)slot * a.H + h) * kda_scr_per_head(DH);
    float* bf = buf0 + bi * B::FLOATS;
    __half* hq = reinterpret_cast<__half*>(bf);
    const __half* rh = reinterpret_cast<const __half*>(rec);
    for (int e = tid; e < 3 * kC * (DH / 8); e += blockDim.x) {      // 16-byte pieces of the fp16 tiles
      const int m = e / (kC * (DH / 8)), t = (e / (DH / 8)) % kC, c = e % (DH / 8);
      cp16(hq + m * kC * LH + t * LH + c * 8, rh + (int64_t)m * kC * DH + t * DH + c * 8, 16u);
    }
    const __half* rt = reinterpret_cast<const __half*>(rec + 3 * kC * DH / 2);
    __half* ht = reinterpret_cast<__half*>(bf + B::T_OFF);
    for (int e = tid; e < 2 * kC * (kC / 8); e += blockDim.x) {       // T then P, fp16
      const int m = e / (kC * (kC / 8)), t = (e / (kC / 8)) % kC, c = e % (kC / 8);
      cp16(ht + m * kC * LT + t * LT + c * 8, rt + m * kC * kC + t * kC + c * 8, 16u);
    }
    const float* re = rec + 3 * kC * DH / 2 + kC * kC;
    for (int e = tid; e < DH / 4; e += blockDim.x) cp16(bf + B::E_OFF + e * 4, re + e * 4, 16u);
    const int c0 = ci * kC, n = min(kC, n_all - c0);
    __nv_bfloat16* vr = reinterpret_cast<__nv_bfloat16*>(bf + B::V_OFF);
    for (int e = tid; e < kC * 4; e += blockDim.x) {                  // 4 x 16 bytes per value row
      const int t = e >> 2, c = e & 3;
      const __nv_bfloat16* src = a.qkv + (int64_t)(base + c0 + (t < n ? t : 0)) * 3 * HD + 2 * HD + h * DH + v0 + c * 8;
      cp16(vr + t * 32 + c * 8, src, t < n ? 16u : 0u);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  {
    const float* sin = a.S_pool + a.s_in[b] * sstride + ((int64_t)h * DH + v0) * DH;
    for (int e = tid; e < 32 * DH / 4; e += blockDim.x) {
      const int v = e / (DH / 4), c = (e % (DH / 4)) * 4;
      *reinterpret_cast<float4*>(sS + v * LD + c) = *reinterpret_cast<const float4*>(sin + v * DH + c);
    }
  }
  if (nchunks > 0) issue(0, 0);
  // warp tiles: [kC x 32] outputs -> m-tile mt (16 rows), n-tiles 2 nh, 2 nh + 1 (8 columns each)
  const int mt = warp >> 1, nh = warp & 1;
  for (int ci = 0; ci < nchunks; ++ci) {
    const int c0 = ci * kC;
    const int n = min(kC, n_all - c0);
    if (chunk_slot(base, b, ci) >= a.scr_slots) break;
    if (!DB && ci > 0) {
      __syncthreads();                       // every thread is done with chunk ci - 1's record: reuse the buffer
      issue(ci, 0);
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();                         // chunk ci landed for every thread; DB: buffer (ci + 1) % 2 is free
    if (DB && ci + 1 < nchunks) issue(ci + 1, (ci + 1) & 1);
    const float* bf = buf0 + (DB ? (ci & 1) : 0) * B::FLOATS;
    const __half* sQ = reinterpret_cast<const __half*>(bf);
    const __half* sKt = sQ + kC * LH;
    const __half* sKb = sKt + kC * LH;
    const __half* sT = reinterpret_cast<const __half*>(bf + B::T_OFF);
    const __half* sP = reinterpret_cast<const __half*>(bf + B::P_OFF);
    const float* sE = bf + B::E_OFF;
    const __nv_bfloat16* vr = reinterpret_cast<const __nv_bfloat16*>(bf + B::V_OFF);
    for (int e = tid; e < kC * 32; e += blockDim.x) {
      const int t = e >> 5, v = e & 31;
      sZ[t * LV + v] = bf2f(vr[t * 32 + v]);
    }
    __syncthreads();
    // (1) Z = V - K~ S0^T
    {
      float acc[2][4] = {};
      for (int k0 = 0; k0 < DH; k0 += 8) {
        uint32_t fa[4];
        frag_a_row_h(sKt + mt * 16 * LH + k0, LH, fa);
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
        frag_a_row_h(sT + mt * 16 * LT + k0, LT, fa);
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
        frag_a_row_h(sQ + mt * 16 * LH + k0, LH, fa);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          uint32_t b0, b1;
          frag_b_nk(sS + (nh * 16 + j * 8) * LD + k0, LD, b0, b1);
          mma_tf32(acc[j], fa, b0, b1);
        }
      }
      for (int k0 = 0; k0 < (mt + 1) * 16; k0 += 8) {
        uint32_t fa[4];
        frag_a_row_h(sP + mt * 16 * LT + k0, LT, fa);
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
          frag_b_kn_h(sKb + k0 * LH + (nb0 + j) * 8, LH, b0, b1);
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
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  float* sout = a.S_pool + a.s_out[b] * sstride + ((int64_t)h * DH + v0) * DH;
  for (int e = tid; e < 32 * DH / 4; e += blockDim.x) {
    const int v = e / (DH / 4), c = (e % (DH / 4)) * 4;
    *reinterpret_cast<float4*>(sout + v * DH + c) = *reinterpret_cast<const float4*>(sS + v * LD + c);
  }
}

template <int DH, bool DB>
cudaError_t launch_scan(const KdaArgs& a, cudaStream_t st) {
  const size_t smem = sizeof(float) * ((size_t)(DB ? 2 : 1) * ScanBuf<DH>::FLOATS + 32 * (DH + 4) + 2 * kC * 36);
  cudaError_t e = cudaFuncSetAttribute(kda_scan_kernel<DH, DB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kda_scan_kernel<DH, DB><<<dim3(a.H, DH / 32, a.B), 256, smem, st>>>(a);
  return cudaGetLastError();
}

static int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      n = 148;
  }
  return n;
}

template <int DH>
cudaError_t launch_chunk(const KdaArgs& a, cudaStream_t st) {
  const size_t smem_prep = sizeof(float) * (size_t)prep_smem_floats();
  cudaError_t e = cudaFuncSetAttribute(kda_prep_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem_prep);
  if (e != cudaSuccess) return e;
  const dim3 gp((a.R + kC - 1) / kC, a.H, a.B);     // chunks past a sequence's rows exit at once
  kda_prep_kernel<DH><<<gp, 256, smem_prep, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  // scan CTAs: (head, 32 value rows, sequence); more of them than SMs -> the single-buffer, two-per-SM form
  if ((int64_t)a.H * (DH / 32) * a.B > sm_count()) return launch_scan<DH, false>(a, st);
  return launch_scan<DH, true>(a, st);
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
