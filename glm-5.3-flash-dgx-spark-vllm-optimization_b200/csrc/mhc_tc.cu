// mHC partial pass of prefill-sized launches on the 5th-generation tensor cores (S = 4 streams).
//
// The mixing dots of the pre step are a skinny GEMM: mix[r, i] = sum_k X[r, k] fn[i, k] over k = (stream, column),
// 4 D = 16384 long, 24 outputs.  One CTA owns 128 rows x 512 columns (all 4 streams of them) and walks the columns
// in steps of 64:
//   256 threads  load X (4 streams) and the branch, apply the post of the previous block in fp32 exactly as the
//                CUDA-core kernel does (comb mix in stream order, then post * bf16(branch), bf16 rounding), write X back
//                to global memory and into the 128-byte-swizzled K-major A tile (one 64-column block per stream),
//                copy the matching 24 x 256 slice of fn into the B tile and accumulate the sums of squares;
//                the next step's loads are issued before the current step is processed
//   thread 0     issues tcgen05.mma kind::f16 (bf16 x bf16 -> fp32, M = 128 rows, N = 32 mixing columns, 24 used)
//                into one TMEM accumulator and commits; the tiles are rewritten once that commit has arrived
// At the end warps 0-3 read the accumulator (lane = row) and write part[r, block, 0..23] plus the sum of squares in
// slot 24; hc_finish_kernel sums the D / 512 blocks of a row.  The products are exact (bf16 x bf16 in fp32); only
// the summation order differs from the CUDA-core kernel.  Every wait is bounded (error word, early exit).
// Reference counterpart: the prenorm GEMM of the reference's mHC prefill (deep_gemm tf32_hc_prenorm_gemm through
// code/fork/overlay/patch_mhc_sp.py:6-10; code/fork/kernels/mhc_post_prenorm.cu:34 for post + prenorm).
#include "common.cuh"
#include "launchers.h"
#include "tc05.cuh"

namespace g53 {
namespace hct {

constexpr int S = 4;
constexpr int kRows = 128;                  // rows per CTA (MMA M)
constexpr int kCols = 512;                  // columns per CTA (of each stream)
constexpr int kStep = 64;                   // columns per step (one 128-byte swizzle row of bf16)
constexpr int kN = 32;                      // MMA N (24 mixing outputs, zero padded)
constexpr int kNM = 2 * S + S * S;          // 24
constexpr int kThreads = 256;
constexpr int A_BYTES = S * kRows * 128;    // 64 KB
constexpr int B_BYTES = S * kN * 128;       // 16 KB

struct Pass {                               // one thread's share of a step: 16 columns of one row
  uint4 x[S][2];
  float4 b[4];
};

__device__ __forceinline__ void load_pass(const HcArgs& a, int r, int c0, Pass& p) {
  if (r < a.R) {
    const __nv_bfloat16* xr = a.X + (int64_t)r * S * a.D + c0;
#pragma unroll
    for (int s = 0; s < S; ++s) {
      p.x[s][0] = *reinterpret_cast<const uint4*>(xr + (int64_t)s * a.D);
      p.x[s][1] = *reinterpret_cast<const uint4*>(xr + (int64_t)s * a.D + 8);
    }
    if (a.branch) {
      const float4* br = reinterpret_cast<const float4*>(a.branch + (int64_t)r * a.D + c0);
#pragma unroll
      for (int i = 0; i < 4; ++i) p.b[i] = br[i];
    }
  } else {
#pragma unroll
    for (int s = 0; s < S; ++s) p.x[s][0] = p.x[s][1] = make_uint4(0u, 0u, 0u, 0u);
  }
}

__global__ void __launch_bounds__(kThreads, 1) hc_partial_tc_kernel(HcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = sm;                         // [stream][128 rows x 128 B]
  uint8_t* sB = sm + A_BYTES;               // [stream][32 rows x 128 B]
  __shared__ __align__(8) uint64_t mma_done;
  __shared__ uint32_t tmem_base;
  __shared__ volatile int fail;
  __shared__ float ssm[kRows];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r0 = blockIdx.y * kRows, d0 = blockIdx.x * kCols, NB = gridDim.x;
  const int q = tid & 3;                    // 16-column quarter of a step
  const bool post = a.branch != nullptr;

  if (tid == 0) {
    fail = 0;
    tc::bar_init(&mma_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // padding rows 24..31 of the B tile stay zero
  for (int i = tid; i < S * (kN - kNM) * 8; i += kThreads) {
    const int s = i / ((kN - kNM) * 8), rr = kNM + (i / 8) % (kN - kNM), c = i % 8;
    *reinterpret_cast<uint4*>(sB + s * kN * 128 + tc::sw128_chunk(rr, c)) = make_uint4(0u, 0u, 0u, 0u);
  }
  if (warp == 0) tc::tmem_alloc(&tmem_base, kN);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = tmem_base;

  // the post mix of this thread's two rows (pass 0: row tid / 4, pass 1: row 64 + tid / 4)
  float cm[2][S * S], pw[2][S];
#pragma unroll
  for (int pa = 0; pa < 2; ++pa) {
    const int r = r0 + pa * 64 + (tid >> 2);
#pragma unroll
    for (int i = 0; i < S * S; ++i) cm[pa][i] = (post && r < a.R) ? a.comb[r * S * S + i] : 0.f;
#pragma unroll
    for (int s = 0; s < S; ++s) pw[pa][s] = (post && r < a.R) ? a.post[r * S + s] : 0.f;
  }
  float ss[2] = {0.f, 0.f};
  constexpr int kSteps = kCols / kStep;
  Pass cur, nxt;
  load_pass(a, r0 + (tid >> 2), d0 + q * 16, cur);
  bool ok = true;
  const uint32_t id = tc::idesc(1, kN, kRows);
#pragma unroll 2
  for (int it = 0; it < 2 * kSteps; ++it) {
    const int step = it >> 1, pa = it & 1;
    const int rl = pa * 64 + (tid >> 2), r = r0 + rl;
    const int c0 = d0 + step * kStep + q * 16;
    if (it + 1 < 2 * kSteps) {
      const int step1 = (it + 1) >> 1, pa1 = (it + 1) & 1;
      load_pass(a, r0 + pa1 * 64 + (tid >> 2), d0 + step1 * kStep + q * 16, nxt);
    }
    if (pa == 0 && step > 0) {
      // the MMAs of the previous step have read the tiles (one thread waits, the barrier makes it every thread's)
      if (tid == 0) tc::bar_wait(&mma_done, (step - 1) & 1, &fail, a.err, 31);
      __syncthreads();
      if (fail) { ok = false; break; }
      tc::fence_after();
    }
    // post (fp32, same operation order as the CUDA-core kernel), write back, swizzled A tile
    uint32_t o[S][8];
#pragma unroll
    for (int e = 0; e < 16; e += 2) {
      float bv[2] = {0.f, 0.f};
      if (post) {
        const float* bp = reinterpret_cast<const float*>(&cur.b[e >> 2]);
        bv[0] = round_bf16(bp[e & 3]);
        bv[1] = round_bf16(bp[(e & 3) + 1]);
      }
      float x[S][2];
#pragma unroll
      for (int s = 0; s < S; ++s) {
        const uint32_t wv = reinterpret_cast<const uint32_t*>(&cur.x[s][e >> 3])[(e & 7) >> 1];
        x[s][0] = __uint_as_float(wv << 16);
        x[s][1] = __uint_as_float(wv & 0xffff0000u);
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float nx[S];
#pragma unroll
        for (int s = 0; s < S; ++s) {
          if (post) {
            float m = 0.f;
#pragma unroll
            for (int j = 0; j < S; ++j) m += cm[pa][j * S + s] * x[j][h];
            nx[s] = round_bf16(pw[pa][s] * bv[h] + m);
          } else {
            nx[s] = x[s][h];
          }
        }
#pragma unroll
        for (int s = 0; s < S; ++s) { x[s][h] = nx[s]; ss[pa] += nx[s] * nx[s]; }
      }
#pragma unroll
      for (int s = 0; s < S; ++s) {
        __nv_bfloat162 p2 = __floats2bfloat162_rn(x[s][0], x[s][1]);
        o[s][e >> 1] = *reinterpret_cast<uint32_t*>(&p2);
      }
    }
#pragma unroll
    for (int s = 0; s < S; ++s) {
      const uint4 w0 = make_uint4(o[s][0], o[s][1], o[s][2], o[s][3]);
      const uint4 w1 = make_uint4(o[s][4], o[s][5], o[s][6], o[s][7]);
      if (post && r < a.R) {
        __nv_bfloat16* xr = a.X + (int64_t)r * S * a.D + (int64_t)s * a.D + c0;
        *reinterpret_cast<uint4*>(xr) = w0;
        *reinterpret_cast<uint4*>(xr + 8) = w1;
      }
      uint8_t* at = sA + s * kRows * 128;
      *reinterpret_cast<uint4*>(at + tc::sw128_chunk(rl, 2 * q)) = w0;
      *reinterpret_cast<uint4*>(at + tc::sw128_chunk(rl, 2 * q + 1)) = w1;
    }
    if (pa == 1) {
      // fn slice of this step: rows i < 24, streams s, 64 columns -> B tile (3 chunks per thread)
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        const int idx = tid + k * kThreads;           // 0 .. 767
        const int i = idx >> 5, s = (idx >> 3) & 3, c = idx & 7;
        const uint4 v = *reinterpret_cast<const uint4*>(a.fn + (int64_t)i * S * a.D + (int64_t)s * a.D + d0 +
                                                        step * kStep + c * 8);
        *reinterpret_cast<uint4*>(sB + s * kN * 128 + tc::sw128_chunk(i, c)) = v;
      }
      tc::fence_async_smem();
      __syncthreads();
      if (tid == 0) {
        tc::fence_after();
        const uint32_t aa = tc::saddr(sA), bb = tc::saddr(sB);
#pragma unroll
        for (int s = 0; s < S; ++s)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc::mma_f16(tmem, tc::desc_sw128(aa + s * kRows * 128 + k * 32), tc::desc_sw128(bb + s * kN * 128 + k * 32),
                        id, (step | s | k) ? 1u : 0u);
        tc::commit(&mma_done);
      }
    }
    cur = nxt;
  }
  // sums of squares: the 4 threads of a row are adjacent lanes
#pragma unroll
  for (int pa = 0; pa < 2; ++pa) {
    float t = ss[pa];
    t += __shfl_xor_sync(0xffffffffu, t, 1);
    t += __shfl_xor_sync(0xffffffffu, t, 2);
    if (q == 0) ssm[pa * 64 + (tid >> 2)] = t;
  }
  if (ok && tid == 0) tc::bar_wait(&mma_done, (kSteps - 1) & 1, &fail, a.err, 32);
  __syncthreads();
  tc::fence_after();
  if (ok && !fail && warp < 4) {
    const int rl = warp * 32 + lane, r = r0 + rl;
    float v[32];
    tc::tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16), v);
    if (r < a.R) {
      float* dst = a.part + ((int64_t)r * NB + blockIdx.x) * 32;
#pragma unroll
      for (int i = 0; i < kNM; ++i) dst[i] = v[i];
      dst[kNM] = ssm[rl];
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_free(tmem, kN);
}

}  // namespace hct
}  // namespace g53

cudaError_t g53_hc_partial_tc(const HcArgs& a, cudaStream_t st) {
  using namespace g53::hct;
  if (a.S != S || a.D % kCols || a.fn == nullptr || a.gath != nullptr || a.err == nullptr || a.R < 1)
    return cudaErrorInvalidValue;
  if (a.branch && (a.post == nullptr || a.comb == nullptr)) return cudaErrorInvalidValue;
  const int smem = A_BYTES + B_BYTES + 1024;
  cudaError_t e = cudaFuncSetAttribute(hc_partial_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  dim3 grid(a.D / kCols, (a.R + kRows - 1) / kRows);
  hc_partial_tc_kernel<<<grid, kThreads, smem, st>>>(a);
  return cudaGetLastError();
}
