// Decode projection ("GEMV", M <= 16 activation rows) for large fp8 weights, streamed by the bulk-copy (TMA) engine.
//
// Y[M, N] = X[M, K] @ (W8[N, K] * s[N])^T.  A decode projection reads every weight byte once, so its speed of light
// is HBM bandwidth; what keeps a load-per-lane kernel below it is too few bytes in flight per SM.  Here one CTA per
// SM is persistent over 16-row tiles: a producer warp streams each tile in stages of 16 rows x KC bytes (KC = 1, 2
// or 4 KB) into a ring of shared-memory buffers with cp.async.bulk (one row segment per lane, completion counted in
// bytes on the stage's mbarrier, L2 evict-first: the weights are read once), so about 200 KB per SM are in flight
// independent of how long the math warps take.  The copy size matters: with 1 KB copies the stream stalled near
// 2.5-3 TB/s whatever the ring depth, 4 KB copies reach 5.8 TB/s.  Sixteen consumer warps split each stage's k
// range, load their 16-byte weight segments from shared memory (rows padded by 64 bytes: the two rows a
// quarter-warp reads fall in disjoint bank halves), convert e4m3 -> f16 exactly and run swap-AB mma.m16n8k16 (the
// weight tile is the 16-row A operand, the at most 16 activation rows the B operand, with the same k permutation
// inside each 64-element chunk as the load-per-lane kernel); the activation fragments stay in registers for the
// CTA's life when K is small enough.  The per-warp partial tiles are summed in fixed warp order (deterministic)
// through a shared array, and the output modes are those of the load-per-lane kernel (bf16, fp32, fp32 accumulate,
// interleaved SwiGLU, fused push of the fp32 partial to every tensor-parallel peer).
//
// The weight stream does not depend on the previous kernel, so the producer starts before griddepcontrol.wait
// (programmatic dependent launch); the consumers wait before touching X or Y.  Every mbarrier wait is bounded: on a
// timeout the kernel sets the error word and a CTA-wide stop flag, the remaining waits are skipped, every consumer
// still reaches each named barrier, and the producer waits (bounded) for its own copies in flight before exiting.
//
// Reference counterpart: code/fork/kernels/fp8_gemv.cu:96 (fp8 GEMV for M <= 64 rows on the load path).
#include <cstdint>
#include <cstdlib>
#include "common.cuh"
#include "launchers.h"

namespace g53 {
namespace gb {

constexpr int kRows = 16;                       // weight rows per tile (mma M)
constexpr int kCons = 16;                       // consumer warps
constexpr int kThreads = (kCons + 1) * 32;
constexpr uint32_t kSpin = 1u << 22;
constexpr int kErrCode = 0x6b01;                // error word value of a timed-out wait in this kernel
constexpr int kSmemBudget = 227 * 1024;

// A stage is 16 rows x KC bytes with KC = CPW x 1 KB (every consumer warp takes CPW 64-element chunks of it); rows
// sit at a pitch of KC + 64 bytes.  The weight ring takes what the reduction buffers leave of the 227 KB a CTA may
// hold (e.g. 3 stages of 64 KB for CPW = 4), since HBM latency under a full-GPU stream needs far more bytes in
// flight per SM than a few small stages.  The activations live in registers (or come from L2), so no L1 capacity
// is kept back.
template <bool TWO, int CPW>
struct Smem {
  static constexpr int kKC = CPW * 1024;
  static constexpr int kPitch = kKC + 64;
  static constexpr int kStageBytes = kRows * kPitch;
  static constexpr int kHalves = TWO ? 2 : 1;
  static constexpr int kFixed = kHalves * kCons * kRows * 17 * 4 + kRows * 17 * 4 + 256;
  static constexpr int kStagesFit = (kSmemBudget - kFixed) / (kStageBytes + 16);
  static constexpr int kStages = kStagesFit > 16 ? 16 : kStagesFit;
  static_assert(kStages >= 2, "weight ring needs two stages");
  alignas(128) uint8_t w[kStages][kStageBytes];
  float red[kHalves][kCons][kRows][17];         // [token half][warp][row][token]
  float tot[kRows][17];
  uint64_t full[kStages], empty[kStages];
  int stop;
};

__device__ __forceinline__ uint32_t su32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      ::"r"(su32(dst)), "l"(src), "r"(bytes), "r"(su32(bar)), "l"(pol) : "memory");
}
__device__ __forceinline__ void bar_init(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n));
}
__device__ __forceinline__ void bar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ void bar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool bar_try(uint64_t* b, uint32_t ph) {
  uint32_t ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0,1,0,p;\n}\n"
               : "=r"(ok) : "r"(su32(b)), "r"(ph) : "memory");
  return ok != 0;
}
// bounded wait for the completion of phase parity `ph`; false (stop flag and error word set) on a timeout, or
// false at once when another warp already stopped the CTA (unless `drain`)
__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t ph, volatile int* stop, int* err, bool drain = false) {
  uint32_t n = 0;
  while (!bar_try(b, ph)) {
    if (!drain && *stop) return false;
    if (++n > kSpin) {
      *stop = 1;
      if (err) atomicExch(err, kErrCode);
      return false;
    }
    if (n > 64) __nanosleep(64);
  }
  return true;
}
__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n)); }

template <bool TWO, int NX, int CPW>
__global__ void __launch_bounds__(kThreads, 1) gemv_bulk_kernel(GemvArgs p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  using SM = Smem<TWO, CPW>;
  constexpr int kStages = SM::kStages;
  constexpr int kc = SM::kKC;
  constexpr int kPitch = SM::kPitch;
  SM& sm = *reinterpret_cast<SM*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T = (p.N + kRows - 1) / kRows;
  const int nkc = p.K / kc;
  volatile int* stop = &sm.stop;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      bar_init(&sm.full[s], 1);
      bar_init(&sm.empty[s], kCons);
    }
    sm.stop = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_trigger();

  if (warp == kCons) {
    // ------------------------------------------------------------------ producer: weight stages into the ring
    const uint64_t pol = policy_evict_first();
    const uint8_t* W = reinterpret_cast<const uint8_t*>(p.w);
    uint32_t it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < T && ok; t += gridDim.x) {
      const int n0 = t * kRows;
      const int rows = min(kRows, p.N - n0);
      for (int s = 0; s < nkc; ++s, ++it) {
        const int slot = it % kStages;
        const uint32_t round = it / kStages;
        if (round > 0) {
          bool w8 = true;
          if (lane == 0) w8 = bar_wait(&sm.empty[slot], (round - 1) & 1, stop, p.err);
          ok = __shfl_sync(0xffffffffu, w8, 0);
          if (!ok) break;
        }
        if (lane == 0) bar_expect_tx(&sm.full[slot], (uint32_t)(rows * kc));
        __syncwarp();
        if (lane < rows)
          bulk_g2s(&sm.w[slot][lane * kPitch], W + (int64_t)(n0 + lane) * p.K + (int64_t)s * kc, (uint32_t)kc,
                   &sm.full[slot], pol);
      }
    }
    if (!ok && lane == 0) {
      // stopped: wait (bounded) until the copies this warp issued into the ring have landed
      const uint32_t first = it > (uint32_t)kStages ? it - kStages : 0;
      for (uint32_t j = first; j < it; ++j) bar_wait(&sm.full[j % kStages], (j / kStages) & 1, stop, p.err, true);
    }
  } else {
    // ------------------------------------------------------------------ consumers
    // warp w owns the 64-element chunks w*CPW .. w*CPW+CPW-1 of every stage; lane (g, q) the 16 k values q*16..
    // of rows g and g+8 in each
    const int g = lane >> 2, q = lane & 3;
    const bool t0 = g < p.M, t1 = TWO && (g + 8) < p.M;
    pdl_wait();
    const __nv_bfloat16* x0 = p.x + (int64_t)g * p.ldx + warp * CPW * 64 + q * 16;
    const __nv_bfloat16* x1 = p.x + (int64_t)(g + 8) * p.ldx + warp * CPW * 64 + q * 16;
    // the activation fragments of one chunk (f16x2, converted once)
    auto load_x = [&](int64_t koff, uint32_t (&xa)[8], uint32_t (&xc)[8]) {
      uint4 a0 = make_uint4(0, 0, 0, 0), a1 = a0, c0 = a0, c1 = a0;
      if (t0) {
        a0 = *reinterpret_cast<const uint4*>(x0 + koff);
        a1 = *reinterpret_cast<const uint4*>(x0 + koff + 8);
      }
      if (t1) {
        c0 = *reinterpret_cast<const uint4*>(x1 + koff);
        c1 = *reinterpret_cast<const uint4*>(x1 + koff + 8);
      }
      const uint32_t av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const uint32_t cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        xa[i] = bf16x2_to_f16x2(av[i]);
        if (TWO) xc[i] = bf16x2_to_f16x2(cv[i]);
      }
    };
    auto mma_chunk = [&](int slot, int cc, const uint32_t (&xa)[8], const uint32_t (&xc)[8], float (&acc0)[4],
                         float (&acc1)[4]) {
      const int kl = (warp * CPW + cc) * 64 + q * 16;
      const uint4 wa = *reinterpret_cast<const uint4*>(&sm.w[slot][g * kPitch + kl]);
      const uint4 wb = *reinterpret_cast<const uint4*>(&sm.w[slot][(g + 8) * kPitch + kl]);
      const uint32_t wav[4] = {wa.x, wa.y, wa.z, wa.w};
      const uint32_t wbv[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
      for (int k4 = 0; k4 < 4; ++k4) {
        uint32_t a[4];
        a[0] = e4m3x2_to_f16x2((uint16_t)(wav[k4] & 0xffffu));
        a[1] = e4m3x2_to_f16x2((uint16_t)(wbv[k4] & 0xffffu));
        a[2] = e4m3x2_to_f16x2((uint16_t)(wav[k4] >> 16));
        a[3] = e4m3x2_to_f16x2((uint16_t)(wbv[k4] >> 16));
        mma_f16_16816(acc0, a, xa[2 * k4], xa[2 * k4 + 1]);
        if (TWO) mma_f16_16816(acc1, a, xc[2 * k4], xc[2 * k4 + 1]);
      }
    };
    // NX > 0: every stage's fragments stay in registers for the CTA's whole life (K = NX * KC)
    constexpr int kXR = NX > 0 ? NX * CPW : 1;
    uint32_t xr[kXR][8], xr1[kXR][8];
    if constexpr (NX > 0) {
#pragma unroll
      for (int st = 0; st < NX; ++st)
#pragma unroll
        for (int cc = 0; cc < CPW; ++cc) load_x((int64_t)st * kc + cc * 64, xr[st * CPW + cc], xr1[st * CPW + cc]);
    }
    // NX == 0: the next stage's fragments, loaded one stage ahead
    uint32_t xn[CPW][8], xn1[CPW][8];
    if constexpr (NX == 0) {
#pragma unroll
      for (int cc = 0; cc < CPW; ++cc) load_x(cc * 64, xn[cc], xn1[cc]);
    }
    uint32_t it = 0;
    bool dead = false;
    // epilogue element of this thread: (row r, token tok) of every tile (threads 0..255)
    const int e = threadIdx.x;
    const bool act = e < kRows * 16;
    // consecutive threads own consecutive output columns of one row: the final stores (and the tensor-parallel
    // push into the peers' receive buffers over NVLink) are coalesced
    const int r = e & (kRows - 1), tok = (e >> 4) & 15;
    const bool swiglu = p.mode == GEMV_SWIGLU;
    for (int t = blockIdx.x; t < T; t += gridDim.x) {
      float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
      // the epilogue's global operands (row scales, the accumulated output) are loaded now, so their latency
      // passes under the tile's stages instead of stalling the epilogue
      const int n0 = t * kRows;
      const int n = n0 + r;
      const bool live = act && tok < p.M && n < p.N;
      const float sc = (p.scale && act && n < p.N) ? __ldg(p.scale + n) : 1.f;
      const float sc2 = (swiglu && p.scale && act && r < 8 && n + 8 < p.N) ? __ldg(p.scale + n + 8) : 1.f;
      const int64_t off = (int64_t)tok * p.ldy + n;
      const float yold = (p.mode == GEMV_F32_ACC && live) ? reinterpret_cast<const float*>(p.y)[off] : 0.f;
      if constexpr (NX > 0) {
#pragma unroll
        for (int s = 0; s < NX; ++s, ++it) {
          const int slot = it % kStages;
          if (!dead) {
            const bool w8 = bar_wait(&sm.full[slot], (it / kStages) & 1, stop, p.err);
            dead = !__all_sync(0xffffffffu, w8);
          }
          if (!dead) {
#pragma unroll
            for (int cc = 0; cc < CPW; ++cc) mma_chunk(slot, cc, xr[s * CPW + cc], xr1[s * CPW + cc], acc0, acc1);
          }
          __syncwarp();
          if (lane == 0 && !dead) bar_arrive(&sm.empty[slot]);
        }
      } else {
        for (int s = 0; s < nkc; ++s, ++it) {
          const int slot = it % kStages;
          uint32_t xa[CPW][8], xc[CPW][8];
#pragma unroll
          for (int cc = 0; cc < CPW; ++cc)
#pragma unroll
            for (int i = 0; i < 8; ++i) { xa[cc][i] = xn[cc][i]; xc[cc][i] = xn1[cc][i]; }
          const int64_t knext = (int64_t)(s + 1 < nkc ? s + 1 : 0) * kc;
#pragma unroll
          for (int cc = 0; cc < CPW; ++cc) load_x(knext + cc * 64, xn[cc], xn1[cc]);
          if (!dead) {
            const bool w8 = bar_wait(&sm.full[slot], (it / kStages) & 1, stop, p.err);
            dead = !__all_sync(0xffffffffu, w8);
          }
          if (!dead) {
#pragma unroll
            for (int cc = 0; cc < CPW; ++cc) mma_chunk(slot, cc, xa[cc], xc[cc], acc0, acc1);
          }
          __syncwarp();
          if (lane == 0 && !dead) bar_arrive(&sm.empty[slot]);
        }
      }
      // ---------------------------------------------------------------- tile epilogue (fixed warp order)
      float (*r0)[17] = sm.red[0][warp];
      r0[g][2 * q] = acc0[0];
      r0[g][2 * q + 1] = acc0[1];
      r0[g + 8][2 * q] = acc0[2];
      r0[g + 8][2 * q + 1] = acc0[3];
      if (TWO) {
        float (*r1)[17] = sm.red[TWO ? 1 : 0][warp];
        r1[g][2 * q] = acc1[0];
        r1[g][2 * q + 1] = acc1[1];
        r1[g + 8][2 * q] = acc1[2];
        r1[g + 8][2 * q + 1] = acc1[3];
      }
      named_sync(1, kCons * 32);
      float v = 0.f;
      if (act && tok < p.M) {
        const int h = tok >> 3, c = tok & 7;
#pragma unroll
        for (int w2 = 0; w2 < kCons; ++w2) v += sm.red[TWO ? h : 0][w2][r][c];
      }
      if (swiglu) {
        // rows 0..7 of the tile are gate rows j0..j0+7, rows 8..15 the matching up rows (the barrier also ends
        // every read of red, which the next tile rewrites)
        if (act) sm.tot[r][tok] = v;
        named_sync(1, kCons * 32);
        if (act && r < 8 && tok < p.M && n0 + r + 8 < p.N) {
          float gv = sm.tot[r][tok] * sc, uv = sm.tot[r + 8][tok] * sc2;
          gv = fminf(round_bf16(gv), p.limit);
          uv = fminf(fmaxf(round_bf16(uv), -p.limit), p.limit);
          reinterpret_cast<__nv_bfloat16*>(p.y)[(int64_t)tok * p.ldy + (n0 >> 1) + r] = f2bf(siluf_(gv) * uv);
        }
        // tot is rewritten by the next tile only after that tile's first named barrier, which every thread
        // reaches after finishing the reads above
        continue;
      }
      named_sync(1, kCons * 32);                     // every read of red done before the next tile rewrites it
      if (live) {
        v *= sc;
        if (p.mode == GEMV_BF16) {
          reinterpret_cast<__nv_bfloat16*>(p.y)[off] = f2bf(v);
        } else {
          float* yf = reinterpret_cast<float*>(p.y);
          v += yold;
          yf[off] = v;
          if (p.push_ptrs) {
            const int64_t so = (int64_t)p.push_rank * p.push_slot + off;
            for (int j = 0; j < p.push_world; ++j) p.push_ptrs[j][so] = v;
          }
        }
      }
    }
  }
  if (p.push_ptrs) {
    // the last CTA to finish raises this rank's arrival flag on every rank (release after all CTAs' stores)
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();
      const unsigned total = gridDim.x;
      const unsigned prev = atomicAdd(p.push_done, 1u);
      if (prev == total - 1) {
        *p.push_done = 0u;
        __threadfence_system();
        for (int j = 0; j < p.push_world; ++j) red_release_sys_add(p.push_flags[j] + p.push_rank, 1u);
      }
    }
  }
}

static int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

template <bool TWO, int NX, int CPW>
static cudaError_t launch(const GemvArgs& p, bool pdl, cudaStream_t st) {
  static bool attr = false;
  const int smem = (int)sizeof(Smem<TWO, CPW>);
  if (!attr) {
    cudaError_t e =
        cudaFuncSetAttribute(gemv_bulk_kernel<TWO, NX, CPW>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const int T = (p.N + kRows - 1) / kRows;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(std::min(T, sm_count()));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_bulk_kernel<TWO, NX, CPW>, p);
}

// stage width (CPW x 1 KB per row) and register-resident activations (NX stages) by K and the row count:
//   up to 8 rows   K % 4096 == 0: 4 KB stages, activations in registers for K <= 8192;  else 1 KB stages
//   9..16 rows     K % 2048 == 0: 2 KB stages, activations in registers for K <= 4096;  else 1 KB stages
static cudaError_t launch_cfg(const GemvArgs& p, bool pdl, cudaStream_t st) {
  const int K = p.K;
  if (p.M <= 8) {
    if (K % 4096 == 0) {
      if (K == 4096) return launch<false, 1, 4>(p, pdl, st);
      if (K == 8192) return launch<false, 2, 4>(p, pdl, st);
      return launch<false, 0, 4>(p, pdl, st);
    }
    if (K == 1024) return launch<false, 1, 1>(p, pdl, st);
    if (K == 2048) return launch<false, 2, 1>(p, pdl, st);
    return launch<false, 0, 1>(p, pdl, st);
  }
  if (K % 2048 == 0) {
    if (K == 2048) return launch<true, 1, 2>(p, pdl, st);
    if (K == 4096) return launch<true, 2, 2>(p, pdl, st);
    return launch<true, 0, 2>(p, pdl, st);
  }
  if (K == 1024) return launch<true, 1, 1>(p, pdl, st);
  return launch<true, 0, 1>(p, pdl, st);
}

}  // namespace gb
}  // namespace g53

// eligible: fp8 weights, one batch, 16-byte aligned rows of a K that splits into 1024-byte stages
bool g53_gemv_bulk_ok(const GemvArgs& p) {
  return p.batch == 1 && p.M >= 1 && p.M <= 16 && p.N >= 16 && p.K % 1024 == 0 &&
         reinterpret_cast<uintptr_t>(p.w) % 16 == 0;
}

cudaError_t g53_gemv_bulk(const GemvArgs& p, bool pdl, cudaStream_t st) {
  if (!g53_gemv_bulk_ok(p)) return cudaErrorInvalidValue;
  return g53::gb::launch_cfg(p, pdl, st);
}
