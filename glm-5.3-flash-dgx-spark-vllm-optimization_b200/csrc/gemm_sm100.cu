// Large-M GEMM for prefill on the 5th-generation tensor cores: Y[M, N] = (A[M, K] @ B[N, K]^T) * scales.
//
//   A  activations, K-major (bf16, or e4m3 with one fp32 scale per row)
//   B  weights [N, K], K-major (bf16, or e4m3 with one fp32 scale per output row: the engine's fp8 weights)
//
// Persistent: one CTA per SM walks the 128 x BN output tiles in a grouped order (bands of 8 M-tiles).  Warp roles
// (192 threads):
//   warp 0    TMA producer: one elected thread loads 128-byte-swizzled K-slices of A and B into a STAGES-deep
//             shared-memory ring (cp.async.bulk.tensor, mbarrier complete_tx), continuously across tiles
//   warp 1    allocates 2 x BN TMEM columns (two accumulators); one thread issues tcgen05.mma (M=128, N=BN,
//             kind::f16 or kind::f8f6f4) from shared-memory descriptors; tcgen05.commit frees each ring slot and
//             signals "accumulator full"; it waits for "accumulator empty" before reusing a buffer
//   warps 2-5 epilogue: tcgen05.ld of the accumulator (one TMEM lane = one output row per thread), scales,
//             optional SwiGLU over (8 gate, 8 up) row groups of the weight, 16-byte bf16 / fp32 /
//             fp32-accumulate stores; then it releases the buffer, so it overlaps the next tile's main loop
// Every mbarrier wait is bounded; a wait that runs out sets an error word and the CTA stops issuing work (and
// frees its TMEM), so a broken pipeline returns an error to the host instead of hanging the GPU.
// No TMA multicast is used.
// Reference counterparts: code/fork/kernels/fp8_w8a8.cu:134-219 (CUTLASS SM120 W8A8 GEMM) and
// code/fork/kernels/fp8_large_m.cu (dequant + GEMM for large M).
#include <cuda.h>
#include <algorithm>
#include "common.cuh"
#include "launchers.h"

namespace g53 {

constexpr int kBM = 128;
constexpr uint32_t kSpinLimit = 1u << 26;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// bounded wait: returns false (and records `code`) when the limit is reached or another thread already failed
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* fail, int* err, int code) {
  uint32_t n = 0;
  while (!mbar_try_wait(bar, parity)) {
    if (*fail) return false;
    if (++n > kSpinLimit) {
      *fail = 1;
      atomicExch(err, code);
      return false;
    }
    if (n > 64) __nanosleep(64);
  }
  return true;
}

// 3-D tiled load (k, row, batch); x = k is a multiple of the 128-byte box row, so it is 16-byte aligned
__device__ __forceinline__ void tma_load_3d(const CUtensorMap* map, uint64_t* bar, void* dst, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// UMMA shared-memory descriptor: K-major operand, 128-byte swizzle, 8-row groups 1024 bytes apart
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;                     // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;           // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                     // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                     // layout: 128-byte swizzle
  return d;
}

// instruction descriptor: D f32, A/B format, both K-major, N and M
__device__ __forceinline__ uint32_t umma_idesc(int fmt_ab, int n, int m) {
  uint32_t d = 0;
  d |= 1u << 4;                                // D = f32
  d |= (uint32_t)fmt_ab << 7;                  // A format
  d |= (uint32_t)fmt_ab << 10;                 // B format
  d |= (uint32_t)(n >> 3) << 17;
  d |= (uint32_t)(m >> 4) << 24;
  return d;
}

template <bool FP8>
__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  if constexpr (FP8) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.u32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
  } else {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.u32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
  }
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void named_bar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// tile t of the persistent schedule -> (m0, n0): bands of kGroupM M-tiles, N-tiles walked inside a band, so the
// CTAs resident at one time share a few A row-blocks and a few B column-blocks in L2
constexpr int kGroupM = 8;
__device__ __forceinline__ void tile_coords(int t, int MT, int NT, int BN, int& m0, int& n0, int mrot = 0) {
  const int band = t / (kGroupM * NT);
  const int gm = min(kGroupM, MT - band * kGroupM);
  const int idx = t - band * kGroupM * NT;
  m0 = ((band * kGroupM + idx % gm + mrot) % MT) * kBM;    // all-gather: start at this rank's own rows
  n0 = (idx / gm) * BN;
}

// 32 accumulator columns of one row -> output (scales, mode); vectorised 16-byte stores when the row is aligned
__device__ __forceinline__ void store_chunk(const GemmArgs& p, void* ybase, const float* bscale, int row, int nb,
                                            float rs, const float (&v)[32]) {
  const bool full = p.vec && nb + 32 <= p.N;
  float sc[32];
  if (bscale && full) {
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      const float4 t = *reinterpret_cast<const float4*>(bscale + nb + i);
      sc[i] = t.x; sc[i + 1] = t.y; sc[i + 2] = t.z; sc[i + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) sc[i] = (bscale && nb + i < p.N) ? bscale[nb + i] : 1.f;
  }
  if (p.mode == GEMV_SWIGLU) {
    // columns: two groups of (8 gate rows, 8 matching up rows) of the interleaved weight -> 16 outputs
    __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(ybase) + (int64_t)row * p.ldy + (nb >> 1);
    float o[16];
#pragma unroll
    for (int g = 0; g < 2; ++g)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float gv = round_bf16(v[g * 16 + i] * rs * sc[g * 16 + i]);
        float uv = round_bf16(v[g * 16 + 8 + i] * rs * sc[g * 16 + 8 + i]);
        gv = fminf(gv, p.limit);
        uv = fminf(fmaxf(uv, -p.limit), p.limit);
        o[g * 8 + i] = siluf_(gv) * uv;
      }
    if (full) {
      uint32_t w[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        __nv_bfloat162 b = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
        w[i] = *reinterpret_cast<uint32_t*>(&b);
      }
      reinterpret_cast<uint4*>(y)[0] = make_uint4(w[0], w[1], w[2], w[3]);
      reinterpret_cast<uint4*>(y)[1] = make_uint4(w[4], w[5], w[6], w[7]);
    } else {
#pragma unroll
      for (int g = 0; g < 2; ++g)
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (nb + g * 16 + 8 + i < p.N) y[g * 8 + i] = f2bf(o[g * 8 + i]);
    }
    return;
  }
  const int64_t off = (int64_t)row * p.ldy + nb;
  if (p.mode == GEMV_BF16) {
    __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(ybase) + off;
    if (full) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int j = c * 8 + 2 * i;
          __nv_bfloat162 b = __floats2bfloat162_rn(v[j] * rs * sc[j], v[j + 1] * rs * sc[j + 1]);
          w[i] = *reinterpret_cast<uint32_t*>(&b);
        }
        reinterpret_cast<uint4*>(y)[c] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (nb + i < p.N) y[i] = f2bf(v[i] * rs * sc[i]);
    }
    return;
  }
  float* y = reinterpret_cast<float*>(ybase) + off;
  const bool acc = p.mode == GEMV_F32_ACC;
  const int64_t poff = p.push_rank * p.push_slot + off;       // this rank's slot in every receive buffer
  if (full) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float4 o = make_float4(v[4 * c] * rs * sc[4 * c], v[4 * c + 1] * rs * sc[4 * c + 1],
                             v[4 * c + 2] * rs * sc[4 * c + 2], v[4 * c + 3] * rs * sc[4 * c + 3]);
      if (acc) {
        const float4 old = reinterpret_cast<const float4*>(y)[c];
        o.x += old.x; o.y += old.y; o.z += old.z; o.w += old.w;
      }
      reinterpret_cast<float4*>(y)[c] = o;
      for (int j = 0; j < p.push_world; ++j) reinterpret_cast<float4*>(p.push_ptrs[j] + poff)[c] = o;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if (nb + i >= p.N) break;
      const float val = v[i] * rs * sc[i];
      const float o = acc ? y[i] + val : val;
      y[i] = o;
      for (int j = 0; j < p.push_world; ++j) p.push_ptrs[j][poff + i] = o;
    }
  }
}

// Persistent kernel: gridDim.x CTAs (at most one per SM) walk the output tiles in the grouped order; the TMEM
// holds two 128 x BN accumulators so the epilogue of one tile overlaps the main loop of the next.
// Tensor maps of one launch.  All-gather + GEMM (ag_world > 0): A is row-sharded over the ranks of a group and
// a[j] maps rank j's shard (its memory, reached over NVLink: plain TMA loads, no multicast); output rows
// [j * ag_rows, (j + 1) * ag_rows) come from shard j.
constexpr int kMaxAg = 8;
struct GemmMaps {
  CUtensorMap a[kMaxAg];
  CUtensorMap b;
};

template <int BN, bool FP8, int STAGES>
__global__ void __launch_bounds__(192, 1) gemm_sm100_kernel(const __grid_constant__ GemmMaps maps, GemmArgs p) {
  constexpr int BK = FP8 ? 128 : 64;               // one 128-byte swizzle row per operand row
  constexpr int A_BYTES = kBM * 128;
  constexpr int B_BYTES = BN * 128;
  constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr int UK = FP8 ? 32 : 16;                // K per tcgen05.mma
  constexpr uint32_t TMEM_COLS = 2 * BN;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t tfull[2];
  __shared__ __align__(8) uint64_t tempty[2];
  __shared__ uint32_t tmem_base;
  __shared__ volatile int fail;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int MT = (p.M + kBM - 1) / kBM, NT = (p.N + BN - 1) / BN, per_batch = MT * NT;
  const int tiles = per_batch * max(p.batch, 1);
  const int nk = (p.K + BK - 1) / BK;
  const int mrot = p.ag_world > 0 ? p.ag_rank * (p.ag_rows / kBM) : 0;

  if (threadIdx.x == 0) {
    fail = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);                    // one arrival per epilogue warp
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      int kbg = 0;
      for (int t = blockIdx.x; t < tiles && !fail; t += gridDim.x) {
        int m0, n0;
        const int bz = t / per_batch;
        tile_coords(t - bz * per_batch, MT, NT, BN, m0, n0, mrot);
        const CUtensorMap* ma = &maps.a[0];
        int am0 = m0;
        if (p.ag_world > 0) {
          const int owner = m0 / p.ag_rows;
          if (owner == p.ag_rank) {
            ma = &maps.a[0];                          // this rank's own shard
            am0 = m0 - owner * p.ag_rows;
          } else {
            // a peer's row block, copied once into the local staging buffer by the epilogue warps of some CTA
            ma = &maps.a[1];
            if (!wait_flag_geq(reinterpret_cast<const unsigned*>(p.ag_ready) + m0 / kBM, (unsigned)kBM * p.ag_target,
                               p.err, 5)) {
              fail = 1;
              break;
            }
            asm volatile("fence.proxy.async.global;" ::: "memory");
          }
        }
        for (int kb = 0; kb < nk; ++kb, ++kbg) {
          const int s = kbg % STAGES;
          const uint32_t ph = (kbg / STAGES) & 1;
          if (kbg >= STAGES && !mbar_wait(&empty_bar[s], ph ^ 1, &fail, p.err, 1)) break;
          uint8_t* a_dst = smem + s * STAGE_BYTES;
          uint8_t* b_dst = a_dst + A_BYTES;
          mbar_expect_tx(&full_bar[s], STAGE_BYTES);
          tma_load_3d(ma, &full_bar[s], a_dst, kb * BK, am0, bz);
          tma_load_3d(&maps.b, &full_bar[s], b_dst, kb * BK, n0, bz);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc(FP8 ? 0 : 1, BN, kBM);
      int kbg = 0, it = 0;
      for (int t = blockIdx.x; t < tiles && !fail; t += gridDim.x, ++it) {
        const int buf = it & 1;
        if (it >= 2 && !mbar_wait(&tempty[buf], ((it >> 1) & 1) ^ 1, &fail, p.err, 4)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d = tmem + (uint32_t)(buf * BN);
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb, ++kbg) {
          const int s = kbg % STAGES;
          const uint32_t ph = (kbg / STAGES) & 1;
          if (!mbar_wait(&full_bar[s], ph, &fail, p.err, 2)) { ok = false; break; }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t a_addr = smem_u32(smem + s * STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / UK; ++k) {
            const uint32_t koff = k * UK * (FP8 ? 1 : 2);    // bytes along the swizzled row
            umma<FP8>(d, umma_desc_sw128(a_addr + koff), umma_desc_sw128(b_addr + koff), idesc,
                      (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[s]);
        }
        if (!ok) break;
        umma_commit(&tfull[buf]);
      }
    }
  } else {
    // epilogue warps 2..5 -> TMEM lane quadrant (warp % 4)
    const int quad = warp & 3;
    if (p.ag_world > 0) {
      // all-gather: before their first tile, the 4 epilogue warps of every CTA copy a share of the peers' rows over
      // NVLink into the local staging buffer (each remote row crosses once), 4 rows (16 x 16-byte loads in flight
      // per thread) at a time, and count the copied rows of each 128-row block (ready[block] reaches 128 x target)
      const int et = threadIdx.x - 64;              // 0..127
      const int per_shard = p.ag_rows / kBM;
      const int vec = p.K / 8;                       // 16-byte vectors per row
      const int units = (p.ag_world - 1) * p.ag_rows / 4;
      int seen = -1;                                 // owner whose publish flag was observed
      for (int u = blockIdx.x; u < units && !fail; u += gridDim.x) {
        const int rr = u * 4;                        // row among the remote rows (peer order, skipping this rank)
        int owner = rr / p.ag_rows;
        owner += owner >= p.ag_rank ? 1 : 0;
        const int orow = rr % p.ag_rows;             // row within the owner's shard
        if (owner != seen) {
          if (et == 0 && !wait_flag_geq(p.ag_flags + owner, p.ag_target, p.err, 6)) fail = 1;
          named_bar(1, 128);
          seen = owner;
          if (fail) break;
        }
        const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(p.ag_ptrs_dev[owner]) + (int64_t)orow * p.lda;
        const int grow = owner * p.ag_rows + orow;  // row of the gathered matrix
        __nv_bfloat16* dst = p.ag_stage + (int64_t)grow * p.K;
        for (int i0 = et; i0 < 4 * vec; i0 += 128 * 16) {
          uint4 v[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const int j = i0 + k * 128;
            if (j < 4 * vec) v[k] = *reinterpret_cast<const uint4*>(src + (int64_t)(j / vec) * p.lda + (j % vec) * 8);
          }
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const int j = i0 + k * 128;
            if (j < 4 * vec) *reinterpret_cast<uint4*>(dst + (int64_t)(j / vec) * p.K + (j % vec) * 8) = v[k];
          }
        }
        // generic-proxy stores -> visible to the TMA (async proxy) loads of other CTAs, then counted
        asm volatile("fence.proxy.async.global;" ::: "memory");
        __threadfence();
        named_bar(1, 128);
        if (et == 0) atomicAdd(reinterpret_cast<unsigned*>(p.ag_ready) + grow / kBM, 4u);
      }
      (void)per_shard;
    }
    int it = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++it) {
      const int buf = it & 1;
      int m0, n0;
      const int bz = t / per_batch;
      tile_coords(t - bz * per_batch, MT, NT, BN, m0, n0, mrot);
      void* ybase = reinterpret_cast<uint8_t*>(p.y) +
                    bz * p.bsy * ((p.mode == GEMV_F32 || p.mode == GEMV_F32_ACC) ? 4 : 2);
      const float* bscale = p.b_scale ? p.b_scale + bz * p.bss : nullptr;
      int okw = 0;
      if (lane == 0) okw = mbar_wait(&tfull[buf], (it >> 1) & 1, &fail, p.err, 3) ? 1 : 0;
      const bool ok = __shfl_sync(0xffffffffu, okw, 0) != 0;     // warp-uniform: tcgen05.ld is .sync.aligned
      if (!ok) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int row = m0 + quad * 32 + lane;
      const float rs = (p.a_scale && row < p.M) ? p.a_scale[row] : 1.f;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * BN + c0), v);
        if (row < p.M && n0 + c0 < p.N) store_chunk(p, ybase, bscale, row, n0 + c0, rs, v);
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
  if (p.push_world > 0 && threadIdx.x == 0) {
    // every row of this CTA is stored in the peers' slots: count in; the last CTA releases the flags
    __threadfence_system();
    const unsigned prev = atomicAdd(p.push_done, 1u);
    if (prev == gridDim.x - 1) {
      *p.push_done = 0u;
      __threadfence_system();
      for (int j = 0; j < p.push_world; ++j) red_release_sys_add(p.push_flags[j] + p.push_rank, 1u);
    }
  }
}

// per-row e4m3 quantisation of bf16 activations: scale = amax / 448
__global__ void __launch_bounds__(256) quant_rows_e4m3_kernel(const __nv_bfloat16* x, int64_t ldx, int K,
                                                              uint8_t* q, float* scale) {
  const int r = blockIdx.x;
  __shared__ float red[32];
  float amax = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) amax = fmaxf(amax, fabsf(bf2f(x[(int64_t)r * ldx + k])));
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  float m = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) m = fmaxf(m, red[i]);
  const float s = fmaxf(m, 1e-8f) / 448.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const __nv_fp8_e4m3 v(bf2f(x[(int64_t)r * ldx + k]) / s);
    q[(int64_t)r * K + k] = v.__x;
  }
  if (threadIdx.x == 0) scale[r] = s;
}

// exact e4m3 -> bf16 widening of a weight matrix (16 bytes in, 32 bytes out per thread-iteration)
__global__ void e4m3_to_bf16_kernel(const uint8_t* w, int64_t n16, __nv_bfloat16* out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 v = reinterpret_cast<const uint4*>(w)[i];
    const uint32_t ws[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t h01 = e4m3x2_to_f16x2((uint16_t)(ws[k] & 0xffffu));
      const uint32_t h23 = e4m3x2_to_f16x2((uint16_t)(ws[k] >> 16));
      const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&h01));
      const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&h23));
      __nv_bfloat162 b01 = __floats2bfloat162_rn(f01.x, f01.y), b23 = __floats2bfloat162_rn(f23.x, f23.y);
      o[2 * k] = *reinterpret_cast<uint32_t*>(&b01);
      o[2 * k + 1] = *reinterpret_cast<uint32_t*>(&b23);
    }
    uint4* dst = reinterpret_cast<uint4*>(out) + 2 * i;
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

}  // namespace g53

using namespace g53;

cudaError_t g53_e4m3_to_bf16(const uint8_t* w, int64_t n, __nv_bfloat16* out, cudaStream_t st) {
  if (n % 16 || (reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
    return cudaErrorInvalidValue;
  const int64_t n16 = n / 16;
  const int blocks = (int)std::min<int64_t>((n16 + 255) / 256, 148 * 16);
  e4m3_to_bf16_kernel<<<blocks, 256, 0, st>>>(w, n16, out);
  return cudaGetLastError();
}

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 3-D K-major tile map: batch x rows x K, box = 1 x box_rows x 128 bytes, 128-byte swizzle
bool make_map(CUtensorMap* m, const void* base, bool fp8, int64_t rows, int64_t K, int64_t ld_elems, int64_t batch,
              int64_t bs_elems, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const int esz = fp8 ? 1 : 2;
  if (batch <= 1) { batch = 1; bs_elems = rows * ld_elems; }
  cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(ld_elems * esz), (cuuint64_t)(bs_elems * esz)};
  cuuint32_t box[3] = {(cuuint32_t)(128 / esz), (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base),
                  dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int BN, bool FP8, int STAGES>
cudaError_t launch(const GemmArgs& p, cudaStream_t st) {
  GemmMaps maps;
  if (p.ag_world > 0) {
    if (p.ag_world > kMaxAg || p.ag_rows % kBM || p.M != p.ag_world * p.ag_rows || p.batch > 1 || FP8 ||
        !p.ag_stage || !p.ag_ready || !p.ag_ptrs_dev || p.K % 8)
      return cudaErrorInvalidValue;
    if (!make_map(&maps.a[0], reinterpret_cast<const void*>(p.ag_ptrs[p.ag_rank]), FP8, p.ag_rows, p.K, p.lda, 1, 0,
                  kBM) ||
        !make_map(&maps.a[1], p.ag_stage, FP8, p.M, p.K, p.K, 1, 0, kBM))
      return cudaErrorInvalidValue;
  } else if (!make_map(&maps.a[0], p.a, FP8, p.M, p.K, p.lda, p.batch, p.bsa, kBM)) {
    return cudaErrorInvalidValue;
  }
  if (!make_map(&maps.b, p.b, FP8, p.N, p.K, p.ldb, p.batch, p.bsb, BN)) return cudaErrorInvalidValue;
  const int smem = STAGES * (kBM * 128 + BN * 128) + 1024;
  auto kern = gemm_sm100_kernel<BN, FP8, STAGES>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  static int sms[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && sms[dev] == 0) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  const int n_sm = (dev < 64 && sms[dev] > 0) ? sms[dev] : 148;
  const int tiles = ((p.M + kBM - 1) / kBM) * ((p.N + BN - 1) / BN) * std::max(p.batch, 1);
  GemmArgs q = p;
  // 16-byte epilogue stores need an aligned output base and row pitch
  const int out_esz = (p.mode == GEMV_F32 || p.mode == GEMV_F32_ACC) ? 4 : 2;
  q.vec = ((reinterpret_cast<uintptr_t>(p.y) & 15) == 0 && ((p.ldy * out_esz) & 15) == 0 &&
           ((p.bsy * out_esz) & 15) == 0 && ((p.bss * 4) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(p.b_scale) & 15) == 0) ? 1 : 0;
  kern<<<std::min(tiles, n_sm), 192, smem, st>>>(maps, q);
  return cudaGetLastError();
}

}  // namespace

cudaError_t g53_gemm_sm100(const GemmArgs& p, cudaStream_t st) {
  // alignment rules of the tensor maps: 16-byte aligned bases and row strides
  const int esz = p.fp8 ? 1 : 2;
  if ((p.ag_world == 0 && (reinterpret_cast<uintptr_t>(p.a) & 15)) || (reinterpret_cast<uintptr_t>(p.b) & 15) ||
      ((p.lda * esz) & 15) || ((p.ldb * esz) & 15) || (p.K * esz) % 16)
    return cudaErrorInvalidValue;
  if (p.batch > 1 && (((p.bsa * esz) & 15) || ((p.bsb * esz) & 15) || p.a_scale)) return cudaErrorInvalidValue;
  if (p.fp8) return p.N >= 256 ? launch<256, true, 4>(p, st) : launch<128, true, 6>(p, st);
  return p.N >= 256 ? launch<256, false, 4>(p, st) : launch<128, false, 6>(p, st);
}

cudaError_t g53_quant_rows_e4m3(const __nv_bfloat16* x, int64_t ldx, int R, int K, uint8_t* q, float* scale,
                                cudaStream_t st) {
  quant_rows_e4m3_kernel<<<R, 256, 0, st>>>(x, ldx, K, q, scale);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}
