// Routed EXL3 MoE for prefill chunks on the 5th-generation tensor cores.
//
// One CTA = (128 output channels of one expert, that expert's token rows).  Swap-AB: the 128 output channels are
// the MMA's M dimension (TMEM lanes) and the expert's tokens (up to 256 per pass) are N (TMEM columns), so the
// weights of an expert are decoded once per pass however many tokens it received.
//
//   warps 0-7   trellis decoders: each 16x16 tile is decoded in registers (ExLlamaV3's mcg codebook, the same
//               arithmetic as moe.cu) and stored to shared memory in the K-major 128-byte-swizzled layout that a
//               UMMA descriptor reads (the lane's fragment registers are (k, k+1) pairs, one 32-bit store each);
//               after the main loop they are the epilogue warps
//   warp 8      TMA producer: rotated activations of the expert's token rows (rows of one expert are contiguous in
//               the sorted pair order) as 64x64 boxes, 128-byte swizzle, no multicast
//   warp 9      TMEM allocation; one thread issues tcgen05.mma kind::f16 (f16 x f16 -> f32) per 16-wide k step
// Stages are handed over with mbarriers (decoders arrive after fence.proxy.async, TMA by complete_tx, the MMA
// frees a stage with tcgen05.commit).  Epilogue per 32 token columns: tcgen05.ld -> shared-memory transpose ->
// per token row: Hadamard-128, * svh, then
//   gate/up  SwiGLU with clamp, * suh of the down projection, Hadamard-128 -> f16 rotated down input
//   down     * routing weight -> fp32 per-pair output
// All waits are bounded (error word + early exit); TMEM is freed on every path.
// Reference counterpart: code/fork/kernels/moe_e4m3.cu:1500 (persistent prefill MoE) and
// code/fork/docs/ref/mia_exl3-fat-kernel (ExLlamaV3 fat grouped kernels).
#include <cuda.h>
#include "common.cuh"
#include "launchers.h"

namespace g53 {
namespace mp {

constexpr uint32_t kSpin = 1u << 26;
// decoder warps: gate/up (two TMEM accumulators = all 512 columns, one CTA per SM) uses 16; down (256 columns,
// two stages) runs two CTAs of 8 decoder warps per SM so one CTA's epilogue overlaps the other's decode
template <bool GU> struct Cfg {
  static constexpr int kDecWarps = GU ? 16 : 8;
  static constexpr int kThreads = (kDecWarps + 2) * 32;
  static constexpr int kStages = 2;
  static constexpr int kMinBlocks = GU ? 1 : 2;
};
constexpr int kNmax = 256;            // tokens per pass
constexpr int kBK = 64;               // k per stage (one 128-byte swizzle row of f16)

__device__ __forceinline__ uint32_t su32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

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
__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t ph, volatile int* fail, int* err, int code) {
  uint32_t n = 0;
  while (!bar_try(b, ph)) {
    if (*fail) return false;
    if (++n > kSpin) { *fail = 1; atomicExch(err, code); return false; }
    if (n > 64) __nanosleep(32);
  }
  return true;
}
__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n)); }

__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
__device__ __forceinline__ uint32_t idesc_f16(int n) {
  // D f32, A f16, B f16 (format 0), K-major both, N, M = 128
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}
__device__ __forceinline__ void mma_f16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile("{\n .reg .pred p;\n setp.ne.u32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
               ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void mma_commit(uint64_t* b) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(b)) : "memory");
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
__device__ __forceinline__ void tma_2d(const CUtensorMap* m, uint64_t* bar, void* dst, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
               ::"r"(su32(dst)), "l"(m), "r"(x), "r"(y), "r"(su32(bar)) : "memory");
}

// mcg trellis decode (same rules as moe.cu): 4 f16x2 fragment registers of lane l from words cur (l) / prev (l-1).
// The window extraction pairs windows b and b + 16 as the decode kernels do (moe.cu, trellis_tile_mma): for any
// 32-bit t holding window b in its low half, s_b * C = t * C - (t >> 16) * (C << 16) (mod 2^32), and t >> 16 is
// window b + 16, so 7 ALU extractions and 12 IMADs give the 8 masked products (instead of 10 ALU extractions and
// 8 IMADs); the two fp16 halves of each product are then added (one HADD2 per two values) as the format specifies.
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
__device__ __forceinline__ uint32_t mcg_mask_(uint32_t x) {       // (x & 0x8FFF8FFF) ^ 0x3B603B60, one LOP3
  uint32_t r;
  asm("lop3.b32 %0, %1, 0x8FFF8FFF, 0x3B603B60, 0x6a;" : "=r"(r) : "r"(x));
  return r;
}
// (fp16(lo0) + fp16(hi0), fp16(lo1) + fp16(hi1)) of two masked products
__device__ __forceinline__ uint32_t mcg_sum2(uint32_t x0, uint32_t x1) {
  const uint32_t lo = prmt_<0x5410>(x0, x1), hi = prmt_<0x7632>(x0, x1);
  __half2 r = __hadd2(*reinterpret_cast<const __half2*>(&lo), *reinterpret_cast<const __half2*>(&hi));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ void frags(uint32_t cur, uint32_t prev, uint32_t (&b)[4]) {
  constexpr uint32_t C = 0xCBAC1FEDu, Cn = 0u - (C << 16);
  const uint32_t s16 = prmt_<0x4432>(cur, 0u);          // stream bits [16, 32) above cur's LSB
  const uint32_t t8 = prmt_<0x4321>(cur, prev);         // [8, 40)
  const uint32_t s24 = prmt_<0x4432>(t8, 0u);           // [24, 40)
  const uint32_t t4 = shf_r_<4>(cur, prev);             // [4, 36)
  const uint32_t s20 = prmt_<0x4432>(t4, 0u);           // [20, 36)
  const uint32_t t12 = shf_r_<12>(cur, prev);           // [12, 44)
  const uint32_t s28 = prmt_<0x4432>(t12, 0u);          // [28, 44)
  b[0] = mcg_sum2(mcg_mask_(s28 * C), mcg_mask_(s24 * C));
  b[1] = mcg_sum2(mcg_mask_(s20 * C), mcg_mask_(s16 * C));
  b[2] = mcg_sum2(mcg_mask_(t12 * C + s28 * Cn), mcg_mask_(t8 * C + s24 * Cn));
  b[3] = mcg_sum2(mcg_mask_(t4 * C + s20 * Cn), mcg_mask_(cur * C + s16 * Cn));
}

__device__ __forceinline__ void stsm_x4(uint32_t addr, const uint32_t (&r)[4]) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(r[0]), "r"(r[1]),
               "r"(r[2]), "r"(r[3])
               : "memory");
}

// byte offset of element (row, k) (k even) in a 128-row x 64-k f16 tile, K-major, 128-byte swizzle
__device__ __forceinline__ uint32_t sw_off(int row, int k) {
  return (uint32_t)(row * 128 + ((((k * 2) >> 4) ^ (row & 7)) << 4) + ((k * 2) & 15));
}

// expert parallelism: the last CTA of the down launch (every output row stored into the source ranks' combine
// buffers and made visible system-wide) releases one flag on every source rank
__device__ __forceinline__ void ep_count_in(const MoePrefillArgs& p) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned prev = atomicAdd(p.done, 1u);
    if (prev == gridDim.x * gridDim.y * gridDim.z - 1) {
      *p.done = 0u;
      __threadfence_system();
      for (int s = 0; s < p.push_world; ++s) red_release_sys_add(reinterpret_cast<unsigned*>(p.push_flags[s]), 1u);
    }
  }
}

template <bool GU>
__global__ void __launch_bounds__(Cfg<GU>::kThreads, Cfg<GU>::kMinBlocks) moe_prefill_kernel(const __grid_constant__ CUtensorMap tb0,
                                                                  const __grid_constant__ CUtensorMap tb1,
                                                                  MoePrefillArgs p) {
  constexpr int NM = GU ? 2 : 1;                       // weight matrices
  constexpr int STAGES = Cfg<GU>::kStages;
  constexpr int kDecWarps = Cfg<GU>::kDecWarps;
  constexpr int A_BYTES = 128 * 128;                   // 128 rows x 64 f16
  constexpr int B_BYTES = kNmax * 128;                 // 256 token rows x 64 f16
  constexpr int STAGE = NM * (A_BYTES + B_BYTES);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t a_full[STAGES], b_full[STAGES], empty[STAGES], acc_full, tmem_free;
  __shared__ uint32_t tmem_base;
  __shared__ volatile int fail;

  const int u = blockIdx.y;
  if (u >= p.group_count[0] || u >= p.max_groups) {
    if (!GU && p.out_ptrs) ep_count_in(p);          // expert parallelism: every CTA counts towards the release
    return;
  }
  const int e = p.group_expert[u];
  if (!g53_in_bounds(e, p.n_experts, 6)) {
    if (!GU && p.out_ptrs) ep_count_in(p);
    return;
  }
  const int p0 = p.group_offset[u];
  const int np = p.group_offset[u + 1] - p0;
  const int nb = blockIdx.x;                            // 128-channel output block
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KT = p.K / 16, NT = p.N / 16;
  const int nkb = p.K / kBK;
  const int passes = (np + kNmax - 1) / kNmax;

  if (threadIdx.x == 0) {
    fail = 0;
    for (int s = 0; s < STAGES; ++s) {
      bar_init(&a_full[s], kDecWarps);
      bar_init(&b_full[s], 1);
      bar_init(&empty[s], 1);
    }
    bar_init(&acc_full, 1);
    bar_init(&tmem_free, kDecWarps);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kDecWarps + 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_base)),
                 "r"((uint32_t)(NM * kNmax)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;

  if (warp < kDecWarps) {
    // ------------------------------------------------------------------ decoders, then epilogue
    constexpr int TILES = NM * 4 * 8;                   // (matrix, k-tile, n-tile) of one stage
    constexpr int PER = TILES / kDecWarps;
    const int src = (lane + 31) & 31;
    // The warp's PER tiles of a stage, tile i = (matrix idx / 32, k-tile (idx / 8) % 4, n-tile idx % 8) with
    // idx = warp + i * kDecWarps, are the same in every stage: their trellis word addresses advance by one stage
    // of k-tiles (4 * NT tiles of 32 words) and their shared-memory offsets repeat.  Both are formed once here, so
    // the decode loop is the trellis arithmetic, one load and four stores per tile.
    // the expert's words of both matrices; tile i's word within them (u32: an expert holds KT * NT * 32 words)
    const uint32_t* wb0 = reinterpret_cast<const uint32_t*>(p.tr0) + (int64_t)e * KT * NT * 32;
    const uint32_t* wb1 = reinterpret_cast<const uint32_t*>(p.tr1) + (int64_t)e * KT * NT * 32;
    uint32_t wo[PER];                                   // word offset of tile i in stage 0
    uint32_t so[PER];                                   // byte offset of this lane's stmatrix row of tile i
    const uint32_t kstep = 4u * NT * 32u;               // words per stage of k-tiles
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int idx = warp + i * kDecWarps;
      const int m = idx / 32, kt = (idx / 8) & 3, nt = idx & 7;
      wo[i] = (uint32_t)((kt * NT + nb * 8 + nt) * 32 + lane);
      // stmatrix x4: lane l addresses row l % 8 of 8 x 8 block l / 8; blocks 0..3 = (rows 0-7 | 8-15) x
      // (k 0-7 | 8-15) of the 16 x 16 tile, in the order of the fragment registers b[0..3]
      const int mrow = nt * 16 + (lane & 7) + ((lane >> 4) & 1) * 8, mk = kt * 16 + ((lane >> 3) & 1) * 8;
      so[i] = (uint32_t)(m * A_BYTES) + sw_off(mrow, mk);
    }
    const uint32_t sbase = su32(sm);
    int it = 0;                                         // global stage counter (continues across passes)
    for (int pass = 0; pass < passes; ++pass) {
      const int rows = min(kNmax, np - pass * kNmax);
      uint32_t koff = 0;                                // every pass decodes the same K range from stage 0
      auto load = [&](uint32_t (&w)[PER]) {            // the stage at koff, then advance koff one stage
#pragma unroll
        for (int i = 0; i < PER; ++i) {
          // matrix of tile i: (warp + i * kDecWarps) / 32 = i * kDecWarps / 32, a constant (warp < kDecWarps <= 16)
          constexpr int kDW = kDecWarps;
          const bool m1 = NM > 1 && (i * kDW) / 32 > 0;
          w[i] = ldg_nc_u32((m1 ? wb1 : wb0) + (wo[i] + koff));
        }
        koff += kstep;
      };
      uint32_t wcur[PER], wnext[PER];                   // trellis words of this stage and the next
      load(wcur);
      if (nkb > 1) load(wnext);
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        uint32_t wnext2[PER];                           // two stages ahead of the decode
        if (kb + 2 < nkb) load(wnext2);
        if (it >= STAGES) {
          int okw = 0;
          if (lane == 0) okw = bar_wait(&empty[s], ph ^ 1, &fail, p.err, 11) ? 1 : 0;
          if (!__shfl_sync(0xffffffffu, okw, 0)) break;
        }
        const uint32_t ab = sbase + (uint32_t)(s * STAGE);
#pragma unroll
        for (int i = 0; i < PER; ++i) {
          uint32_t b[4];
          frags(wcur[i], __shfl_sync(0xffffffffu, wcur[i], src), b);
          // b[0..3] hold (row g, k 2q..2q+1) of the blocks (n0, k0), (n0, k0 + 8), (n0 + 8, k0), (n0 + 8, k0 + 8):
          // the mma fragment layout that stmatrix stores, each block row a 16-byte chunk of the swizzled tile
          stsm_x4(ab + so[i], b);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) bar_arrive(&a_full[s]);
#pragma unroll
        for (int i = 0; i < PER; ++i) { wcur[i] = wnext[i]; wnext[i] = wnext2[i]; }
      }
      // ---- epilogue of this pass
      int okw = 0;
      if (lane == 0) okw = bar_wait(&acc_full, pass & 1, &fail, p.err, 12) ? 1 : 0;
      const bool ok = __shfl_sync(0xffffffffu, okw, 0) != 0;
      __syncwarp();
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      float* zb = reinterpret_cast<float*>(sm);          // [2][32][132] transposition buffer (stages are idle)
      constexpr int ZS = 132;                            // row stride: 16-byte aligned rows, conflict-free stores
      const int quad = warp & 3, half = (warp >> 2) & 1;
      for (int c0 = 0; c0 < rows; c0 += 32) {
        if (ok && warp < 8) {                            // warps 0-7 read TMEM (4 lane quadrants x 2 halves)
          float v[32];
          if (GU) {
            // warps 0-3: gate columns, warps 4-7: up columns
            tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + half * kNmax + c0, v);
#pragma unroll
            for (int j = 0; j < 32; ++j) zb[(half * 32 + j) * ZS + quad * 32 + lane] = v[j];
          } else {
            // warps 0-3: columns c0.., warps 4-7: columns c0+32..
            tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + c0 + half * 32, v);
#pragma unroll
            for (int j = 0; j < 32; ++j) zb[(half * 32 + j) * ZS + quad * 32 + lane] = v[j];
          }
        }
        named_sync(1, kDecWarps * 32);
        const int ncols = GU ? min(32, rows - c0) : min(64, rows - c0);
        for (int j = warp; j < ncols; j += kDecWarps) {
          const int pr = p0 + pass * kNmax + c0 + j;        // sorted pair row
          const int col = nb * 128 + lane * 4;
          if (GU) {
            float vg[4], vu[4];
            const float4 g4 = *reinterpret_cast<const float4*>(&zb[j * ZS + lane * 4]);
            const float4 u4 = *reinterpret_cast<const float4*>(&zb[(32 + j) * ZS + lane * 4]);
            vg[0] = g4.x; vg[1] = g4.y; vg[2] = g4.z; vg[3] = g4.w;
            vu[0] = u4.x; vu[1] = u4.y; vu[2] = u4.z; vu[3] = u4.w;
            fwht128_warp_fma(vg);
            fwht128_warp_fma(vu);
            float act[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              float gv = vg[i] * __half2float(p.svh0[(int64_t)e * p.N + col + i]);
              float uv = vu[i] * __half2float(p.svh1[(int64_t)e * p.N + col + i]);
              gv = fminf(gv, p.limit);
              uv = fminf(fmaxf(uv, -p.limit), p.limit);
              act[i] = siluf_(gv) * uv * __half2float(p.suh_next[(int64_t)e * p.N + col + i]);
            }
            fwht128_warp_fma(act);
            __half2* o = reinterpret_cast<__half2*>(reinterpret_cast<__half*>(p.out) + (int64_t)pr * p.N + col);
            o[0] = __floats2half2_rn(act[0], act[1]);
            o[1] = __floats2half2_rn(act[2], act[3]);
          } else {
            float v[4];
            const float4 v4 = *reinterpret_cast<const float4*>(&zb[j * ZS + lane * 4]);
            v[0] = v4.x; v[1] = v4.y; v[2] = v4.z; v[3] = v4.w;
            fwht128_warp_fma(v);
            const float w = p.pair_w[pr];
            float4 o;
            o.x = v[0] * __half2float(p.svh0[(int64_t)e * p.N + col + 0]) * w;
            o.y = v[1] * __half2float(p.svh0[(int64_t)e * p.N + col + 1]) * w;
            o.z = v[2] * __half2float(p.svh0[(int64_t)e * p.N + col + 2]) * w;
            o.w = v[3] * __half2float(p.svh0[(int64_t)e * p.N + col + 3]) * w;
            float* dst = p.out_ptrs ? reinterpret_cast<float*>(p.out_ptrs[pr])       // the source rank's row
                                    : reinterpret_cast<float*>(p.out) + (int64_t)pr * p.N;
            *reinterpret_cast<float4*>(dst + col) = o;
          }
        }
        named_sync(1, kDecWarps * 32);
        if (!GU) c0 += 32;                               // down consumed 64 columns in this step
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) bar_arrive(&tmem_free);
      if (!ok) break;
    }
  } else if (warp == kDecWarps) {
    // ------------------------------------------------------------------ TMA producer (B: token rows)
    if (lane == 0) {
      int it = 0;
      for (int pass = 0; pass < passes; ++pass) {
        const int rows = min(kNmax, np - pass * kNmax);
        const int boxes = (rows + 63) / 64;
        // the epilogue of the previous pass uses the stage buffers as its transposition buffer
        if (pass > 0 && !bar_wait(&tmem_free, (pass - 1) & 1, &fail, p.err, 17)) break;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (it >= STAGES && !bar_wait(&empty[s], ph ^ 1, &fail, p.err, 13)) break;
          uint8_t* bbase = sm + s * STAGE + NM * A_BYTES;
          bar_expect_tx(&b_full[s], (uint32_t)(NM * boxes * 64 * 128));
          for (int bx = 0; bx < boxes; ++bx) {
            const int row = p0 + pass * kNmax + bx * 64;
            tma_2d(&tb0, &b_full[s], bbase + bx * 64 * 128, kb * kBK, row);
            if (GU) tma_2d(&tb1, &b_full[s], bbase + B_BYTES + bx * 64 * 128, kb * kBK, row);
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int it = 0;
      for (int pass = 0; pass < passes && !fail; ++pass) {
        const int rows = min(kNmax, np - pass * kNmax);
        const int n = (rows + 15) / 16 * 16;
        const uint32_t idesc = idesc_f16(n);
        if (pass > 0 && !bar_wait(&tmem_free, (pass - 1) & 1, &fail, p.err, 14)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        bool broke = false;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!bar_wait(&a_full[s], ph, &fail, p.err, 15) || !bar_wait(&b_full[s], ph, &fail, p.err, 16)) {
            broke = true;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t a0 = su32(sm + s * STAGE);
          const uint32_t b0 = a0 + NM * A_BYTES;
#pragma unroll
          for (int m = 0; m < NM; ++m) {
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k) {
              mma_f16(tmem + m * kNmax, desc_sw128(a0 + m * A_BYTES + k * 32), desc_sw128(b0 + m * B_BYTES + k * 32),
                      idesc, (kb > 0 || k > 0) ? 1u : 0u);
            }
          }
          mma_commit(&empty[s]);
        }
        mma_commit(&acc_full);
        if (broke) break;
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == kDecWarps + 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)(NM * kNmax)));
  }
  if (!GU && p.out_ptrs) ep_count_in(p);
}

}  // namespace mp
}  // namespace g53

using namespace g53;

namespace {
typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                             const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                             CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeFn enc() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(ptr);
  }
  return fn;
}
bool act_map(CUtensorMap* m, const void* base, int64_t rows, int64_t K) {
  EncodeFn fn = enc();
  if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) || (K * 2) % 16) return false;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(K * 2)};
  cuuint32_t box[2] = {64, 64};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

cudaError_t g53_moe_prefill(const MoePrefillArgs& p, bool gate_up, cudaStream_t st) {
  using namespace g53::mp;
  if (p.K % kBK || p.N % 128) return cudaErrorInvalidValue;
  CUtensorMap t0, t1;
  if (!act_map(&t0, p.x0, p.rows, p.K)) return cudaErrorInvalidValue;
  if (gate_up && !act_map(&t1, p.x1, p.rows, p.K)) return cudaErrorInvalidValue;
  if (!gate_up) t1 = t0;
  const int NM = gate_up ? 2 : 1, STAGES = gate_up ? Cfg<true>::kStages : Cfg<false>::kStages;
  const int smem = STAGES * NM * (128 * 128 + kNmax * 128) + 1024;
  dim3 grid(p.N / 128, p.max_groups);
  cudaError_t e;
  if (gate_up) {
    e = cudaFuncSetAttribute(moe_prefill_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    moe_prefill_kernel<true><<<grid, Cfg<true>::kThreads, smem, st>>>(t0, t1, p);
  } else {
    e = cudaFuncSetAttribute(moe_prefill_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    moe_prefill_kernel<false><<<grid, Cfg<false>::kThreads, smem, st>>>(t0, t1, p);
  }
  return cudaGetLastError();
}
