// Sparse MLA attention over the fp8 latent cache (absorbed form, no rope) on the 5th-generation tensor cores.
//
// One work item = one query row r (all H heads of this rank) and one range of its DSA-selected keys.  The keys are
// gathered through the selection list in tiles of 128 (the MMA's M side), the heads sit on the N side (H padded to
// HN = 16, 32 or 64), so the same kernel serves every tensor-parallel size:
//
//   S^T[key, head] = K8[key, :] . Q[head, :]          kind::f8f6f4, A = key tile (K-major), B = Q (K-major)
//   O^T[dim, head] += V8[key, dim]^T . P^T[key, head]  kind::f8f6f4, A = the same key tile read MN-major (V = K:
//                                                      the latent row is both key and value), B = P^T (K-major)
//
// Numerics: the cached keys/values are used exactly (e4m3 with one fp32 scale per token).  The queries and the
// probabilities are each carried as two e4m3 terms, x = hi + lo with hi = e4m3(x), lo = e4m3(x - hi) (about 8
// significant bits, the precision of bf16), each term one MMA: queries with one scale per head (max |q| -> 448),
// probabilities times the key scale with one scale per work item (the item's largest key scale -> 256 / 2^tau).
// Softmax runs in fp32 in the log2 domain.  A head's running maximum is raised only when a tile exceeds it by more
// than tau = 0.75 (probabilities then stay below 2^tau); a raise rescales that head's O^T column in TMEM and its
// partial sums before the next PV.  The row sums are kept per thread in fp32 and reduced once per item.
//
// Warp roles (352 threads, one CTA per SM, persistent over work items):
//   warps 0-1   producers: per item the queries (two e4m3 terms, swizzled K-major; loads of the next item are issued
//               while the current one finishes) and the largest key scale; per tile two key rows per thread
//               gathered through the selection list with cp.async into the 128-byte-swizzled tile (zero rows past
//               the range), plus the key scales
//   warp 2      TMEM owner and MMA issuer: polls the readiness of the next QK (key tile landed, S buffer free) and of
//               the oldest pending PV (P written) and issues whichever is ready, so the tensor core never waits on
//               a key gather for a PV
//   warps 3-10  softmax / correction / epilogue: TMEM lane = key (S^T) or latent dim (O^T); two warps per lane
//               quadrant, each owning half of the head columns; per-head column maxima by a butterfly
//               transpose-reduction inside the warp, then across the 4 quadrants in shared memory
// Every wait is bounded (mbarrier polls; the softmax warps leave their loops together right after a named barrier,
// on a stop flag sampled before it), so a wait that runs out records an error code, the CTA frees its TMEM and exits.
// Reference counterpart: the sparse MLA prefill kernel (code/fork/kernels/mla_prefill/mla_prefill_kernel.cuh:176,
// one CTA per query token over the selected keys) and FlashInfer's sparse MLA decode used for decode
// (code/fork/docs/MLA_PREFILL.md:23-28).
#include <algorithm>
#include <cuda_fp8.h>
#include "common.cuh"
#include "launchers.h"
#include "tc05.cuh"

namespace g53 {
namespace mtc {

constexpr int kKeys = 128;                     // keys per tile (M)
constexpr int kL = 512;                        // latent dims
constexpr int kStages = 2;                     // key tiles in flight
constexpr int kTile = kKeys * kL;              // bytes of a key tile (e4m3)
constexpr int kBlk = kKeys * 128;              // bytes of one 128-dim block of a key tile
constexpr int kProd = 64;                      // producer threads (warps 0-1)
constexpr int kMmaWarp = 2;
constexpr int kSoft = 256;                     // softmax threads (warps 3-10)
constexpr int kThreads = kProd + 32 + kSoft;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kQMax = 448.f;                 // e4m3 largest finite value
constexpr float kPMax = 256.f;                 // largest scaled probability (leaves headroom below 448)
constexpr float kTau = 0.75f;                  // a head's maximum is raised (and O^T rescaled) only past 2^kTau
constexpr float kTauF = 1.6817928305074290f;   // 2^kTau: probabilities stay below it

// MN-major operand of 8-bit elements whose M extent is one 128-byte swizzle atom: 8-row K groups 1024 B apart
// (the same bytes as a K-major key tile; both offset fields carry the group stride)
__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t s) {
  uint64_t d = (uint64_t)((s >> 4) & 0x3FFF);
  d |= (uint64_t)(1024 >> 4) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
// kind::f8f6f4 instruction descriptor: A and B e4m3, D f32, N, M; A MN-major when a_mn
__device__ __forceinline__ uint32_t idesc_e4m3(int n, int m, bool a_mn) {
  return (1u << 4) | (a_mn ? (1u << 15) : 0u) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void mma_e4m3(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.u32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n"
      ::"r"(d), "l"(a), "l"(b), "r"(id), "r"(acc));
}

// TMEM <-> registers: N (8, 16 or 32) consecutive fp32 columns of this thread's lane
template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float* v) {
  static_assert(N == 8 || N == 16 || N == 32, "columns");
  uint32_t r[N];
  if constexpr (N == 32) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
  } else if constexpr (N == 16) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
  } else {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
  }
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = __uint_as_float(r[i]);
}
template <int N>
__device__ __forceinline__ void tmem_st(uint32_t taddr, const float* v) {
  static_assert(N == 8 || N == 16 || N == 32, "columns");
  uint32_t r[N];
#pragma unroll
  for (int i = 0; i < N; ++i) r[i] = __float_as_uint(v[i]);
  if constexpr (N == 32) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
        "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
          "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
          "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
  } else if constexpr (N == 16) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
  } else {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
                 ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
                   "r"(r[7])
                 : "memory");
  }
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// one step of the butterfly transpose-reduction: lanes with bit `off` set keep the upper half of the array
template <int SZ, bool MAX>
__device__ __forceinline__ void tr_step(float* y, int lane, int off, int& base) {
  const bool u = (lane & off) != 0;
#pragma unroll
  for (int i = 0; i < SZ; ++i) {
    const float mine = u ? y[i + SZ] : y[i];
    const float oth = u ? y[i] : y[i + SZ];
    const float r = __shfl_xor_sync(0xffffffffu, oth, off);
    y[i] = MAX ? fmaxf(mine, r) : mine + r;
  }
  base += u ? SZ : 0;
}

// column-wise max / sum of x[N] (N = 8, 16 or 32) over the 32 lanes of the warp; out[c] = the warp's result for
// column c (written by one lane per column)
template <int N, bool MAX>
__device__ __forceinline__ void warp_col_reduce(const float (&x)[N], int lane, float* out) {
  static_assert(N == 8 || N == 16 || N == 32, "columns");
  constexpr int H1 = N / 2;
  float y[H1];
  const bool up = (lane & 16) != 0;
#pragma unroll
  for (int i = 0; i < H1; ++i) {
    const float mine = up ? x[i + H1] : x[i];
    const float oth = up ? x[i] : x[i + H1];
    const float r = __shfl_xor_sync(0xffffffffu, oth, 16);
    y[i] = MAX ? fmaxf(mine, r) : mine + r;
  }
  int base = up ? H1 : 0;
  int rest;                                      // lane bits below the ones that split columns
  if constexpr (N == 32) {
    tr_step<8, MAX>(y, lane, 8, base);
    tr_step<4, MAX>(y, lane, 4, base);
    tr_step<2, MAX>(y, lane, 2, base);
    tr_step<1, MAX>(y, lane, 1, base);
    rest = 0;
  } else if constexpr (N == 16) {
    tr_step<4, MAX>(y, lane, 8, base);
    tr_step<2, MAX>(y, lane, 4, base);
    tr_step<1, MAX>(y, lane, 2, base);
    rest = 1;
  } else {
    tr_step<2, MAX>(y, lane, 8, base);
    tr_step<1, MAX>(y, lane, 4, base);
    rest = 3;
  }
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    if (off <= rest) {
      const float r = __shfl_xor_sync(0xffffffffu, y[0], off);
      y[0] = MAX ? fmaxf(y[0], r) : y[0] + r;
    }
  }
  if ((lane & rest) == 0) out[base] = y[0];
}

// named barrier of the 8 softmax warps
__device__ __forceinline__ void softmax_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// 16-byte asynchronous copy global -> shared; src_bytes = 0 writes zeros without reading
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n cp.async.wait_group 0;" ::: "memory");
}

// (x0, x1) -> hi = e4m3(x), lo = e4m3(x - hi), two bytes each (x0 in the low byte)
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __nv_fp8x2_storage_t h = __nv_cvt_float2_to_fp8x2(make_float2(x0, x1), __NV_SATFINITE, __NV_E4M3);
  const uint32_t hf = e4m3x2_to_f16x2((uint16_t)h);
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hf));
  const __nv_fp8x2_storage_t l =
      __nv_cvt_float2_to_fp8x2(make_float2(x0 - f.x, x1 - f.y), __NV_SATFINITE, __NV_E4M3);
  hi = (uint32_t)h;
  lo = (uint32_t)l;
}

// 4 x 4 byte transpose among lanes 4g..4g+3: on entry byte k of lane i is (key i, head k); on exit byte k of lane i
// is (key k, head i)
__device__ __forceinline__ uint32_t transpose4(uint32_t w, int lane) {
  uint32_t o = __shfl_xor_sync(0xffffffffu, w, 2);
  w = (lane & 2) ? __byte_perm(w, o, 0x3276) : __byte_perm(w, o, 0x5410);
  o = __shfl_xor_sync(0xffffffffu, w, 1);
  return (lane & 1) ? __byte_perm(w, o, 0x3715) : __byte_perm(w, o, 0x6240);
}

struct Item {
  int r, sp, kbeg, kend, nt;
};
__device__ __forceinline__ Item item_of(const MlaAttnArgs& a, int it) {
  Item w;
  const int S = a.splits;
  w.r = it / S;
  w.sp = it % S;
  const int count = min(a.sel_count[w.r], a.max_sel);
  if (S == 1) {
    w.kbeg = 0;
    w.kend = count;
  } else {
    int per = (count + S - 1) / S;
    per = (per + kKeys - 1) / kKeys * kKeys;
    w.kbeg = min(count, w.sp * per);
    w.kend = min(count, w.kbeg + per);
  }
  w.nt = w.kend > w.kbeg ? (w.kend - w.kbeg + kKeys - 1) / kKeys : 0;
  return w;
}
// next item of this CTA with at least one key tile (items when none)
__device__ __forceinline__ int next_nonempty(const MlaAttnArgs& a, int it, int items, Item& w) {
  for (; it < items; it += gridDim.x) {
    w = item_of(a, it);
    if (w.nt > 0) return it;
  }
  return items;
}

// 128 latent dims (16 x 16 bytes of bf16) of query unit u of producer thread tid: head (tid / 4) + 16 u, block
// tid % 4 (zeros for padded heads)
__device__ __forceinline__ void load_q_unit(uint4 (&qv)[16], const MlaAttnArgs& a, int r, int u, int tid) {
  const int h = (tid >> 2) + 16 * u, kb = tid & 3;
  const bool on = h < a.H;
  const uint4* src = reinterpret_cast<const uint4*>(a.q_lat + ((int64_t)r * a.H + (on ? h : 0)) * kL + kb * 128);
#pragma unroll
  for (int i = 0; i < 16; ++i) qv[i] = on ? src[i] : make_uint4(0u, 0u, 0u, 0u);
}

template <int HN>
__global__ void __launch_bounds__(kThreads, 1) mla_tc_kernel(MlaAttnArgs a) {
  constexpr int QB = HN * kL;                    // bytes of one query term
  constexpr int PB = HN * kKeys;                 // bytes of one probability term
  constexpr int TCOLS = 6 * HN <= 128 ? 128 : (6 * HN <= 256 ? 256 : 512);
  constexpr int HW = HN / 2;                     // head columns per softmax warp
  constexpr int QU = HN / 16;                    // query units per producer thread
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = sm;                              // kStages key tiles
  uint8_t* sQ = sK + kStages * kTile;            // 2 query terms
  uint8_t* sP = sQ + 2 * QB;                     // 2 probability terms
  __shared__ __align__(8) uint64_t k_full[kStages], k_empty[kStages], qf[2], q_empty, qc_empty[2], s_full[2],
      s_empty[2], p_full, p_empty, o_empty;
  __shared__ uint32_t tmem_base;
  __shared__ volatile int fail;
  __shared__ int stop;
  __shared__ float ksc[kStages][kKeys];          // key scales of a tile (0 past the range)
  __shared__ __align__(16) float qc[2][HN];      // per item parity: sm_scale * log2(e) / query scale
  __shared__ float kmx[2][kProd];                // per item parity: largest key scale seen by each producer thread
  __shared__ __align__(16) float msm[HN];        // running max (log2 domain)
  __shared__ __align__(16) float csm[HN];        // correction factor of the last tile
  __shared__ float fsm[HN];                      // output factor of the item
  __shared__ float red[4][HN];
  __shared__ int cflag[2][2];                    // per tile parity and head half: some head was rescaled

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int items = a.R * a.splits;
  const float qscale = a.sm_scale * kLog2e;

  if (tid == 0) {
    fail = 0;
    stop = 0;
    cflag[0][0] = cflag[0][1] = cflag[1][0] = cflag[1][1] = 0;
    for (int s = 0; s < kStages; ++s) { tc::bar_init(&k_full[s], kProd); tc::bar_init(&k_empty[s], 1); }
    for (int b = 0; b < 2; ++b) {
      tc::bar_init(&qf[b], kProd);
      tc::bar_init(&qc_empty[b], 1);
      tc::bar_init(&s_full[b], 1);
      tc::bar_init(&s_empty[b], 8);
    }
    tc::bar_init(&q_empty, 1);
    tc::bar_init(&p_full, 8);
    tc::bar_init(&p_empty, 1);
    tc::bar_init(&o_empty, 8);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (tid < HN) { msm[tid] = -INFINITY; csm[tid] = 1.f; }
  if (warp == kMmaWarp) tc::tmem_alloc(&tmem_base, TCOLS);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = tmem_base;

  if (warp < 2) {
    // ------------------------------------------------------------------------------------------- producers
    int g = 0, qi = 0;
    for (int it = blockIdx.x; it < items && !fail; it += gridDim.x) {
      const Item w = item_of(a, it);
      if (w.nt == 0) continue;
      const int par = qi & 1;
      const int* sel = a.sel + (int64_t)w.r * a.max_sel;
      // issued before waiting for the previous item to release Q (they overlap its tail): the first query unit
      // and the largest key scale
      uint4 qv[16];
      load_q_unit(qv, a, w.r, 0, tid);
      float km = 0.f;
      for (int k0 = w.kbeg; k0 < w.kend; k0 += 16 * kProd) {
        int sl[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int k = k0 + i * kProd + tid;
          sl[i] = k < w.kend ? g53_checked(sel[k], a.n_slots, 3, -1) : -1;
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) km = fmaxf(km, sl[i] >= 0 ? a.kv_scale[sl[i]] : 0.f);
      }
      if (qi >= 1 && !tc::warp_wait(&q_empty, (qi - 1) & 1, &fail, a.err, 61)) break;
      if (qi >= 2 && !tc::warp_wait(&qc_empty[par], ((qi >> 1) & 1) ^ 1, &fail, a.err, 62)) break;
      kmx[par][tid] = km;
#pragma unroll 1
      for (int u = 0; u < QU; ++u) {
        const int h = (tid >> 2) + 16 * u, kb = tid & 3;
        if (u > 0) load_q_unit(qv, a, w.r, u, tid);
        // |x| of a finite bf16 orders like its low 15 bits: the maximum on the packed halves (no float copies)
        uint32_t m2 = 0u;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          m2 = __vmaxu2(m2, qv[i].x & 0x7fff7fffu);
          m2 = __vmaxu2(m2, qv[i].y & 0x7fff7fffu);
          m2 = __vmaxu2(m2, qv[i].z & 0x7fff7fffu);
          m2 = __vmaxu2(m2, qv[i].w & 0x7fff7fffu);
        }
        float am = __uint_as_float(max(m2 & 0xffffu, m2 >> 16) << 16);
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
        const float qs = am > 0.f ? kQMax / am : 1.f;
#pragma unroll
        for (int c = 0; c < 8; ++c) {            // 16 dims per 16-byte chunk
          const uint32_t wd[8] = {qv[2 * c].x, qv[2 * c].y, qv[2 * c].z, qv[2 * c].w,
                                  qv[2 * c + 1].x, qv[2 * c + 1].y, qv[2 * c + 1].z, qv[2 * c + 1].w};
          uint32_t hw[4], lw[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            uint32_t h0, l0, h1, l1;
            split2(__uint_as_float(wd[2 * e] << 16) * qs, __uint_as_float(wd[2 * e] & 0xffff0000u) * qs, h0, l0);
            split2(__uint_as_float(wd[2 * e + 1] << 16) * qs, __uint_as_float(wd[2 * e + 1] & 0xffff0000u) * qs,
                   h1, l1);
            hw[e] = h0 | (h1 << 16);
            lw[e] = l0 | (l1 << 16);
          }
          const uint32_t off = (uint32_t)(kb * HN * 128) + tc::sw128_chunk(h, c);
          *reinterpret_cast<uint4*>(sQ + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          *reinterpret_cast<uint4*>(sQ + QB + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
        if (kb == 0) qc[par][h] = h < a.H ? qscale / qs : 0.f;
      }
      tc::fence_async_smem();
      tc::bar_arrive(&qf[par]);
      // key tiles: rows tid and tid + 64; the selection entries of the next tile are loaded one tile ahead
      bool ok = true;
      int slot[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int k = w.kbeg + tid + e * kProd;
        slot[e] = k < w.kend ? g53_checked(sel[k], a.n_slots, 3, -1) : -1;
      }
      for (int j = 0; j < w.nt; ++j) {
        const int gg = g + j, s = gg % kStages;
        float scl[2];
        int nxt[2] = {-1, -1};
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          scl[e] = slot[e] >= 0 ? a.kv_scale[slot[e]] : 0.f;
          const int k = w.kbeg + (j + 1) * kKeys + tid + e * kProd;
          if (j + 1 < w.nt && k < w.kend) nxt[e] = g53_checked(sel[k], a.n_slots, 3, -1);
        }
        if (gg >= kStages && !tc::warp_wait(&k_empty[s], ((gg / kStages) & 1) ^ 1, &fail, a.err, 63)) {
          ok = false;
          break;
        }
        const uint32_t dst = tc::saddr(sK + s * kTile);
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int row = tid + e * kProd;
          const uint8_t* src = a.kv_cache + (int64_t)(slot[e] >= 0 ? slot[e] : 0) * kL;
          const uint32_t nb = slot[e] >= 0 ? 16u : 0u;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            cp_async16(dst + (uint32_t)((i >> 3) * kBlk) + tc::sw128_chunk(row, i & 7), src + i * 16, nb);
          ksc[s][row] = scl[e];
        }
        cp_async_wait_all();
        tc::fence_async_smem();
        tc::bar_arrive(&k_full[s]);
        slot[0] = nxt[0];
        slot[1] = nxt[1];
      }
      if (!ok) break;
      g += w.nt;
      ++qi;
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t id_qk = idesc_e4m3(HN, kKeys, false);
      const uint32_t id_pv = idesc_e4m3(HN, kKeys, true);
      const uint32_t q_addr = tc::saddr(sQ), p_addr = tc::saddr(sP), k_addr = tc::saddr(sK);
      // QK cursor
      Item wq;
      int itq = next_nonempty(a, blockIdx.x, items, wq);
      int jq = 0, gq = 0, qiq = 0;
      bool qf_ok = false;
      // pending PVs (QK issued, PV not yet), oldest first
      int pv_g[2], pv_q[2];
      bool pv_first[2];
      int pv_n = 0;
      uint32_t idle = 0;
      while ((itq < items || pv_n > 0) && !fail) {
        bool prog = false;
        if (itq < items && pv_n < 2) {
          const int gg = gq, s = gg % kStages, b = gg & 1;
          if (!qf_ok) qf_ok = tc::bar_try(&qf[qiq & 1], (qiq >> 1) & 1);
          if (qf_ok && tc::bar_try(&k_full[s], (gg / kStages) & 1) &&
              (gg < 2 || tc::bar_try(&s_empty[b], ((gg >> 1) & 1) ^ 1))) {
            tc::fence_after();
            tc::fence_async_smem();              // key rows written by cp.async (generic proxy)
            const uint32_t ka = k_addr + (uint32_t)(s * kTile);
#pragma unroll
            for (int term = 0; term < 2; ++term)
#pragma unroll
              for (int kb = 0; kb < 4; ++kb)
#pragma unroll
                for (int k = 0; k < 4; ++k)
                  mma_e4m3(tmem + (uint32_t)(b * HN), tc::desc_sw128(ka + kb * kBlk + k * 32),
                           tc::desc_sw128(q_addr + term * QB + kb * HN * 128 + k * 32), id_qk,
                           (term | kb | k) ? 1u : 0u);
            tc::commit(&s_full[b]);
            if (jq == wq.nt - 1) tc::commit(&q_empty);
            pv_g[pv_n] = gg;
            pv_q[pv_n] = qiq;
            pv_first[pv_n] = jq == 0;
            ++pv_n;
            ++gq;
            if (++jq == wq.nt) {
              jq = 0;
              ++qiq;
              qf_ok = false;
              itq = next_nonempty(a, itq + gridDim.x, items, wq);
            }
            prog = true;
          }
        }
        if (pv_n > 0) {
          const int gg = pv_g[0], q = pv_q[0];
          const bool first = pv_first[0];
          if (tc::bar_try(&p_full, gg & 1) && (!first || q == 0 || tc::bar_try(&o_empty, (q - 1) & 1))) {
            tc::fence_after();
            const int s = gg % kStages;
            const uint32_t ka = k_addr + (uint32_t)(s * kTile);
#pragma unroll
            for (int t = 0; t < 4; ++t)
#pragma unroll
              for (int term = 0; term < 2; ++term)
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                  mma_e4m3(tmem + (uint32_t)((2 + t) * HN), desc_mn_sw128(ka + t * kBlk + kk * 4096),
                           tc::desc_sw128(p_addr + term * PB + kk * 32), id_pv,
                           (first && term == 0 && kk == 0) ? 0u : 1u);
            tc::commit(&k_empty[s]);
            tc::commit(&p_empty);
            pv_g[0] = pv_g[1];
            pv_q[0] = pv_q[1];
            pv_first[0] = pv_first[1];
            --pv_n;
            prog = true;
          }
        }
        if (prog) {
          idle = 0;
        } else if (++idle > tc::kSpin) {
          fail = 1;
          atomicExch(a.err, 64);
          break;
        } else if (idle > 256) {
          __nanosleep(20);
        }
      }
    }
  } else {
    // ------------------------------------------------------------------------------------------- softmax
    const int quad = warp & 3, hf = (warp - 3) >> 2, L = quad * 32 + lane, st = tid - kProd - 32;
    const int h0 = hf * HW;                      // this warp's head columns [h0, h0 + HW)
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    int g = 0, qi = 0;
    for (int it = blockIdx.x; it < items; it += gridDim.x) {
      const Item w = item_of(a, it);
      const int S = a.splits;
      if (w.nt == 0) {
        // empty key range: neutral partial (or zero output)
        for (int i = st; i < a.H * kL; i += kSoft) {
          if (S == 1) a.o_lat[(int64_t)w.r * a.H * kL + i] = __float2bfloat16(0.f);
          else a.part_o[((int64_t)w.r * S + w.sp) * a.H * kL + i] = 0.f;
        }
        if (S > 1 && st < a.H) {
          float* ml = a.part_ml + (((int64_t)w.r * S + w.sp) * a.H + st) * 2;
          ml[0] = -INFINITY;
          ml[1] = 0.f;
        }
        continue;
      }
      const int par = qi & 1;
      bool ok = tc::warp_wait(&qf[par], (qi >> 1) & 1, &fail, a.err, 69);
      float F = 1.f;
      if (ok) {
        float km = fmaxf(kmx[par][lane], kmx[par][lane + 32]);
        km = warp_max(km);
        F = km > 0.f ? kPMax / (km * kTauF) : 1.f;
      }
      float lp[HW];                              // this thread's partial row sums (its key, its heads)
#pragma unroll
      for (int i = 0; i < HW; ++i) lp[i] = 0.f;
      for (int j = 0; j < w.nt; ++j) {
        const int gg = g + j, s = gg % kStages, b = gg & 1;
        ok = ok && tc::warp_wait(&s_full[b], (gg >> 1) & 1, &fail, a.err, 70);
        // the key scales of this tile (written before k_full; its next phase needs this tile's P first)
        ok = ok && tc::warp_wait(&k_full[s], (gg / kStages) & 1, &fail, a.err, 78);
        float v[HW];
        if (ok) {
          tc::fence_after();
          tmem_ld<HW>(lane_base + (uint32_t)(b * HN + h0), v);
          tc::fence_before();
          __syncwarp();
          if (lane == 0) tc::bar_arrive(&s_empty[b]);
          const float ks = ksc[s][L];
#pragma unroll
          for (int i = 0; i < HW; i += 4) {
            const float4 q4 = *reinterpret_cast<const float4*>(&qc[par][h0 + i]);
            v[i] *= ks * q4.x; v[i + 1] *= ks * q4.y; v[i + 2] *= ks * q4.z; v[i + 3] *= ks * q4.w;
          }
          if (j == w.nt - 1 && w.kbeg + j * kKeys + L >= w.kend) {
#pragma unroll
            for (int i = 0; i < HW; ++i) v[i] = -INFINITY;
          }
          warp_col_reduce<HW, true>(v, lane, &red[quad][h0]);
        }
        softmax_bar();
        if (st < HN) {
          const int h = st;
          const float mt = fmaxf(fmaxf(red[0][h], red[1][h]), fmaxf(red[2][h], red[3][h]));
          const float mo = msm[h];
          float mn = mo, c = 1.f;
          if (mo == -INFINITY) {
            mn = mt;
          } else if (mt > mo + kTau) {           // rescale only when the maximum rose by more than 2^kTau
            mn = mt;
            c = exp2f(mo - mn);
          }
          msm[h] = mn;
          csm[h] = c;
          if (c != 1.f) cflag[gg & 1][h / HW] = 1;
        }
        if (st == 0) stop = fail;
        softmax_bar();
        if (stop) { ok = false; break; }
        const bool corr = j > 0 && cflag[gg & 1][hf] != 0;
        if (st < 2) cflag[(gg + 1) & 1][st] = 0;
        if (corr) {
#pragma unroll
          for (int i = 0; i < HW; i += 4) {
            const float4 c4 = *reinterpret_cast<const float4*>(&csm[h0 + i]);
            lp[i] *= c4.x; lp[i + 1] *= c4.y; lp[i + 2] *= c4.z; lp[i + 3] *= c4.w;
          }
        }
        // the previous PV has finished: P may be overwritten and O^T is stable
        if (gg >= 1) ok = tc::warp_wait(&p_empty, (gg - 1) & 1, &fail, a.err, 73);
        if (ok) {
          tc::fence_after();
          if (corr) {
            constexpr int CC = HW < 16 ? HW : 16;    // columns per TMEM access
#pragma unroll 1
            for (int t = 0; t < 4; ++t) {
#pragma unroll
              for (int c0 = 0; c0 < HW; c0 += CC) {
                float o[CC];
                const uint32_t ta = lane_base + (uint32_t)((2 + t) * HN + h0 + c0);
                tmem_ld<CC>(ta, o);
#pragma unroll
                for (int i = 0; i < CC; i += 4) {
                  const float4 c4 = *reinterpret_cast<const float4*>(&csm[h0 + c0 + i]);
                  o[i] *= c4.x; o[i + 1] *= c4.y; o[i + 2] *= c4.z; o[i + 3] *= c4.w;
                }
                tmem_st<CC>(ta, o);
              }
            }
            tmem_st_wait();
          }
          // p = 2^(s - m), the partial sums, then P^T as two e4m3 terms (4 heads x 4 keys per 32-bit store)
          const float pf = ksc[s][L] * F;
#pragma unroll
          for (int i = 0; i < HW; i += 4) {
            const float4 m4 = *reinterpret_cast<const float4*>(&msm[h0 + i]);
            const float p0 = exp2f(v[i] - m4.x), p1 = exp2f(v[i + 1] - m4.y);
            const float p2 = exp2f(v[i + 2] - m4.z), p3 = exp2f(v[i + 3] - m4.w);
            lp[i] += p0; lp[i + 1] += p1; lp[i + 2] += p2; lp[i + 3] += p3;
            uint32_t h01, l01, h23, l23;
            split2(p0 * pf, p1 * pf, h01, l01);
            split2(p2 * pf, p3 * pf, h23, l23);
            const uint32_t th = transpose4(h01 | (h23 << 16), lane);
            const uint32_t tl = transpose4(l01 | (l23 << 16), lane);
            const int row = h0 + i + (lane & 3);   // this lane now holds 4 keys of head `row`
            const uint32_t off =
                (uint32_t)(row * 128) + (uint32_t)((((L >> 4) ^ (row & 7)) << 4) + (L & 12));
            *reinterpret_cast<uint32_t*>(sP + off) = th;
            *reinterpret_cast<uint32_t*>(sP + PB + off) = tl;
          }
          tc::fence_async_smem();
          tc::fence_before();
          __syncwarp();
          if (lane == 0) tc::bar_arrive(&p_full);
        }
      }
      // ---- item end: row sums over the 128 keys, then O^T once the last PV has finished
      if (ok) warp_col_reduce<HW, false>(lp, lane, &red[quad][h0]);
      softmax_bar();
      if (st < HN) {
        const int h = st;
        const float l = red[0][h] + red[1][h] + red[2][h] + red[3][h];
        if (S > 1 && h < a.H) {
          float* ml = a.part_ml + (((int64_t)w.r * S + w.sp) * a.H + h) * 2;
          ml[0] = msm[h] * kLn2;
          ml[1] = l;
        }
        fsm[h] = S == 1 ? (l > 0.f ? 1.f / (F * l) : 0.f) : 1.f / F;   // factor applied to O^T
      }
      if (st == 0) stop = fail || !ok;
      softmax_bar();
      if (stop) break;
      const int glast = g + w.nt - 1;
      ok = tc::warp_wait(&p_empty, glast & 1, &fail, a.err, 76);
      if (ok) {
        tc::fence_after();
        constexpr int CC = HW < 16 ? HW : 16;        // columns per TMEM access
        const int64_t row0 = S == 1 ? (int64_t)w.r * a.H : ((int64_t)w.r * S + w.sp) * a.H;
#pragma unroll 1
        for (int t = 0; t < 4; ++t) {
          const int dim = t * 128 + L;
#pragma unroll 1
          for (int c0 = 0; c0 < HW; c0 += CC) {
            float o[CC];
            tmem_ld<CC>(lane_base + (uint32_t)((2 + t) * HN + h0 + c0), o);
            const int hb = h0 + c0;
            if (S == 1) {
              __nv_bfloat16* dst = a.o_lat + (row0 + hb) * kL + dim;
#pragma unroll
              for (int i = 0; i < CC; ++i)
                if (hb + i < a.H) dst[(int64_t)i * kL] = __float2bfloat16(o[i] * fsm[hb + i]);
            } else {
              float* dst = a.part_o + (row0 + hb) * kL + dim;
#pragma unroll
              for (int i = 0; i < CC; ++i)
                if (hb + i < a.H) dst[(int64_t)i * kL] = o[i] * fsm[hb + i];
            }
          }
        }
        tc::fence_before();
        __syncwarp();
        if (lane == 0) tc::bar_arrive(&o_empty);
      }
      if (st == 0) stop = fail || !ok;
      softmax_bar();
      if (stop) break;
      if (st < HN) { msm[st] = -INFINITY; csm[st] = 1.f; }
      if (st == 0) tc::bar_arrive(&qc_empty[par]);
      g += w.nt;
      ++qi;
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == kMmaWarp) tc::tmem_free(tmem, TCOLS);
}

template <int HN>
cudaError_t launch(const MlaAttnArgs& a, cudaStream_t st) {
  const int smem = kStages * kTile + 2 * HN * kL + 2 * HN * kKeys + 1024;
  cudaError_t e = cudaFuncSetAttribute(mla_tc_kernel<HN>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int items = a.R * a.splits;
  const int grid = std::max(1, std::min(items, sms));
  mla_tc_kernel<HN><<<grid, kThreads, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace mtc
}  // namespace g53

cudaError_t g53_mla_attn_tc(const MlaAttnArgs& a, cudaStream_t st) {
  using namespace g53::mtc;
  if (a.L != kL || a.rope != 0 || a.H < 1 || a.H > 64 || a.R < 1 || a.splits < 1 || a.err == nullptr)
    return cudaErrorInvalidValue;
  if (a.splits > 1 && (a.part_o == nullptr || a.part_ml == nullptr)) return cudaErrorInvalidValue;
  if (a.H <= 16) return launch<16>(a, st);
  if (a.H <= 32) return launch<32>(a, st);
  return launch<64>(a, st);
}
