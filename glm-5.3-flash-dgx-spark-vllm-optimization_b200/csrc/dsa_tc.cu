// DSA indexer logits on the 5th-generation tensor cores.
//
//   logits[r, j] = sum_h w[r, h] * relu(s_j * (Hq[r, h] . k_j)) / sqrt(IH * ID)      for pools j < pos_r / kpool
//
// One CTA owns QR = 256 / IH query rows (all IH heads: N = 256 columns of (row, head)) and sweeps the pool keys
// of its rows' sequence in tiles of 128 pools (M = 128), K = ID = 128:
//   warps 0-3  operand producers: the query tile once per sequence group (bf16 Hadamard-rotated queries, written
//              straight into the 128-byte-swizzled K-major layout), then for every pool tile one pool per thread:
//              16-byte loads of the e4m3 key through the page table, exact widening to bf16, swizzled stores
//   warp 4     TMEM (2 x 256 columns, double-buffered accumulator) and the MMA issuer: 8 x tcgen05.mma
//              (128 x 256 x 16, kind::f16 bf16) per tile
//   warps 5-8  epilogue: TMEM lane = pool; per query row the IH head columns of that lane are reduced in
//              registers (relu * scale * head weight), one coalesced logit store per (row, pool)
// Pools sit on the MMA's M side so the head reduction stays inside one thread.  Rows of a CTA that belong to
// different sequences are processed as consecutive groups (the query tile is rebuilt per group).  blockIdx.y splits
// a group's pool tiles across CTAs (decode windows: few rows, many pools).  Every wait is bounded; a wait that runs
// out sets the error word and the CTA stops.  No TMA is used (keys are gathered through the page table).
#include <algorithm>
#include "common.cuh"
#include "launchers.h"
#include "tc05.cuh"

namespace g53 {

constexpr int kTP = 128;                 // pools per tile (M)
constexpr int kTN = 256;                 // (row, head) columns (N)
constexpr int kStages = 3;
constexpr int kA = kTP * 256;            // bytes of a key tile: 128 rows x 128 bf16 (two 64-element k blocks)
constexpr int kB = kTN * 256;            // bytes of the query tile
constexpr int kThreadsTC = 9 * 32;
constexpr int kMaxQR = 64;

__device__ __forceinline__ int slot_of_tc(const int* bt, int bs, int p) { return bt[p / bs] * bs + p % bs; }

// byte offset of element k (0..127) of `row` in a [rows][128] bf16 tile stored as two [rows][64] swizzled blocks
__device__ __forceinline__ uint32_t kmajor_off(int rows, int row, int k) {
  return (uint32_t)((k >> 6) * rows * 128) + tc::sw128_chunk(row, (k & 63) >> 3) + (uint32_t)((k & 7) * 2);
}

template <int IH>
__global__ void __launch_bounds__(kThreadsTC, 1) dsa_logits_tc_kernel(DsaArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sB = sm;                                  // query tile
  uint8_t* sA = sm + kB;                             // kStages key tiles
  __shared__ __align__(8) uint64_t a_full[kStages], a_empty[kStages], b_full, b_empty, t_full[2], t_empty[2];
  __shared__ uint32_t tmem_base;
  __shared__ volatile int fail;
  __shared__ int r_pos[kMaxQR], r_c[kMaxQR], r_seq[kMaxQR], r_grp[kMaxQR];
  __shared__ int g_seq[kMaxQR], g_jhi[kMaxQR], n_groups;
  __shared__ float r_w[kTN];                         // head weights, column order (row, head)

  constexpr int QR = kTN / IH;
  if (a.tc_min_pools > 0 && !dsa_long_rows(a)) return;    // short rows: the CUDA-core kernel of this pair runs
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int r0 = blockIdx.x * QR;
  const int split = blockIdx.y, nsplit = gridDim.y;

  if (tid < QR) {
    const int r = r0 + tid;
    const bool ok = r < a.R;
    r_pos[tid] = ok ? a.positions[r] : 0;
    r_c[tid] = ok ? a.positions[r] / a.kpool : 0;
    r_seq[tid] = ok ? a.row_seq[r] : -1;
  }
  for (int i = tid; i < kTN; i += blockDim.x) {
    const int r = r0 + i / IH;
    r_w[i] = r < a.R ? a.iproj[(int64_t)r * a.ldi + a.ID + (i % IH)] : 0.f;
  }
  if (tid == 0) {
    fail = 0;
    int ng = 0;
    for (int i = 0; i < QR; ++i) {
      if (r_seq[i] < 0) { r_grp[i] = -1; continue; }
      if (ng == 0 || g_seq[ng - 1] != r_seq[i]) { g_seq[ng] = r_seq[i]; g_jhi[ng] = 0; ++ng; }
      r_grp[i] = ng - 1;
      g_jhi[ng - 1] = max(g_jhi[ng - 1], r_c[i]);
    }
    n_groups = ng;
    for (int s = 0; s < kStages; ++s) { tc::bar_init(&a_full[s], 128); tc::bar_init(&a_empty[s], 1); }
    tc::bar_init(&b_full, 128);
    tc::bar_init(&b_empty, 1);
    for (int b = 0; b < 2; ++b) { tc::bar_init(&t_full[b], 1); tc::bar_init(&t_empty[b], 4); }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 4) tc::tmem_alloc(&tmem_base, 2 * kTN);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = tmem_base;
  const int ng = n_groups;
  const float inv = rsqrtf((float)(IH * a.ID));
  static_assert(kTN % IH == 0 && IH <= 32 && 32 % IH == 0 && kTN / IH <= kMaxQR, "head count");

  if (warp < 4) {
    // ---------------------------------------------------------------- producers
    int kt = 0, pg = 0;                              // key tiles produced (ring position), groups processed
    for (int gi = 0; gi < ng; ++gi) {
      const int ntiles = (g_jhi[gi] + kTP - 1) / kTP;
      if (split >= ntiles) continue;                 // no tile of this group for this CTA (all roles skip it)
      if (pg > 0 && !tc::bar_wait(&b_empty, (pg - 1) & 1, &fail, a.err, 41)) break;
      ++pg;
      // query tile: 2 (row, head) pairs per warp iteration, Hadamard by fwht128_warp, rows of other groups zero
      for (int n = warp; n < kTN; n += 4) {
        const int i = n / IH, h = n % IH;
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        if (r_grp[i] == gi) {
          const __nv_bfloat16* qp = a.qi + (int64_t)(r0 + i) * IH * 128 + h * 128 + lane * 4;
#pragma unroll
          for (int e = 0; e < 4; ++e) v[e] = bf2f(qp[e]);
          fwht128_warp(v);
        }
        __nv_bfloat162 p0 = __floats2bfloat162_rn(v[0], v[1]), p1 = __floats2bfloat162_rn(v[2], v[3]);
        uint2 w;
        w.x = *reinterpret_cast<uint32_t*>(&p0);
        w.y = *reinterpret_cast<uint32_t*>(&p1);
        *reinterpret_cast<uint2*>(sB + kmajor_off(kTN, n, lane * 4)) = w;
      }
      tc::fence_async_smem();
      tc::bar_arrive(&b_full);
      const int* bt = a.block_table + (int64_t)g_seq[gi] * a.bt_ld;
      const int jhi = g_jhi[gi];
      for (int t = split; t < ntiles; t += nsplit, ++kt) {
        const int s = kt % kStages;
        if (kt >= kStages && !tc::bar_wait(&a_empty[s], ((kt / kStages) & 1) ^ 1, &fail, a.err, 42)) break;
        uint8_t* at = sA + s * kA;
        const int p = tid;                           // pool row of the tile
        const int j = t * kTP + p;
        uint4 kw[8];
        if (j < jhi) {
          const int pslot = g53_checked(slot_of_tc(bt, a.block_size, j * a.kpool) / a.kpool, a.n_pools, 4, 0);
          const uint4* src = reinterpret_cast<const uint4*>(a.pool_cache + (int64_t)pslot * 128);
#pragma unroll
          for (int c = 0; c < 8; ++c) kw[c] = src[c];
        } else {
#pragma unroll
          for (int c = 0; c < 8; ++c) kw[c] = make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) {                // 16 e4m3 -> 16 bf16 = two 16-byte chunks
          const uint32_t ws[4] = {kw[c].x, kw[c].y, kw[c].z, kw[c].w};
          uint32_t o[8];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const uint32_t h01 = e4m3x2_to_f16x2((uint16_t)(ws[e] & 0xffffu));
            const uint32_t h23 = e4m3x2_to_f16x2((uint16_t)(ws[e] >> 16));
            const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&h01));
            const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&h23));
            __nv_bfloat162 b01 = __floats2bfloat162_rn(f01.x, f01.y), b23 = __floats2bfloat162_rn(f23.x, f23.y);
            o[2 * e] = *reinterpret_cast<uint32_t*>(&b01);
            o[2 * e + 1] = *reinterpret_cast<uint32_t*>(&b23);
          }
          const int k0 = c * 16;
          *reinterpret_cast<uint4*>(at + kmajor_off(kTP, p, k0)) = make_uint4(o[0], o[1], o[2], o[3]);
          *reinterpret_cast<uint4*>(at + kmajor_off(kTP, p, k0 + 8)) = make_uint4(o[4], o[5], o[6], o[7]);
        }
        tc::fence_async_smem();
        tc::bar_arrive(&a_full[s]);
      }
      if (fail) break;
    }
  } else if (warp == 4) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t id = tc::idesc(1, kTN, kTP);
      int kt = 0, pg = 0;
      for (int gi = 0; gi < ng && !fail; ++gi) {
        const int ntiles = (g_jhi[gi] + kTP - 1) / kTP;
        if (split >= ntiles) continue;
        if (!tc::bar_wait(&b_full, pg & 1, &fail, a.err, 43)) break;
        ++pg;
        tc::fence_after();
        const uint32_t b_addr = tc::saddr(sB);
        bool ok = true;
        for (int t = split; t < ntiles; t += nsplit, ++kt) {
          const int s = kt % kStages, buf = kt & 1;
          if (kt >= 2 && !tc::bar_wait(&t_empty[buf], ((kt >> 1) & 1) ^ 1, &fail, a.err, 44)) { ok = false; break; }
          if (!tc::bar_wait(&a_full[s], (kt / kStages) & 1, &fail, a.err, 45)) { ok = false; break; }
          tc::fence_after();
          const uint32_t a_addr = tc::saddr(sA + s * kA);
#pragma unroll
          for (int kb = 0; kb < 2; ++kb)
#pragma unroll
            for (int k = 0; k < 4; ++k)
              tc::mma_f16(tmem + (uint32_t)(buf * kTN), tc::desc_sw128(a_addr + kb * kTP * 128 + k * 32),
                          tc::desc_sw128(b_addr + kb * kTN * 128 + k * 32), id, (kb | k) ? 1u : 0u);
          tc::commit(&a_empty[s]);
          tc::commit(&t_full[buf]);
        }
        if (!ok) break;
        tc::commit(&b_empty);                        // the query tile may be rewritten once these MMAs finish
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 5..8 -> quadrants 1,2,3,0)
    const int quad = warp & 3;
    const int p = quad * 32 + lane;
    int kt = 0;
    for (int gi = 0; gi < ng; ++gi) {
      const int ntiles = (g_jhi[gi] + kTP - 1) / kTP;
      if (split >= ntiles) continue;
      const int* bt = a.block_table + (int64_t)g_seq[gi] * a.bt_ld;
      bool ok = true;
      for (int t = split; t < ntiles; t += nsplit, ++kt) {
        const int buf = kt & 1;
        if (!tc::warp_wait(&t_full[buf], (kt >> 1) & 1, &fail, a.err, 46)) { ok = false; break; }
        tc::fence_after();
        const int j = t * kTP + p;
        const bool jv = j < g_jhi[gi];
        const float s =
            jv ? a.pool_scale[g53_checked(slot_of_tc(bt, a.block_size, j * a.kpool) / a.kpool, a.n_pools, 4, 0)] : 0.f;
        for (int c0 = 0; c0 < kTN; c0 += 32) {
          float v[32];
          tc::tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * kTN + c0), v);
          // columns c0 .. c0+31 = rows (c0 + e) / IH, heads (c0 + e) % IH
#pragma unroll
          for (int ii = 0; ii < 32 / IH; ++ii) {
            const int i0 = c0 / IH + ii;
            float acc = 0.f;
#pragma unroll
            for (int h = 0; h < IH; ++h) acc += fmaxf(v[ii * IH + h] * s, 0.f) * r_w[i0 * IH + h];
            if (jv && r_grp[i0] == gi && j < r_c[i0]) a.logits[(int64_t)(r0 + i0) * a.max_pools + j] = acc * inv;
          }
        }
        tc::fence_before();
        __syncwarp();
        if (lane == 0) tc::bar_arrive(&t_empty[buf]);
      }
      if (!ok) break;
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 4) tc::tmem_free(tmem, 2 * kTN);
}

}  // namespace g53

namespace {
template <int IH>
cudaError_t launch_tc(const DsaArgs& a, cudaStream_t st) {
  using namespace g53;
  constexpr int QR = kTN / IH;
  const int bx = (a.R + QR - 1) / QR;
  const int tiles = (a.max_pools + kTP - 1) / kTP;
  // few row blocks (decode windows): split each block's pool tiles over more CTAs
  const int by = std::max(1, std::min(tiles, (2 * 148 + bx - 1) / bx));
  const int smem = kB + kStages * kA + 1024;
  cudaError_t e = cudaFuncSetAttribute(dsa_logits_tc_kernel<IH>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  dsa_logits_tc_kernel<IH><<<dim3(bx, by), kThreadsTC, smem, st>>>(a);
  return cudaGetLastError();
}
}  // namespace

// tensor-core indexer logits; IH in {4, 8, 16, 32}, ID = 128 (otherwise cudaErrorInvalidValue: use the CUDA-core
// kernel)
cudaError_t g53_dsa_logits_tc(const DsaArgs& a, cudaStream_t st) {
  if (a.ID != 128) return cudaErrorInvalidValue;
  switch (a.IH) {
    case 32: return launch_tc<32>(a, st);
    case 16: return launch_tc<16>(a, st);
    case 8: return launch_tc<8>(a, st);
    case 4: return launch_tc<4>(a, st);
    default: return cudaErrorInvalidValue;
  }
}
