// MLA with an fp8 latent KV cache, absorbed form (multi-query attention over the kv_lora latent).
//
//   prep      per row: qr = bf16(rmsnorm(q_a) * w); c = bf16(rmsnorm(kv_a) * w) -> e4m3 with one fp32 scale per token
//             (amax / 448) written to the cache slot; rope key bf16(rope(k_pe)) written beside it
//   decode    flash-decoding over the DSA-selected key slots of each query row: CTA = (row, 16-head tile, key
//             split), 4 warps, each warp owning a quarter of the latent columns.  QK^T: every warp multiplies its
//             column quarter (mma.m16n8k16 f16; the fp8 keys convert exactly to f16 in registers) and the four
//             partial score tiles are summed in shared memory; the per-token key scale is applied to the sum;
//             online softmax in registers; PV: the probabilities (times the key scale) are the A operand, the same
//             fp8 latent rows are V.  Partial (o, m, l) per split, merged by a second kernel.
// Reference counterparts: code/fork/kernels/mla_prefill/mla_prefill_kernel.cuh:176 (sparse MLA prefill, one CTA
// per query token) and FlashInfer's sparse MLA decode used by the reference (code/fork/docs/MLA_PREFILL.md:23-28).
#include "common.cuh"
#include "launchers.h"

namespace g53 {

__device__ __forceinline__ void rope_pair(float x1, float x2, float ang, float& o1, float& o2) {
  float sn, cs;
  sincosf(ang, &sn, &cs);
  o1 = x1 * cs - x2 * sn;
  o2 = x2 * cs + x1 * sn;
}

__global__ void __launch_bounds__(256) mla_prep_kernel(MlaPrepArgs a) {
  pdl_trigger();                       // dependents (the next projection) may start prefetching
  const int r = blockIdx.x;
  __shared__ float red[32];
  __shared__ float vals[1024];
  const __nv_bfloat16* row = a.qkv_a + (int64_t)r * a.ld;
  // q residual
  float ss = 0.f;
  for (int i = threadIdx.x; i < a.q_lora; i += blockDim.x) { const float v = bf2f(row[i]); ss += v * v; }
  ss = block_sum(ss, red);
  float rinv = rsqrtf(ss / (float)a.q_lora + a.eps);
  for (int i = threadIdx.x; i < a.q_lora; i += blockDim.x)
    a.qr[(int64_t)r * a.q_lora + i] = f2bf(bf2f(row[i]) * rinv * bf2f(a.q_norm[i]));
  // latent
  const __nv_bfloat16* kv = row + a.q_lora;
  ss = 0.f;
  for (int i = threadIdx.x; i < a.kv_lora; i += blockDim.x) { const float v = bf2f(kv[i]); ss += v * v; }
  ss = block_sum(ss, red);
  rinv = rsqrtf(ss / (float)a.kv_lora + a.eps);
  float amax = 0.f;
  for (int i = threadIdx.x; i < a.kv_lora; i += blockDim.x) {
    const float c = round_bf16(bf2f(kv[i]) * rinv * bf2f(a.kv_norm[i]));
    vals[i] = c;
    amax = fmaxf(amax, fabsf(c));
  }
  // block max
  amax = warp_max(amax);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  float m = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) m = fmaxf(m, red[i]);
  const float scale = fmaxf(m, 1e-8f) / 448.f;
  const int slot = a.slots[r];
  if (!g53_in_bounds(slot, a.n_slots, 2)) return;        // uniform per CTA (one row)
  for (int i = threadIdx.x; i < a.kv_lora; i += blockDim.x) {
    const __nv_fp8_e4m3 q8(vals[i] / scale);
    a.kv_cache[(int64_t)slot * a.kv_lora + i] = q8.__x;
  }
  if (threadIdx.x == 0) a.kv_scale[slot] = scale;
  // rope key
  if (a.rope > 0) {
    const int half = a.rope / 2;
    const float pos = (float)a.positions[r];
    const __nv_bfloat16* pe = kv + a.kv_lora;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
      const float inv = powf(a.theta, -(float)i / (float)half);
      float o1, o2;
      rope_pair(bf2f(pe[i]), bf2f(pe[i + half]), pos * inv, o1, o2);
      a.kpe_cache[(int64_t)slot * a.rope + i] = f2bf(o1);
      a.kpe_cache[(int64_t)slot * a.rope + i + half] = f2bf(o2);
    }
  }
}

__global__ void rope_q_kernel(__nv_bfloat16* q, int H, int qk, int nope, int rope, const int* positions, float theta) {
  const int r = blockIdx.x;
  const int half = rope / 2;
  const float pos = (float)positions[r];
  for (int idx = threadIdx.x; idx < H * half; idx += blockDim.x) {
    const int h = idx / half, i = idx % half;
    __nv_bfloat16* p = q + ((int64_t)r * H + h) * qk + nope;
    const float inv = powf(theta, -(float)i / (float)half);
    float o1, o2;
    rope_pair(bf2f(p[i]), bf2f(p[i + half]), pos * inv, o1, o2);
    p[i] = f2bf(o1);
    p[i + half] = f2bf(o2);
  }
}

template <int L, int ROPE>
__global__ void __launch_bounds__(128) mla_decode_kernel(MlaAttnArgs a) {
  constexpr int KT = 32;
  constexpr int LW = L / 4;
  constexpr int NTW = LW / 8;
  constexpr int QP = L + 8;
  constexpr int KP = L + 16;
  constexpr int RP = (ROPE > 0 ? ROPE : 8) + 8;
  __shared__ __align__(16) __half qs[16][QP];
  __shared__ __align__(16) __half qpe[16][RP];
  __shared__ __align__(16) uint8_t kt[KT][KP];
  __shared__ __align__(16) __half kpe[KT][RP];
  __shared__ float ksc[KT];
  __shared__ float sred[4][16][KT + 1];
  __shared__ float srope[16][KT + 1];

  const int r = blockIdx.x, ht = blockIdx.y, sp = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, q = lane & 3;
  const int h0 = ht * 16;
  const int count = max(0, min(a.sel_count[r], a.max_sel));   // a row never reads past its max_sel selections
  const int chunk = (count + a.splits - 1) / a.splits;
  const int kbeg = sp * chunk, kend = min(count, kbeg + chunk);

  for (int i = tid; i < 16 * L; i += 128) {
    const int hh = i / L, l = i % L;
    const float v = (h0 + hh < a.H) ? bf2f(a.q_lat[((int64_t)r * a.H + h0 + hh) * L + l]) : 0.f;
    qs[hh][l] = __float2half_rn(v);
  }
  if (ROPE > 0) {
    for (int i = tid; i < 16 * ROPE; i += 128) {
      const int hh = i / ROPE, l = i % ROPE;
      const float v = (h0 + hh < a.H) ? bf2f(a.q_pe[(int64_t)r * a.q_pe_ld + (int64_t)(h0 + hh) * a.q_pe_hs + l]) : 0.f;
      qpe[hh][l] = __float2half_rn(v);
    }
  }
  float o[NTW][4];
#pragma unroll
  for (int i = 0; i < NTW; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int* sel = a.sel + (int64_t)r * a.max_sel;

  for (int kb = kbeg; kb < kend; kb += KT) {
    const int nk = min(KT, kend - kb);
    __syncthreads();
    for (int i = tid; i < KT * (L / 16); i += 128) {
      const int key = i / (L / 16), c = i % (L / 16);
      uint4 v = make_uint4(0, 0, 0, 0);
      if (key < nk)
        v = *reinterpret_cast<const uint4*>(a.kv_cache + (int64_t)g53_checked(sel[kb + key], a.n_slots, 3, 0) * L +
                                            c * 16);
      *reinterpret_cast<uint4*>(&kt[key][c * 16]) = v;
    }
    if (tid < KT) ksc[tid] = tid < nk ? a.kv_scale[g53_checked(sel[kb + tid], a.n_slots, 3, 0)] : 0.f;
    if (ROPE > 0) {
      for (int i = tid; i < KT * ROPE; i += 128) {
        const int key = i / ROPE, l = i % ROPE;
        const float v =
            key < nk ? bf2f(a.kpe_cache[(int64_t)g53_checked(sel[kb + key], a.n_slots, 3, 0) * ROPE + l]) : 0.f;
        kpe[key][l] = __float2half_rn(v);
      }
    }
    __syncthreads();
    // partial scores over this warp's latent columns
    float s[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < LW / 16; ++ks) {
      const int k0 = warp * LW + ks * 16;
      uint32_t af[4];
      af[0] = *reinterpret_cast<const uint32_t*>(&qs[g][k0 + 2 * q]);
      af[1] = *reinterpret_cast<const uint32_t*>(&qs[g + 8][k0 + 2 * q]);
      af[2] = *reinterpret_cast<const uint32_t*>(&qs[g][k0 + 2 * q + 8]);
      af[3] = *reinterpret_cast<const uint32_t*>(&qs[g + 8][k0 + 2 * q + 8]);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int key = nt * 8 + g;
        const uint32_t b0 = e4m3x2_to_f16x2(*reinterpret_cast<const uint16_t*>(&kt[key][k0 + 2 * q]));
        const uint32_t b1 = e4m3x2_to_f16x2(*reinterpret_cast<const uint16_t*>(&kt[key][k0 + 2 * q + 8]));
        mma_f16_16816(s[nt], af, b0, b1);
      }
    }
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      sred[warp][g][nt * 8 + 2 * q] = s[nt][0];
      sred[warp][g][nt * 8 + 2 * q + 1] = s[nt][1];
      sred[warp][g + 8][nt * 8 + 2 * q] = s[nt][2];
      sred[warp][g + 8][nt * 8 + 2 * q + 1] = s[nt][3];
    }
    if (ROPE > 0 && warp == 0) {
      float sr[4][4];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) sr[nt][0] = sr[nt][1] = sr[nt][2] = sr[nt][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < (ROPE > 0 ? ROPE : 16) / 16; ++ks) {
        const int k0 = ks * 16;
        uint32_t af[4];
        af[0] = *reinterpret_cast<const uint32_t*>(&qpe[g][k0 + 2 * q]);
        af[1] = *reinterpret_cast<const uint32_t*>(&qpe[g + 8][k0 + 2 * q]);
        af[2] = *reinterpret_cast<const uint32_t*>(&qpe[g][k0 + 2 * q + 8]);
        af[3] = *reinterpret_cast<const uint32_t*>(&qpe[g + 8][k0 + 2 * q + 8]);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          const int key = nt * 8 + g;
          const uint32_t b0 = *reinterpret_cast<const uint32_t*>(&kpe[key][k0 + 2 * q]);
          const uint32_t b1 = *reinterpret_cast<const uint32_t*>(&kpe[key][k0 + 2 * q + 8]);
          mma_f16_16816(sr[nt], af, b0, b1);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        srope[g][nt * 8 + 2 * q] = sr[nt][0];
        srope[g][nt * 8 + 2 * q + 1] = sr[nt][1];
        srope[g + 8][nt * 8 + 2 * q] = sr[nt][2];
        srope[g + 8][nt * 8 + 2 * q + 1] = sr[nt][3];
      }
    }
    __syncthreads();
    // full scores in the accumulator layout
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = g + (i >= 2 ? 8 : 0);
        const int key = nt * 8 + 2 * q + (i & 1);
        float v = (sred[0][row][key] + sred[1][row][key] + sred[2][row][key] + sred[3][row][key]) * ksc[key];
        if (ROPE > 0) v += srope[row][key];
        v = key < nk ? v * a.sm_scale : -INFINITY;
        s[nt][i] = v;
        if (i < 2) mx0 = fmaxf(mx0, v); else mx1 = fmaxf(mx1, v);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float al0 = (mn0 == -INFINITY) ? 1.f : __expf(m0 - mn0);
    const float al1 = (mn1 == -INFINITY) ? 1.f : __expf(m1 - mn1);
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      s[nt][0] = (s[nt][0] == -INFINITY) ? 0.f : __expf(s[nt][0] - mn0);
      s[nt][1] = (s[nt][1] == -INFINITY) ? 0.f : __expf(s[nt][1] - mn0);
      s[nt][2] = (s[nt][2] == -INFINITY) ? 0.f : __expf(s[nt][2] - mn1);
      s[nt][3] = (s[nt][3] == -INFINITY) ? 0.f : __expf(s[nt][3] - mn1);
      rs0 += s[nt][0] + s[nt][1];
      rs1 += s[nt][2] + s[nt][3];
    }
    rs0 += __shfl_xor_sync(0xffffffffu, rs0, 1);
    rs0 += __shfl_xor_sync(0xffffffffu, rs0, 2);
    rs1 += __shfl_xor_sync(0xffffffffu, rs1, 1);
    rs1 += __shfl_xor_sync(0xffffffffu, rs1, 2);
    l0 = l0 * al0 + rs0;
    l1 = l1 * al1 + rs1;
    m0 = mn0;
    m1 = mn1;
#pragma unroll
    for (int i = 0; i < NTW; ++i) { o[i][0] *= al0; o[i][1] *= al0; o[i][2] *= al1; o[i][3] *= al1; }
    // PV (probabilities times the key scale; V = the fp8 latent rows)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int ka = 16 * j + 2 * q, kb2 = 16 * j + 8 + 2 * q;
      uint32_t af[4];
      af[0] = f32x2_to_f16x2(s[2 * j][0] * ksc[ka], s[2 * j][1] * ksc[ka + 1]);
      af[1] = f32x2_to_f16x2(s[2 * j][2] * ksc[ka], s[2 * j][3] * ksc[ka + 1]);
      af[2] = f32x2_to_f16x2(s[2 * j + 1][0] * ksc[kb2], s[2 * j + 1][1] * ksc[kb2 + 1]);
      af[3] = f32x2_to_f16x2(s[2 * j + 1][2] * ksc[kb2], s[2 * j + 1][3] * ksc[kb2 + 1]);
#pragma unroll
      for (int ot = 0; ot < NTW; ++ot) {
        const int l = warp * LW + ot * 8 + g;
        const uint16_t p0 = (uint16_t)kt[ka][l] | ((uint16_t)kt[ka + 1][l] << 8);
        const uint16_t p1 = (uint16_t)kt[kb2][l] | ((uint16_t)kt[kb2 + 1][l] << 8);
        mma_f16_16816(o[ot], af, e4m3x2_to_f16x2(p0), e4m3x2_to_f16x2(p1));
      }
    }
  }
  // write the split's partial output and statistics
  const int S = a.splits;
#pragma unroll
  for (int ot = 0; ot < NTW; ++ot) {
    const int col = warp * LW + ot * 8 + 2 * q;
    if (h0 + g < a.H) {
      float* p = a.part_o + (((int64_t)r * S + sp) * a.H + h0 + g) * L + col;
      p[0] = o[ot][0]; p[1] = o[ot][1];
    }
    if (h0 + g + 8 < a.H) {
      float* p = a.part_o + (((int64_t)r * S + sp) * a.H + h0 + g + 8) * L + col;
      p[0] = o[ot][2]; p[1] = o[ot][3];
    }
  }
  if (warp == 0 && q == 0) {
    if (h0 + g < a.H) {
      float* p = a.part_ml + (((int64_t)r * S + sp) * a.H + h0 + g) * 2;
      p[0] = m0; p[1] = l0;
    }
    if (h0 + g + 8 < a.H) {
      float* p = a.part_ml + (((int64_t)r * S + sp) * a.H + h0 + g + 8) * 2;
      p[0] = m1; p[1] = l1;
    }
  }
}

__global__ void mla_merge_kernel(MlaAttnArgs a) {
  pdl_trigger();                       // dependents (the next projection) may start prefetching
  const int r = blockIdx.x, h = blockIdx.y;
  const int S = a.splits;
  float M = -INFINITY;
  for (int s = 0; s < S; ++s) M = fmaxf(M, a.part_ml[(((int64_t)r * S + s) * a.H + h) * 2]);
  float den = 0.f;
  float w[16];
  for (int s = 0; s < S; ++s) {
    const float m = a.part_ml[(((int64_t)r * S + s) * a.H + h) * 2];
    const float l = a.part_ml[(((int64_t)r * S + s) * a.H + h) * 2 + 1];
    w[s] = (m == -INFINITY) ? 0.f : __expf(m - M);
    den += w[s] * l;
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  for (int l = threadIdx.x; l < a.L; l += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < S; ++s) acc += w[s] * a.part_o[(((int64_t)r * S + s) * a.H + h) * a.L + l];
    a.o_lat[((int64_t)r * a.H + h) * a.L + l] = f2bf(acc * inv);
  }
}

}  // namespace g53

using namespace g53;

cudaError_t g53_mla_prep(const MlaPrepArgs& a, cudaStream_t st) {
  if (a.kv_lora > 1024) return cudaErrorInvalidValue;
  mla_prep_kernel<<<a.R, 256, 0, st>>>(a);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}

cudaError_t g53_rope_q(__nv_bfloat16* q, int R, int H, int qk, int nope, int rope, const int* positions, float theta,
                       cudaStream_t st) {
  if (rope == 0) return cudaSuccess;
  rope_q_kernel<<<R, 256, 0, st>>>(q, H, qk, nope, rope, positions, theta);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}

cudaError_t g53_mla_decode(const MlaAttnArgs& a, cudaStream_t st) {
  if (a.splits < 1 || a.splits > 16) return cudaErrorInvalidValue;
  if (a.use_tc) {
    cudaError_t e = g53_mla_attn_tc(a, st);
    if (e != cudaSuccess) return e;
    if (a.splits > 1) {
      mla_merge_kernel<<<dim3(a.R, a.H), 128, 0, st>>>(a);
      G53_CHECK_LAUNCH();
    }
    return cudaSuccess;
  }
  dim3 grid(a.R, (a.H + 15) / 16, a.splits);
  if (a.L == 512 && a.rope == 0) mla_decode_kernel<512, 0><<<grid, 128, 0, st>>>(a);
  else if (a.L == 128 && a.rope == 32) mla_decode_kernel<128, 32><<<grid, 128, 0, st>>>(a);
  else if (a.L == 128 && a.rope == 0) mla_decode_kernel<128, 0><<<grid, 128, 0, st>>>(a);
  else return cudaErrorInvalidValue;
  G53_CHECK_LAUNCH();
  dim3 g2(a.R, a.H);
  mla_merge_kernel<<<g2, 128, 0, st>>>(a);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}

// ---------------------------------------------------------------------------------------------------------------
// Allocation-free entry point (declared in mla_noalloc.h): the split partials of the flash-decoding kernel live in
// a file-scope device array instead of caller-provided scratch.
// ---------------------------------------------------------------------------------------------------------------
#include <mutex>
#include "mla_noalloc.h"

static __device__ __align__(256) float g53_mla_noalloc_scratch[G53_MLA_NOALLOC_MAX_PARTIAL + G53_MLA_NOALLOC_MAX_STATS];

namespace {
constexpr int kMaxDevices = 64;
float* g_noalloc_ptr[kMaxDevices] = {};
std::mutex g_noalloc_mu;

// Device address of the scratch array on the current device (looked up once per device).  A host-side use of the
// symbol name itself would give a host stand-in address, not device memory, so the address is always taken from
// cudaGetSymbolAddress with the device current.  Returns 0, the cudaError_t of a failed cudaGetDevice (or
// cudaErrorInvalidDevice past the table), or G53_NOALLOC_ERR_SYMBOL when only the symbol lookup failed.
int noalloc_scratch(float** out) {
  int dev = 0;
  const cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kMaxDevices) return (int)cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g53_mla_noalloc_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();                       // the failed lookup's error is reported as ERR_SYMBOL, not left sticky
      return G53_NOALLOC_ERR_SYMBOL;
    }
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return 0;
}

// the (L, rope) pairs the CUDA-core kernel is instantiated for
bool noalloc_supported(int L, int rope) {
  return (L == 512 && rope == 0) || (L == 128 && rope == 32) || (L == 128 && rope == 0);
}
}  // namespace

extern "C" int g53_mla_decode_noalloc(const void* q_lat, const void* q_pe, int64_t q_pe_ld, int q_pe_hs,
                                      const void* kv_cache, const float* kv_scale, const void* kpe_cache,
                                      const int* sel, const int* sel_count, int max_sel, int R, int H, int L, int rope,
                                      float sm_scale, int splits, void* o_lat, void* stream) {
  if (R < 1 || H < 1 || L < 1 || splits < 1 || splits > 16 || max_sel < 1) return (int)cudaErrorInvalidValue;
  if (!noalloc_supported(L, rope)) return (int)cudaErrorInvalidValue;
  if (!q_lat || !kv_cache || !kv_scale || !sel || !sel_count || !o_lat) return (int)cudaErrorInvalidValue;
  if (rope > 0 && (!q_pe || !kpe_cache)) return (int)cudaErrorInvalidValue;   // the rope kernel reads both
  const int64_t partial = (int64_t)R * splits * H * L;
  const int64_t stats = (int64_t)R * splits * H * 2;
  if (partial > G53_MLA_NOALLOC_MAX_PARTIAL || stats > G53_MLA_NOALLOC_MAX_STATS) return G53_NOALLOC_ERR_TOO_LARGE;
  float* scratch = nullptr;
  const int se = noalloc_scratch(&scratch);
  if (se != 0) return se;
  MlaAttnArgs a{};
  a.q_lat = static_cast<const __nv_bfloat16*>(q_lat);
  a.q_pe = static_cast<const __nv_bfloat16*>(q_pe);
  a.q_pe_ld = q_pe_ld;
  a.q_pe_hs = q_pe_hs;
  a.kv_cache = static_cast<const uint8_t*>(kv_cache);
  a.kv_scale = kv_scale;
  a.kpe_cache = static_cast<const __nv_bfloat16*>(kpe_cache);
  a.sel = sel;
  a.sel_count = sel_count;
  a.max_sel = max_sel;
  a.R = R;
  a.H = H;
  a.L = L;
  a.rope = rope;
  a.sm_scale = sm_scale;
  a.splits = splits;
  a.part_o = scratch;
  a.part_ml = scratch + G53_MLA_NOALLOC_MAX_PARTIAL;
  a.o_lat = static_cast<__nv_bfloat16*>(o_lat);
  return (int)g53_mla_decode(a, static_cast<cudaStream_t>(stream));
}

extern "C" const char* g53_mla_decode_noalloc_error(int code) {
  if (code == 0) return "ok";
  if (code == G53_NOALLOC_ERR_TOO_LARGE)
    return "problem too large for the fixed scratch: R*splits*H*L must be <= 2^20 and R*splits*H*2 <= 2^15";
  if (code == G53_NOALLOC_ERR_SYMBOL) return "could not obtain the device address of the scratch array";
  return cudaGetErrorString(static_cast<cudaError_t>(code));
}
