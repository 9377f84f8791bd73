// Fused KDA decode step: one kernel per verify window instead of five (f_b GEMV, g_b GEMV, causal conv, recurrent
// delta rule, gated output norm).
//
// CTA = (head h, sequence), 512 threads.  In order:
//   1. the head's f_b and g_b weight rows (128 x 128 e4m3 each) are copied to shared memory before
//      griddepcontrol.wait (they do not depend on the previous kernel);
//   2. decay logits f and output-gate logits of the window's rows: swap-AB mma.m16n8k16 (16 warps = 2 matrices x 8
//      tiles of 16 channels; the f_a / g_a inputs are the 128-wide columns of the input projection), x row scale,
//      rounded to bf16 as the GEMVs round them; f is also stored for the commit replay;
//   3. causal depthwise conv (4 taps, SiLU) of the head's 384 q/k/v channels, threads 0..383 one channel each,
//      outputs rounded to bf16 and stored (the commit replay re-reads them);
//   4. per row: l2-normalised q, k, the decay factor exp(g) (once per channel, not per state row) and beta
//      (one warp per row);
//   5. the delta-rule recurrence over the rows with thread (v, kq) holding S[v][kq + 4j], exactly the arithmetic
//      of kda_recurrent_kernel (kda.cu), so a commit that replays fewer rows from the stored conv outputs and
//      decay logits reproduces the state;
//   6. the gated RMS norm of every row's head output (one warp per row), written as the o_proj input.
// The recurrence reads S_in and writes S_out (double buffer), as the unfused path does.
//
// Reference counterparts: code/fork/glm53_kda_lazy.py:160-178 (recurrence and lazy commit) and the decode smallops
// of code/fork/kernels/smallops.cu (conv / gated norm); the f_b / g_b projections are the reference's
// code/fork/fp8_gemv.py decode GEMVs, here folded into the consumer.
#include <cstdlib>
#include "common.cuh"
#include "launchers.h"

namespace g53 {
namespace kd {

constexpr int DH = 128;
constexpr int kThreads = 512;
constexpr int kMaxRows = 16;
constexpr int kWP = DH + 64;     // shared pitch of a weight row: the two rows a quarter-warp reads fall in disjoint banks

struct Smem {
  alignas(16) uint8_t wf[DH][kWP];
  alignas(16) uint8_t wg[DH][kWP];
  float f[kMaxRows][DH];          // decay logits (bf16 values)
  float gate[kMaxRows][DH];       // output-gate logits (bf16 values)
  float q[kMaxRows][DH];          // conv outputs (bf16 values), then normalised
  float k[kMaxRows][DH];
  float v[kMaxRows][DH];
  float g[kMaxRows][DH];          // decay factors exp(g), computed once per channel
  float o[kMaxRows][DH];          // recurrence outputs
  float beta[kMaxRows];
};

__global__ void __launch_bounds__(kThreads, 1) kda_decode_kernel(KdaArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  pdl_trigger();
  const int h = blockIdx.x, b = blockIdx.y;
  if (!g53_in_bounds(a.s_in[b], a.n_states, 5) || !g53_in_bounds(a.s_out[b], a.n_states, 5) ||
      !g53_in_bounds(a.conv_slot[b], a.n_conv, 5))
    return;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int HD = a.H * DH, C3 = 3 * HD;

  // 1. weights of this head (16-byte copies), conv taps of this thread's channel
  for (int i = tid; i < 2 * DH * (DH / 16); i += kThreads) {
    const int m = i / (DH * DH / 16), rem = i % (DH * DH / 16);
    const int row = rem / (DH / 16), col = (rem % (DH / 16)) * 16;
    const uint8_t* src = (m ? a.gb_w : a.fb_w) + (int64_t)(h * DH + row) * DH + col;
    *reinterpret_cast<uint4*>(m ? &sm.wg[row][col] : &sm.wf[row][col]) = ldg_nc_v4(src);
  }
  const int part = tid / DH, cc = tid % DH;                  // conv: q / k / v part and channel within the head
  const int cch = part * HD + h * DH + cc;
  float w[4] = {0.f, 0.f, 0.f, 0.f};
  if (part < 3) {
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = a.conv_w[(int64_t)cch * 4 + i];
  }
  // the head's input state (64 KB, contiguous) was written by an earlier step, not by the kernel this one waits
  // for: pull it towards L2 now, so the recurrence's state loads (issued after three dependent phases) hit L2
  if (tid < 16) {
    const float* sblk = a.S_pool + a.s_in[blockIdx.y] * ((int64_t)a.H * DH * DH) + (int64_t)h * DH * DH;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(sblk + tid * (DH * DH / 16)),
                 "r"((uint32_t)(DH * DH / 16 * 4)) : "memory");
  }
  pdl_wait();                                                 // the input projection and the states are ready
  const int base = a.row0[b], n = min(a.nrows[b], kMaxRows);
  __syncthreads();

  // 2. f and gate logits: warp = (matrix, 16-channel tile), one n8 tile of rows per pass
  {
    const int m = warp >> 3, mt = warp & 7, g = lane >> 2, q = lane & 3;
    const uint8_t (*W)[kWP] = m ? sm.wg : sm.wf;
    const float* sc = (m ? a.gb_s : a.fb_s) + h * DH;
    const int xoff = a.fa_off + m * DH;
    float (*dst)[DH] = m ? sm.gate : sm.f;
    for (int n0 = 0; n0 < n; n0 += 8) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      const int t = n0 + g;
      const bool tv = t < n;
#pragma unroll
      for (int ch = 0; ch < DH / 64; ++ch) {
        const int kb = ch * 64 + q * 16;
        const uint4 wa = *reinterpret_cast<const uint4*>(&W[mt * 16 + g][kb]);
        const uint4 wb = *reinterpret_cast<const uint4*>(&W[mt * 16 + g + 8][kb]);
        uint4 x0 = make_uint4(0, 0, 0, 0), x1 = x0;
        if (tv) {
          const __nv_bfloat16* xr = a.proj + (int64_t)(base + t) * a.ldp + xoff + kb;
          x0 = *reinterpret_cast<const uint4*>(xr);
          x1 = *reinterpret_cast<const uint4*>(xr + 8);
        }
        const uint32_t wav[4] = {wa.x, wa.y, wa.z, wa.w}, wbv[4] = {wb.x, wb.y, wb.z, wb.w};
        const uint32_t xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          uint32_t af[4];
          af[0] = e4m3x2_to_f16x2((uint16_t)(wav[k4] & 0xffffu));
          af[1] = e4m3x2_to_f16x2((uint16_t)(wbv[k4] & 0xffffu));
          af[2] = e4m3x2_to_f16x2((uint16_t)(wav[k4] >> 16));
          af[3] = e4m3x2_to_f16x2((uint16_t)(wbv[k4] >> 16));
          mma_f16_16816(acc, af, bf16x2_to_f16x2(xv[2 * k4]), bf16x2_to_f16x2(xv[2 * k4 + 1]));
        }
      }
      // acc: channel rows (g, g+8) of the tile x rows (2q, 2q+1) of the token tile
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = mt * 16 + g + (j >> 1) * 8, tt = n0 + 2 * q + (j & 1);
        if (tt < n) {
          const float vv = round_bf16(acc[j] * sc[c]);
          dst[tt][c] = vv;
          if (m == 0) a.f_store[(int64_t)(base + tt) * HD + h * DH + c] = f2bf(vv);
        }
      }
    }
  }

  // 3. causal conv of the head's q / k / v channels (window rows oldest first, then the window's rows)
  if (part < 3) {
    const __nv_bfloat16* win = a.conv_pool + (int64_t)a.conv_slot[b] * 3 * C3 + cch;
    // every input of the channel first (window, then the rows: all loads in flight together), then the taps
    float xs[3 + kMaxRows];
#pragma unroll
    for (int i = 0; i < 3; ++i) xs[i] = bf2f(win[(int64_t)i * C3]);
#pragma unroll
    for (int t = 0; t < kMaxRows; ++t) xs[3 + t] = t < n ? bf2f(a.proj[(int64_t)(base + t) * a.ldp + cch]) : 0.f;
    float (*dst)[DH] = part == 0 ? sm.q : (part == 1 ? sm.k : sm.v);
#pragma unroll
    for (int t = 0; t < kMaxRows; ++t) {
      if (t >= n) break;
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) s += w[i] * xs[t + i];
      const __nv_bfloat16 o = f2bf(siluf_(s));
      a.qkv[(int64_t)(base + t) * C3 + cch] = o;
      dst[t][cc] = __bfloat162float(o);
    }
  }
  __syncthreads();

  // 4. normalised q, k, decay factors and beta of every row (one warp per row)
  const float ea = __expf(a.a_log[h]);
  for (int rr = warp; rr < n; rr += kThreads / 32) {
    constexpr int PL = DH / 32;
    float qv[PL], kv[PL];
    float qq = 0.f, kk = 0.f;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      const int c = lane + 32 * i;
      qv[i] = sm.q[rr][c];
      kv[i] = sm.k[rr][c];
      qq += qv[i] * qv[i];
      kk += kv[i] * kv[i];
      sm.g[rr][c] = __expf(a.lower * sigmoidf_(ea * (sm.f[rr][c] + a.dt_bias[h * DH + c])));
    }
    qq = warp_sum(qq);
    kk = warp_sum(kk);
    const float qn = rsqrtf(qq + 1e-6f) * rsqrtf((float)DH), kn = rsqrtf(kk + 1e-6f);
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      sm.q[rr][lane + 32 * i] = qv[i] * qn;
      sm.k[rr][lane + 32 * i] = kv[i] * kn;
    }
    if (lane == 0) sm.beta[rr] = sigmoidf_(bf2f(a.proj[(int64_t)(base + rr) * a.ldp + a.b_off + h]));
  }
  __syncthreads();

  // 5. recurrence: thread (vr, kq) owns S[vr][kq + 4j]
  {
    constexpr int KP = DH / 4;
    const int vr = tid >> 2, kq = tid & 3;
    const int64_t sstride = (int64_t)a.H * DH * DH;
    float S[KP];
    const float* sin = a.S_pool + a.s_in[b] * sstride + ((int64_t)h * DH + vr) * DH + kq;
#pragma unroll
    for (int j = 0; j < KP; ++j) S[j] = sin[4 * j];
    for (int rr = 0; rr < n; ++rr) {
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < KP; ++j) {
        S[j] *= sm.g[rr][kq + 4 * j];
        dot += S[j] * sm.k[rr][kq + 4 * j];
      }
      dot = group_sum<4>(dot);
      const float vn = sm.beta[rr] * (sm.v[rr][vr] - dot);
      float o = 0.f;
#pragma unroll
      for (int j = 0; j < KP; ++j) {
        S[j] += vn * sm.k[rr][kq + 4 * j];
        o += S[j] * sm.q[rr][kq + 4 * j];
      }
      o = group_sum<4>(o);
      if (kq == 0) sm.o[rr][vr] = o;
    }
    float* sout = a.S_pool + a.s_out[b] * sstride + ((int64_t)h * DH + vr) * DH + kq;
#pragma unroll
    for (int j = 0; j < KP; ++j) sout[4 * j] = S[j];
  }
  __syncthreads();

  // 6. gated RMS norm of the head output (one warp per row)
  for (int rr = warp; rr < n; rr += kThreads / 32) {
    float ss = 0.f;
    for (int i = lane; i < DH; i += 32) ss += sm.o[rr][i] * sm.o[rr][i];
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / (float)DH + a.eps);
    __nv_bfloat16* out = a.out + (int64_t)(base + rr) * HD + h * DH;
    for (int i = lane; i < DH; i += 32)
      out[i] = f2bf(sm.o[rr][i] * r * bf2f(a.o_norm[i]) * sigmoidf_(sm.gate[rr][i]));
  }
}

}  // namespace kd
}  // namespace g53

// decode windows of at most 16 rows per sequence, head dim 128, 4 conv taps, 16-byte aligned projection rows
bool g53_kda_decode_ok(const KdaArgs& a) {
  return a.Dh == g53::kd::DH && a.taps == 4 && a.max_rows >= 1 && a.max_rows <= g53::kd::kMaxRows &&
         a.ldp % 8 == 0 && a.fa_off % 8 == 0 && (reinterpret_cast<uintptr_t>(a.proj) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(a.fb_w) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.gb_w) & 15) == 0;
}

cudaError_t g53_kda_decode(const KdaArgs& a, cudaStream_t st) {
  if (!g53_kda_decode_ok(a)) return cudaErrorInvalidValue;
  static bool attr = false;
  const int smem = (int)sizeof(g53::kd::Smem);
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(g53::kd::kda_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         smem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  static int pdl = -1;
  if (pdl < 0) {
    const char* e = std::getenv("GLM53_PDL");
    pdl = (e && e[0] == '0') ? 0 : 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.H, a.B);
  cfg.blockDim = dim3(g53::kd::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl;
  return cudaLaunchKernelEx(&cfg, g53::kd::kda_decode_kernel, a);
}
