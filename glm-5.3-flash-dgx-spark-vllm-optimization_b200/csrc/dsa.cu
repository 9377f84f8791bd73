// DSA lightning indexer over pooled index keys.
//
//   update   per row: index key = LayerNorm(wk x) (bf16) and pool gate scores into row buffers; rows that
//            complete a pool of `kpool` tokens then compress it: per channel softmax over the pool's tokens of
//            (gate + ape), weighted key sum -> bf16 -> Hadamard-128 -> bf16 -> e4m3 with a power-of-two scale
//            (the pool lives at pool slot = token slot of its first token / kpool)
//            (reference: code/fork/tests/kpoolring/ref/kpool_compress_vllm58454.py:139-257).  A pool's tokens
//            come from this launch's row buffers or, for tokens of earlier launches, from the sequence's tail ring
//            (kDsaRing positions, indexed by the sequence's state slot and position mod kDsaRing); after the pools
//            the last kDsaRing rows of every sequence are copied into its ring.  Only open pools ever need raw
//            keys, so the cache keeps no per-token index keys (the reference's kpool tail ring,
//            code/fork/tests/kpoolring/ref/kpool_compress_vllm58454.py:734-887)
//   logits   per (row, pool): sum_h relu((Hq_h . k_pool) * scale) * w_h / sqrt(IH * ID), the queries rotated by
//            the same Hadamard transform (so q.k is preserved) and held in shared memory
//   select   per row: a query sees its own (partial) pool and the top (topk_pools - 1) earlier complete pools,
//            chosen by a 4-pass 8-bit radix select on the logits (ties: lower pool index), expanded to token
//            slots in ascending position order; while the row has at most topk_pools - 1 complete pools it sees
//            every earlier key (dense).
#include <algorithm>
#include "common.cuh"
#include "launchers.h"

namespace g53 {

__device__ __forceinline__ int slot_of(const int* bt, int bs, int p) { return bt[p / bs] * bs + p % bs; }

__global__ void __launch_bounds__(128) dsa_keys_kernel(DsaArgs a) {
  const int r = blockIdx.x;
  const float* x = a.iproj + (int64_t)r * a.ldi;
  __shared__ float red[32];
  const int c = threadIdx.x;   // ID == 128 channels, one per thread
  const float v = x[c];
  const float mean = block_sum(v, red) / (float)a.ID;
  const float d = v - mean;
  const float var = block_sum(d * d, red) / (float)a.ID;
  const float y = d * rsqrtf(var + a.eps) * a.ln_w[c] + a.ln_b[c];
  a.ik_cache[(int64_t)r * a.ID + c] = f2bf(y);
  a.ig_cache[(int64_t)r * a.ID + c] = x[a.ID + a.IH + c];
}

// (index key, gate) row of token position p of row r's sequence: this launch's row buffer when p is one of its
// rows, else the sequence's tail ring
__device__ __forceinline__ int64_t dsa_src_row(const DsaArgs& a, int r, int pos, int p, bool& ring) {
  const int rr = r - (pos - p);
  if (rr >= 0 && a.row_seq[rr] == a.row_seq[r] && a.positions[rr] == p) {
    ring = false;
    return rr;
  }
  ring = true;
  const int owner = g53_checked(a.seq_desc[4 * a.seq_ld + a.row_seq[r]], a.n_owners, 8, 0);
  return (int64_t)owner * kDsaRing + (p % kDsaRing);
}

// after the pools: the last kDsaRing rows of every sequence into its ring (positions mod kDsaRing are distinct)
__global__ void __launch_bounds__(128) dsa_ring_kernel(DsaArgs a) {
  const int r = blockIdx.x;
  const int b = a.row_seq[r];
  const int last = a.seq_desc[b] + a.seq_desc[a.seq_ld + b] - 1;
  if (r <= last - kDsaRing) return;
  const int owner = a.seq_desc[4 * a.seq_ld + b];
  if (!g53_in_bounds(owner, a.n_owners, 8)) return;    // uniform per CTA (one row)
  const int64_t dst = ((int64_t)owner * kDsaRing + a.positions[r] % kDsaRing) * a.ID;
  const int c = threadIdx.x;
  a.ik_ring[dst + c] = a.ik_cache[(int64_t)r * a.ID + c];
  a.ig_ring[dst + c] = a.ig_cache[(int64_t)r * a.ID + c];
}

// one warp per row; rows whose position completes a pool compress it
__global__ void dsa_pool_kernel(DsaArgs a) {
  const int lane = threadIdx.x & 31;
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= a.R) return;
  const int pos = a.positions[r];
  const int kp = a.kpool;
  if ((pos + 1) % kp != 0) return;
  const int p0 = pos + 1 - kp;
  const int* bt = a.block_table + (int64_t)a.row_seq[r] * a.bt_ld;
  float acc[4] = {0.f, 0.f, 0.f, 0.f}, mx[4], den[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < 4; ++i) mx[i] = -INFINITY;
  for (int s = 0; s < kp; ++s) {
    bool ring;
    const int64_t src = dsa_src_row(a, r, pos, p0 + s, ring) * a.ID;
    const float* ig = ring ? a.ig_ring : a.ig_cache;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = lane * 4 + i;
      mx[i] = fmaxf(mx[i], ig[src + c] + a.ape[s * a.ID + c]);
    }
  }
  for (int s = 0; s < kp; ++s) {
    bool ring;
    const int64_t src = dsa_src_row(a, r, pos, p0 + s, ring) * a.ID;
    const float* ig = ring ? a.ig_ring : a.ig_cache;
    const __nv_bfloat16* ik = ring ? a.ik_ring : a.ik_cache;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = lane * 4 + i;
      const float e = __expf(ig[src + c] + a.ape[s * a.ID + c] - mx[i]);
      den[i] += e;
      acc[i] += e * bf2f(ik[src + c]);
    }
  }
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = round_bf16(acc[i] / den[i]);
  fwht128_warp(v);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) { v[i] = round_bf16(v[i]); amax = fmaxf(amax, fabsf(v[i])); }
  amax = fmaxf(warp_max(amax), 1e-4f);
  const float scale = exp2f(ceilf(log2f(amax / 448.f)));
  const int pslot = slot_of(bt, a.block_size, p0) / kp;
  if (!g53_in_bounds(pslot, a.n_pools, 4)) return;       // warp-uniform; nothing follows
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_fp8_e4m3 q8(v[i] / scale);
    a.pool_cache[(int64_t)pslot * a.ID + lane * 4 + i] = q8.__x;
  }
  if (lane == 0) a.pool_scale[pslot] = scale;
}

constexpr int kMaxIH = 64;

__global__ void __launch_bounds__(256) dsa_logits_kernel(DsaArgs a) {
  if (a.tc_min_pools > 0 && dsa_long_rows(a)) return;     // the tcgen05 kernel of this launch pair takes it
  const int r = blockIdx.x;
  const int pos = a.positions[r];
  const int c = pos / a.kpool;
  const int j = blockIdx.y * blockDim.x + threadIdx.x;
  if ((int)(blockIdx.y * blockDim.x) >= c) return;
  __shared__ float qs[kMaxIH][128];
  __shared__ float hw[kMaxIH];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int h = wid; h < a.IH; h += blockDim.x >> 5) {
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = bf2f(a.qi[(int64_t)r * a.IH * 128 + h * 128 + lane * 4 + i]);
    fwht128_warp(v);
#pragma unroll
    for (int i = 0; i < 4; ++i) qs[h][lane * 4 + i] = round_bf16(v[i]);
  }
  if (threadIdx.x < a.IH) hw[threadIdx.x] = a.iproj[(int64_t)r * a.ldi + a.ID + threadIdx.x];
  __syncthreads();
  if (j >= c) return;
  const int* bt = a.block_table + (int64_t)a.row_seq[r] * a.bt_ld;
  const int pslot = g53_checked(slot_of(bt, a.block_size, j * a.kpool) / a.kpool, a.n_pools, 4, 0);
  const uint8_t* pk = a.pool_cache + (int64_t)pslot * 128;
  float kv[128];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint4 w = *reinterpret_cast<const uint4*>(pk + i * 16);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t h01 = e4m3x2_to_f16x2((uint16_t)(ws[k] & 0xffffu));
      const uint32_t h23 = e4m3x2_to_f16x2((uint16_t)(ws[k] >> 16));
      const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&h01));
      const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&h23));
      kv[i * 16 + k * 4 + 0] = f01.x; kv[i * 16 + k * 4 + 1] = f01.y;
      kv[i * 16 + k * 4 + 2] = f23.x; kv[i * 16 + k * 4 + 3] = f23.y;
    }
  }
  const float s = a.pool_scale[pslot];
  float logit = 0.f;
  for (int h = 0; h < a.IH; ++h) {
    float d = 0.f;
#pragma unroll
    for (int i = 0; i < 128; ++i) d += qs[h][i] * kv[i];
    logit += fmaxf(d * s, 0.f) * hw[h];
  }
  a.logits[(int64_t)r * a.max_pools + j] = logit * rsqrtf((float)(a.IH * a.ID));
}

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Rows with more than kSelSplit complete pools are selected by a cluster of kSelNC CTAs (one pool slice each: the
// radix histograms are summed over the cluster through distributed shared memory, the slices' counts give each
// CTA its output offset); shorter rows by rank 0 alone.  Both paths select the same pools in the same order.
constexpr int kSelNC = 8;
constexpr int kSelSplit = 16384;         // measured crossover (8 rows: single CTA 24 us vs cluster 32 us at 8192 pools)

__device__ __forceinline__ void cl_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ const int* cl_map(const int* p, int rank) {
  uint64_t r;
  asm volatile("mapa.u64 %0, %1, %2;" : "=l"(r) : "l"(p), "r"(rank));
  return reinterpret_cast<const int*>(r);
}

// the bin decision of one radix pass from the (summed) 256-bin histogram: lane l holds bins 255 - 8l .. 248 - 8l,
// an exclusive prefix over the lanes gives each lane the count of the bins above its own, and the one lane whose
// range crosses rem (or lane 31) walks its 8 bins; writes the new prefix and remainder
__device__ __forceinline__ void sel_decide(const int (&cnt)[8], uint32_t prefix, int shift, int rem,
                                           uint32_t* s_prefix, int* s_rem) {
  const int lane = threadIdx.x & 31;
  int sum = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) sum += cnt[i];
  int incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  int acc = incl - sum;
  if (acc < rem && (acc + sum >= rem || lane == 31)) {
    int b = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int bin = 255 - 8 * lane - i;
      if (bin == 0) break;                  // bin 0 is taken without a check
      if (acc + cnt[i] >= rem) { b = bin; break; }
      acc += cnt[i];
    }
    *s_prefix = prefix | ((uint32_t)b << shift);
    *s_rem = rem - acc;
  }
}

__global__ void __launch_bounds__(1024) dsa_select_kernel(DsaArgs a) {
  pdl_wait();                               // the logits of the previous kernel
  const int r = blockIdx.x, rank = blockIdx.z, nc = gridDim.z;
  const int tid = threadIdx.x, bd = blockDim.x;
  const int pos = a.positions[r];
  const int kp = a.kpool, P = a.topk_pools;
  const int c = pos / kp;
  const int* bt = a.block_table + (int64_t)a.row_seq[r] * a.bt_ld;
  int* out = a.sel + (int64_t)r * a.max_sel;
  if (nc > 1 && c > kSelSplit && c > P - 1) {
    // ---- cluster path: rank k owns pools [j0, j1)
    __shared__ int hist2[2][256];
    __shared__ uint32_t c_prefix;
    __shared__ int c_rem, c_cnt[2], c_wsum[32];
    const int j0 = (int)((int64_t)c * rank / nc), j1 = (int)((int64_t)c * (rank + 1) / nc);
    const float* lg = a.logits + (int64_t)r * a.max_pools;
    const int K = P - 1;
    uint32_t prefix = 0u, mask = 0u;
    int rem = K;
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      int* h = hist2[pass & 1];
      for (int i = tid; i < 256; i += bd) h[i] = 0;
      __syncthreads();
      for (int j = j0 + tid; j < j1; j += bd) {
        const uint32_t u = order_key(lg[j]);
        if ((u & mask) == prefix) atomicAdd(&h[(u >> shift) & 255u], 1);
      }
      cl_sync();                            // every slice's histogram of this pass is complete
      if (tid < 32) {
        int cnt[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) cnt[i] = 0;
        for (int k = 0; k < nc; ++k) {      // fixed rank order: every CTA forms the same sums
          const int* hk = cl_map(h, k);
#pragma unroll
          for (int i = 0; i < 8; ++i) cnt[i] += hk[255 - 8 * tid - i];
        }
        sel_decide(cnt, prefix, shift, rem, &c_prefix, &c_rem);
      }
      __syncthreads();
      prefix = c_prefix;
      rem = c_rem;
      mask |= 255u << shift;
    }
    // counts of this slice: keys above the threshold and keys equal to it
    if (tid < 2) c_cnt[tid] = 0;
    __syncthreads();
    int gt_l = 0, eq_l = 0;
    for (int j = j0 + tid; j < j1; j += bd) {
      const uint32_t u = order_key(lg[j]);
      gt_l += u > prefix;
      eq_l += u == prefix;
    }
    gt_l = warp_sum_int(gt_l);
    eq_l = warp_sum_int(eq_l);
    if ((tid & 31) == 0) { atomicAdd(&c_cnt[0], gt_l); atomicAdd(&c_cnt[1], eq_l); }
    cl_sync();
    // output offset of this slice: the pools selected by the lower ranks (ties in index order, first rem taken)
    int base_sel = 0, base_eq = 0;
    for (int k = 0; k < rank; ++k) {
      const int* ck = cl_map(c_cnt, k);
      const int gk = ck[0], ek = ck[1];
      base_sel += gk + max(0, min(ek, rem - base_eq));
      base_eq += ek;
    }
    cl_sync();                              // no CTA leaves while another reads its counts
    for (int jb = j0; jb < j1; jb += bd) {
      const int j = jb + tid;
      const uint32_t u = j < j1 ? order_key(lg[j]) : 0u;
      const int eq = (j < j1) && (u == prefix);
      const int gt = (j < j1) && (u > prefix);
      const int2 se = block_scan(eq, c_wsum);
      const int selected = gt || (eq && (base_eq + se.x) < rem);
      const int2 ss = block_scan(selected, c_wsum);
      if (selected) {
        const int o = (base_sel + ss.x) * kp;
        for (int i = 0; i < kp; ++i) out[o + i] = slot_of(bt, a.block_size, j * kp + i);
      }
      base_eq += se.y;
      base_sel += ss.y;
    }
    if (rank == 0) {
      for (int p = c * kp + tid; p <= pos; p += bd) out[K * kp + (p - c * kp)] = slot_of(bt, a.block_size, p);
      if (tid == 0) a.sel_count[r] = K * kp + (pos - c * kp + 1);
    }
    return;
  }
  if (rank != 0) return;                    // short rows: rank 0 alone
  if (c <= P - 1) {
    for (int p = tid; p <= pos; p += bd) out[p] = slot_of(bt, a.block_size, p);
    if (tid == 0) a.sel_count[r] = pos + 1;
    return;
  }
  const int K = P - 1;
  const float* lg = a.logits + (int64_t)r * a.max_pools;
  __shared__ int hist[256];
  __shared__ uint32_t s_prefix;
  __shared__ int s_rem;
  __shared__ int wsum[32];
  uint32_t prefix = 0u, mask = 0u;
  int rem = K;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = tid; i < 256; i += bd) hist[i] = 0;
    __syncthreads();
    for (int j = tid; j < c; j += bd) {
      const uint32_t u = order_key(lg[j]);
      if ((u & mask) == prefix) atomicAdd(&hist[(u >> shift) & 255u], 1);
    }
    __syncthreads();
    if (tid < 32) {
      // the highest bin b whose count from the top (bins 255..b) reaches rem (bin 0 when bins 255..1 do not)
      int cnt[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) cnt[i] = hist[255 - 8 * tid - i];
      sel_decide(cnt, prefix, shift, rem, &s_prefix, &s_rem);
    }
    __syncthreads();
    prefix = s_prefix;
    rem = s_rem;
    mask |= 255u << shift;
  }
  int base_eq = 0, base_sel = 0;
  for (int j0 = 0; j0 < c; j0 += bd) {
    const int j = j0 + tid;
    const uint32_t u = j < c ? order_key(lg[j]) : 0u;
    const int eq = (j < c) && (u == prefix);
    const int gt = (j < c) && (u > prefix);
    const int2 se = block_scan(eq, wsum);
    const int selected = gt || (eq && (base_eq + se.x) < rem);
    const int2 ss = block_scan(selected, wsum);
    if (selected) {
      const int o = (base_sel + ss.x) * kp;
      for (int i = 0; i < kp; ++i) out[o + i] = slot_of(bt, a.block_size, j * kp + i);
    }
    base_eq += se.y;
    base_sel += ss.y;
  }
  for (int p = c * kp + tid; p <= pos; p += bd) out[K * kp + (p - c * kp)] = slot_of(bt, a.block_size, p);
  if (tid == 0) a.sel_count[r] = K * kp + (pos - c * kp + 1);
}

}  // namespace g53

using namespace g53;

cudaError_t g53_dsa_update(const DsaArgs& a, cudaStream_t st) {
  if (a.ID != 128) return cudaErrorInvalidValue;
  dsa_keys_kernel<<<a.R, 128, 0, st>>>(a);
  G53_CHECK_LAUNCH();
  dsa_pool_kernel<<<(a.R + 7) / 8, 256, 0, st>>>(a);
  G53_CHECK_LAUNCH();
  dsa_ring_kernel<<<a.R, 128, 0, st>>>(a);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}

cudaError_t g53_dsa_logits(const DsaArgs& a, cudaStream_t st) {
  if (a.ID != 128 || a.IH > kMaxIH) return cudaErrorInvalidValue;
  // paired with the tcgen05 kernel, this kernel only serves launches whose rows have at most tc_min_pools pools
  const int pools = a.tc_min_pools > 0 ? std::min(a.max_pools, a.tc_min_pools) : a.max_pools;
  dim3 grid(a.R, (pools + 255) / 256);
  dsa_logits_kernel<<<grid, 256, 0, st>>>(a);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}

cudaError_t g53_dsa_select(const DsaArgs& a, cudaStream_t st) {
  // clusters of kSelNC CTAs for decode-sized launches (fewer than 64 rows: one CTA per row would leave most SMs
  // idle) whose logits buffer can hold rows long enough for the split path; prefill chunks keep one CTA per row
  const int nc = (a.R < 64 && a.max_pools > kSelSplit) ? kSelNC : 1;
  return g53_launch_pdl(dsa_select_kernel, dim3(a.R, 1, nc), dim3(1024), 0, st, nc, a);
}
