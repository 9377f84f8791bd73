// Expert-parallel routed MoE with the all-to-all dispatch and combine fused into the kernels (peer memory over
// NVLink; no NCCL on this path).  Rank d owns experts [d*El, (d+1)*El) at full width.
//
// Per step (parity p = step % 2 selects one of two buffer sets, so a rank that runs ahead never overwrites a buffer
// a slower rank still reads; epoch[p] counts completed steps of parity p):
//   source   route (moe.cu) -> pairs sorted by expert, i.e. by (destination rank, local expert)
//            ep_dispatch:   block per sorted pair: the token row (bf16) -> recv_x[p][src][row] on the owner rank
//                           (16-byte peer stores), meta {local expert, source pair, weight}; block 0 also writes the
//                           per-local-expert counts; the last block releases disp_flag[p][src] on every rank
//   receiver ep_plan:       waits (bounded) for every source's flag, orders its rows by (local expert, source) so
//                           each expert is one group (its trellis decoded once), writes the group table
//            ep_pairs:      per receiver row: source row, local expert, weight, and the address of the source's
//                           combine slot for that pair (peer memory)
//            exl3 rot_in / gate_up / down (moe.cu); the down epilogue stores each weighted output row straight
//                           into the source rank's combine buffer and its last CTA releases comb_flag[p][dst] there
//   source   ep_combine:    waits (bounded) for every destination's flag, sums each token's top-k rows in slot
//                           order (deterministic), then advances epoch[p]
// Every wait gives up after ~2^22 polls and records an error code; the host checks it after the step.
// Reference counterpart: the EP path of the reference exists but is not deployed (its MoE runs TP-only:
// code/fork/docs/prod_exl3_reference.py:924-958 expert_map); its all2all backend is NCCL.
#include "common.cuh"
#include "launchers.h"

namespace g53 {

__device__ __forceinline__ int lower_bound_i(const int* a, int n, int v) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (a[mid] < v) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// rows written by peers: read past L1 (no stale lines from an earlier step)
__device__ __forceinline__ float4 ld_volatile_f4(const float* p) {
  float4 v;
  asm volatile("ld.volatile.global.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}

// last block of the grid (after every block's writes are visible system-wide) raises the flags of `world` ranks
__device__ __forceinline__ void last_block_release(unsigned* done, const int64_t* flags, int world) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned prev = atomicAdd(done, 1u);
    if (prev == gridDim.x * gridDim.y * gridDim.z - 1) {
      *done = 0u;
      __threadfence_system();
      for (int d = 0; d < world; ++d) red_release_sys_add(reinterpret_cast<unsigned*>(flags[d]), 1u);
    }
  }
}

// grid (P) blocks x 128 threads
__global__ void __launch_bounds__(128) ep_dispatch_kernel(EpArgs a) {
  const int p = blockIdx.x;
  const int np = *a.n_pairs;
  if (p < np) {
    const int e = a.pair_expert[p];
    const int d = e / a.El;
    const int first = lower_bound_i(a.pair_expert, np, d * a.El);
    const int row = p - first;
    if (row < a.cap) {
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.recv_x[d]) + ((int64_t)a.rank * a.cap + row) * a.K;
      const __nv_bfloat16* src = a.x + (int64_t)a.pair_token[p] * a.ldx;
      for (int c = threadIdx.x * 8; c < a.K; c += blockDim.x * 8)
        *reinterpret_cast<uint4*>(dst + c) = *reinterpret_cast<const uint4*>(src + c);
      if (threadIdx.x == 0) {
        int4* meta = reinterpret_cast<int4*>(a.recv_meta[d]) + (int64_t)a.rank * a.cap + row;
        *meta = make_int4(e - d * a.El, p, __float_as_int(a.pair_w[p]), 0);
      }
    } else if (threadIdx.x == 0) {
      atomicExch(a.err, 52);                      // a source region overflowed (never with cap >= pairs)
    }
  }
  if (p == 0) {
    // counts per (destination, local expert) of this source
    for (int i = threadIdx.x; i < a.world * a.El; i += blockDim.x) {
      const int d = i / a.El, le = i % a.El, ge = d * a.El + le;
      const int c = lower_bound_i(a.pair_expert, np, ge + 1) - lower_bound_i(a.pair_expert, np, ge);
      reinterpret_cast<int*>(a.recv_cnt[d])[a.rank * a.El + le] = c;
    }
  }
  last_block_release(a.done, a.disp_flags, a.world);
}

// 1 block x 1024 threads: wait for all sources, group table (local expert-major, then source)
__global__ void __launch_bounds__(1024) ep_plan_kernel(EpArgs a) {
  __shared__ int base[1024];
  __shared__ int wsum[32];
  __shared__ unsigned target;
  const int tid = threadIdx.x;
  const int n = a.world * a.El;                   // <= 1024 (checked on the host)
  if (tid == 0) {
    target = *reinterpret_cast<volatile unsigned*>(a.epoch) + 1u;
    for (int s = 0; s < a.world; ++s) wait_flag_geq(a.my_disp_flags + s, target, a.err, 51);
  }
  __syncthreads();
  // entry i = le * world + s  (counts were written by source s at [s][le])
  const int le = tid / max(a.world, 1), s = tid % max(a.world, 1);
  const int c = tid < n ? ld_acquire_sys(reinterpret_cast<const unsigned*>(a.my_cnt + s * a.El + le)) : 0;
  const int2 sc = block_scan(c, wsum);
  if (tid < n) {
    base[tid] = sc.x;
    a.seg_base[tid] = sc.x;
    a.seg_cnt[tid] = c;
  }
  if (tid == 0) *a.n_recv = sc.y;
  __syncthreads();
  if (tid == 0) {
    int u = 0;
    for (int l = 0; l < a.El; ++l) {
      const int b0 = base[l * a.world];
      const int b1 = (l + 1) * a.world < n ? base[(l + 1) * a.world] : sc.y;
      if (b1 > b0) { a.group_expert[u] = l; a.group_offset[u] = b0; ++u; }
    }
    a.group_count[0] = u;
    for (int v = u; v <= a.El; ++v) a.group_offset[v] = sc.y;
    // source-region offsets: row of (s, le) segment starts after the source's rows of lower local experts
    for (int s2 = 0; s2 < a.world; ++s2) {
      int acc = 0;
      for (int l = 0; l < a.El; ++l) {
        a.seg_src[l * a.world + s2] = acc;
        acc += ld_acquire_sys(reinterpret_cast<const unsigned*>(a.my_cnt + s2 * a.El + l));
      }
    }
  }
}

// receiver rows: grid (ceil(recv_cap / 256)) x 256
__global__ void __launch_bounds__(256) ep_pairs_kernel(EpArgs a) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int nr = *a.n_recv;
  if (i >= nr) return;
  if (i >= a.recv_cap) {
    if (i == a.recv_cap) atomicExch(a.err, 53);
    return;
  }
  const int n = a.world * a.El;
  // last segment with base <= i
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (a.seg_base[mid] <= i) lo = mid; else hi = mid - 1;
  }
  while (lo + 1 < n && a.seg_cnt[lo] == 0 && a.seg_base[lo + 1] <= i) ++lo;
  const int s = lo % a.world, le = lo / a.world;
  const int row = a.seg_src[lo] + (i - a.seg_base[lo]);
  const int4 m = reinterpret_cast<const int4*>(a.my_meta)[(int64_t)s * a.cap + row];
  a.rp_token[i] = s * a.cap + row;
  a.rp_expert[i] = le;
  a.rp_w[i] = __int_as_float(m.z);
  a.rp_out[i] = a.comb[s] + (int64_t)m.y * a.K * (int64_t)sizeof(float);
}

// grid (K/4/256, R): wait for every destination, out[r] = sum_k comb[pair_of[r, k]]; last block advances the epoch
__global__ void __launch_bounds__(256) ep_combine_kernel(EpArgs a, const int* pair_of, int R, int top_k, float* out) {
  __shared__ unsigned target;
  if (threadIdx.x == 0) {
    target = *reinterpret_cast<volatile unsigned*>(a.epoch) + 1u;
    for (int d = 0; d < a.world; ++d) wait_flag_geq(a.my_comb_flags + d, target, a.err, 54);
  }
  __syncthreads();
  const int r = blockIdx.y;
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (r < R && c < a.K) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < top_k; ++k) {
      const float4 v = ld_volatile_f4(a.my_comb + (int64_t)pair_of[r * top_k + k] * a.K + c);
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    *reinterpret_cast<float4*>(out + (int64_t)r * a.K + c) = acc;
  }
  // every block has read the epoch before counting in: the last one advances it
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(a.done2, 1u);
    if (prev == gridDim.x * gridDim.y - 1) {
      *a.done2 = 0u;
      __threadfence();
      atomicAdd(a.epoch, 1u);
    }
  }
}

}  // namespace g53

using namespace g53;

// one thread: everything this rank wrote before (stream order) becomes visible system-wide, then flag [rank] is
// raised on every rank (publication of a shard for all-gather + GEMM)
__global__ void signal_peers_kernel(const int64_t* flags, int rank, int world) {
  __threadfence_system();
  for (int j = 0; j < world; ++j) red_release_sys_add(reinterpret_cast<unsigned*>(flags[j]) + rank, 1u);
}

cudaError_t g53_signal_peers(const int64_t* flags, int rank, int world, cudaStream_t st) {
  signal_peers_kernel<<<1, 1, 0, st>>>(flags, rank, world);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}

cudaError_t g53_ep_dispatch(const EpArgs& a, int max_pairs, cudaStream_t st) {
  if (a.K % 8 || a.world * a.El > 1024 || max_pairs < 0) return cudaErrorInvalidValue;
  // at least one block: it writes the (possibly zero) counts and releases the flags
  ep_dispatch_kernel<<<max_pairs > 0 ? max_pairs : 1, 128, 0, st>>>(a);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}

cudaError_t g53_ep_plan(const EpArgs& a, cudaStream_t st) {
  if (a.world * a.El > 1024) return cudaErrorInvalidValue;
  ep_plan_kernel<<<1, 1024, 0, st>>>(a);
  G53_CHECK_LAUNCH();
  ep_pairs_kernel<<<(a.recv_cap + 255) / 256, 256, 0, st>>>(a);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}

cudaError_t g53_ep_combine(const EpArgs& a, const int* pair_of, int R, int top_k, float* out, cudaStream_t st) {
  if (a.K % 4 || R < 0) return cudaErrorInvalidValue;
  dim3 grid((a.K / 4 + 255) / 256, R > 0 ? R : 1);   // a rank without tokens still waits and advances its epoch
  ep_combine_kernel<<<grid, 256, 0, st>>>(a, pair_of, R, top_k, out);
  G53_CHECK_LAUNCH();
  return cudaSuccess;
}
