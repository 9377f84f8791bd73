// Small sm_100a building blocks shared by the tcgen05 kernels: mbarriers with bounded waits, UMMA shared-memory and
// instruction descriptors for K-major 128-byte-swizzled operands, tcgen05.mma / commit / ld, TMEM alloc.
#pragma once
#include <cstdint>

namespace g53 {
namespace tc {

constexpr uint32_t kSpin = 1u << 26;     // bounded mbarrier waits (then an error word is set and the CTA stops)

__device__ __forceinline__ uint32_t saddr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void bar_init(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(b)), "r"(n));
}
__device__ __forceinline__ void bar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(b)) : "memory");
}
__device__ __forceinline__ bool bar_try(uint64_t* b, uint32_t ph) {
  uint32_t ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0,1,0,p;\n}\n"
               : "=r"(ok) : "r"(saddr(b)), "r"(ph) : "memory");
  return ok != 0;
}
// false when the limit ran out (records `code` in *err) or another thread of the CTA already failed
__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t ph, volatile int* fail, int* err, int code) {
  uint32_t n = 0;
  while (!bar_try(b, ph)) {
    if (*fail) return false;
    if (++n > kSpin) {
      *fail = 1;
      if (err) atomicExch(err, code);
      return false;
    }
    if (n > 64) __nanosleep(32);
  }
  return true;
}
// warp-uniform wait: lane 0 polls, the result is broadcast
__device__ __forceinline__ bool warp_wait(uint64_t* b, uint32_t ph, volatile int* fail, int* err, int code) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = bar_wait(b, ph, fail, err, code) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// shared-memory writes by threads become visible to the tensor core (async proxy)
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// K-major operand, 128-byte swizzle, 8-row groups 1024 bytes apart
__device__ __forceinline__ uint64_t desc_sw128(uint32_t s) {
  uint64_t d = (uint64_t)((s >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
// D f32; A/B format (0 f16, 1 bf16), both K-major; N; M
__device__ __forceinline__ uint32_t idesc(int fmt, int n, int m) {
  return (1u << 4) | ((uint32_t)fmt << 7) | ((uint32_t)fmt << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void mma_f16(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile("{\n .reg .pred p;\n setp.ne.u32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
               ::"r"(d), "l"(a), "l"(b), "r"(id), "r"(acc));
}
__device__ __forceinline__ void commit(uint64_t* b) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(b)) : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// one warp allocates (and later frees) `cols` TMEM columns; the base address lands in *dst
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(dst)), "r"(cols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_free(uint32_t base, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols));
}

// 32 consecutive fp32 columns of this thread's TMEM lane (warp quadrant = warp % 4)
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

// byte offset of the 16-byte chunk holding elements [8c, 8c + 8) (16-bit elements) of row `row` in a K-major
// tile whose rows are 128 bytes (64 elements) and which is 1024-byte aligned: 128-byte swizzle
__device__ __forceinline__ uint32_t sw128_chunk(int row, int c) {
  return (uint32_t)(row * 128 + ((c ^ (row & 7)) << 4));
}

}  // namespace tc
}  // namespace g53
