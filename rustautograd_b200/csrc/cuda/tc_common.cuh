// Device primitives shared by the tcgen05 kernels (gemm_tc.cu, attention.cu): mbarriers with
// bounded waits, the K-major 128-byte-swizzle shared-memory descriptor, single-CTA TF32 products
// into TMEM and their commits, TMEM loads, and the TF32 split.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace rgc {
namespace tc {

// Every mbarrier wait gives up after this long (2 s) and reports through an error flag.
constexpr unsigned long long WAIT_LIMIT_NS = 2000000000ull;

__device__ __forceinline__ uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(bar)) : "memory");
}

// CLUSTER: acquire at cluster scope, for barriers that the other CTA of a pair arrives on.
template <bool CLUSTER = false> __device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  if (CLUSTER)
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(saddr(bar)), "r"(phase)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(saddr(bar)), "r"(phase)
        : "memory");
  return ok != 0;
}

// Waits for `phase` of `bar`; gives up after WAIT_LIMIT_NS or when another role aborted.
template <bool CLUSTER = false> __device__ bool mbar_wait(uint64_t* bar, uint32_t phase, volatile int* abort, int* err, int code) {
  unsigned long long t0 = 0;
  for (int spin = 0;; ++spin) {
    if (mbar_try<CLUSTER>(bar, phase)) return true;
    if (*abort) return false;
    if (spin == 64) t0 = now_ns();
    if (spin > 64 && now_ns() - t0 > WAIT_LIMIT_NS) {
      *abort = 1;
      atomicExch(err, code);
      return false;
    }
  }
}

// Shared-memory matrix descriptors (tcgen05 "matrix descriptor", version 1, 128-byte swizzle).
// K-major tile: rows of 32 fp32 (128 B) along K, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t desc_k(uint32_t addr) {
  uint64_t d = (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;            // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;  // stride byte offset: next 8-row group
  d |= (uint64_t)1 << 46;            // descriptor version
  d |= (uint64_t)2 << 61;            // 128-byte swizzle
  return d;
}
__device__ __forceinline__ void mma_tf32(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  const uint32_t no_mask = 0;  // disable-output-lane mask: every lane written
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(no_mask)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(bar)) : "memory");
}

__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,"
      "%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]),
        "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]),
        "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]),
        "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// The TF32 value the tensor cores take from an fp32 operand: its low 13 mantissa bits dropped.
__device__ __forceinline__ float tf32_trunc(float v) { return __uint_as_float(__float_as_uint(v) & 0xFFFFE000u); }

}  // namespace tc
}  // namespace rgc
