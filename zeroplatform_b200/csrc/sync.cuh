// sync.cuh -- mbarrier, bulk-copy and bounded-wait helpers shared by the TMA-fed kernels (sm_100a).
//
// Every wait on an mbarrier is bounded: after WAIT_LIMIT polls or WAIT_NS nanoseconds the waiting thread
// raises its CTA's abort flag, records a code in a device status word and returns false, so a kernel whose
// producer or consumer failed ends with an error the host can read instead of hanging the GPU.
#pragma once

#include <stdint.h>

namespace zc {

constexpr uint32_t WAIT_LIMIT = 1u << 24;    // try_wait polls before a wait is declared hung
constexpr uint64_t WAIT_NS = 2000000000ull;  // ... or two seconds

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait: gives up after WAIT_LIMIT polls or WAIT_NS nanoseconds, whichever comes first, raising
// the CTA abort flag and recording `code` in the device status word.  Returns false when it gave up or
// when another role of the CTA already aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status,
                                          int code) {
  uint64_t t0 = 0;
  for (uint32_t i = 0; i < WAIT_LIMIT; ++i) {
    if (mbar_try(bar, parity)) return true;
    if ((i & 255) == 255) {
      if (*abort_flag) return false;
      const uint64_t now = global_ns();
      if (t0 == 0) t0 = now;
      else if (now - t0 > WAIT_NS) break;
    }
  }
  *abort_flag = 1;
  atomicExch(status, code);
  return false;
}

// Bulk copy global -> shared (no tensor map, no multicast): `bytes` and both addresses are multiples of 16;
// completion is signalled on `bar` as transaction bytes.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// Bulk prefetch of [src, src + bytes) into L2 (no shared memory, no completion signal); 16-byte multiples.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

}  // namespace zc
