// Bulk-copy staging pipeline shared by the streaming (HBM-bound) kernels.
//
// One producer thread per CTA streams input tiles from HBM into a ring of
// shared-memory stages with cp.async.bulk (completion counted in bytes on a
// "full" mbarrier per stage); the consumer warps compute from shared memory,
// write their results straight to global memory and release the stage on
// its "empty" mbarrier.  Every wait is bounded: after ~2 s it records
// MOSS_ERR_TIMEOUT in the device error word and reports failure, and the
// caller then stops issuing work, drains the copies it has in flight and
// returns.
#pragma once

#include "common.cuh"

namespace moss {
namespace pipe {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(unsigned long long* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(unsigned long long* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(unsigned long long* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(unsigned long long* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Waits for the phase of the given parity; false (after recording a
// timeout) when it has not completed within `limit_ns` (~2 s by default).
__device__ __forceinline__ bool mbar_wait(unsigned long long* bar, uint32_t parity,
                                          uint64_t limit_ns = kWaitLimitNs) {
  return bounded_wait([&] { return mbar_try_wait(bar, parity); }, limit_ns);
}
// Global -> shared bulk copy; dst, src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Barrier among the first `threads` threads of the CTA (the consumer warps).
__device__ __forceinline__ void consumer_sync(int threads) {
  asm volatile("bar.sync 1, %0;" ::"r"(threads) : "memory");
}

}  // namespace pipe
}  // namespace moss
