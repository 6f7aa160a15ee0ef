// bulk.cuh -- bulk copies (cp.async.bulk, global -> shared) that complete
// on an mbarrier, and bounded waits on it.
//
// Every wait gives up after kBulkWaitNs of global time (or 2^22 polls);
// the caller then counts a fault in the context's device counter, which
// ckks_sync reports, and leaves its outputs unwritten, so a copy that never
// completes cannot hang the GPU.
#pragma once
#include <cstdint>

namespace ckks {

constexpr uint64_t kBulkWaitNs = 1000000000ull;  // one second

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// waits for the barrier's phase `parity` to complete; gives up after
// kBulkWaitNs of global time or 2^22 polls, whichever comes first
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0; i < (1u << 22); ++i) {
    if (mbar_test(bar, parity)) return true;
    if ((i & 31u) == 31u && global_ns() - t0 > kBulkWaitNs) return false;
  }
  return false;
}

}  // namespace ckks
