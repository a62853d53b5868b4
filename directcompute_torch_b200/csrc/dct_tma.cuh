// Bulk-copy (TMA engine) and mbarrier helpers for sm_100a, as inline PTX.
//
// Only the non-multicast, CTA-local forms are used: a 1-D
// cp.async.bulk global -> this CTA's shared memory, completing on an mbarrier
// with a transaction-byte count.  Every wait is bounded: a wait that runs out
// sets the library's device error word and returns false, so a kernel can
// finish its (uniform) control flow instead of hanging.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "dct_common.cuh"

namespace dct {

DCT_DEV uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

DCT_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

DCT_DEV void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

// arrive (count 1) and add `bytes` to the expected transaction count
DCT_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

DCT_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for phase `parity` of `bar`: at most `limit` polls; false (and
// the error bit set) when they run out.
DCT_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err, uint32_t limit = 1u << 22) {
  for (uint32_t spins = 0; spins < limit; ++spins)
    if (mbar_try_wait(bar, parity)) return true;
  if (err) atomicOr(err, DCT_DEVERR_WAIT_TIMEOUT);
  return false;
}

// 1-D bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned)
// from global memory into this CTA's shared memory, completing on `bar`.
DCT_DEV void bulk_load(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// order this thread's generic-proxy shared-memory accesses before later
// async-proxy (bulk copy) accesses to the same memory
DCT_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

}  // namespace dct
