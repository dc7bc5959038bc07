// Tensor-memory-accelerator (TMA) copies and shared-memory mbarriers for
// sm_100a, as inline PTX; host-side tensor-map encoding through the driver
// entry point (no link-time dependency on libcuda).
//
// Every wait here is bounded: after `kSpinLimit` polls it gives up and
// returns false, so a copy that never lands cannot hang the GPU; callers
// record an error and stop.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace fxpr {
namespace tma {

constexpr uint32_t kSpinLimit = 1u << 22;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// arrive once and add `bytes` to the transaction count the phase waits for
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred P; mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2; selp.u32 %0, 1, 0, P; }"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded wait for the phase with the given parity to complete
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// order this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (TMA) writes to the same buffer
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// L2 policy: stream once (evict first)
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 4-D tiled load of one box into shared memory, completing on `bar`
__device__ __forceinline__ void load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                        int c3, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_addr(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// contiguous copy global -> shared (16-byte aligned, size a multiple of 16)
__device__ __forceinline__ void load_bulk(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------
// Encode a 4-D tiled tensor map of 2-byte elements: dims (innermost first)
// and byte strides of dims 1..3; box sizes per dim. Returns false (with the
// library error set) if the driver entry point is missing or rejects it.
bool encode_4d_u16(CUtensorMap* map, const void* base, const uint64_t dims[4],
                   const uint64_t strides_bytes[3], const uint32_t box[4]);

}  // namespace tma
}  // namespace fxpr
