// Shared-memory staging with the sm_100 bulk-copy engine (TMA, 1-D form):
// cp.async.bulk global -> shared completing on an mbarrier transaction
// count, plus the bounded wait every kernel here uses on such a barrier.
//
// No wait in this library spins forever: after kWaitPolls polls of
// mbarrier.try_wait (each of which may suspend the thread for a short,
// hardware-chosen time) the wait gives up and the kernel counts the event
// in f4s_wait_timeouts, a module-global the host reads back
// (f4s_hotpath_wait_timeouts).  A non-zero count means some output was not
// written.
#pragma once

#include "common.cuh"

// Number of bounded waits that gave up since the host last cleared it.
__device__ unsigned int f4s_wait_timeouts;

namespace f4s {

constexpr uint32_t kWaitPolls = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t arrivals) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(arrivals) : "memory");
}

// Makes barrier initialisation visible to the bulk-copy (async) proxy.
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Arrive once and add `bytes` to the phase's expected transaction count.
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Bulk copy `bytes` (multiple of 16, both addresses 16-byte aligned) from
// global memory into this CTA's shared memory; completion is counted on
// `bar`.  No multicast.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses before
// a following bulk copy into the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{ .reg .pred p;\n"
      "  mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "  selp.u32 %0, 1, 0, p; }"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Wait for the phase of `bar` with the given parity to complete, at most
// `polls` polls; false when it gave up.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t polls = kWaitPolls) {
  for (uint32_t i = 0; i < polls; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  return false;
}

}  // namespace f4s

// Diagnostic: arms an mbarrier for 16 bytes that no copy will deliver and
// waits for it with the same bounded wait as the staging kernels, `polls`
// polls at most.  The give-up path counts in f4s_wait_timeouts exactly as
// a real timeout would; the host checks that the count rises and that the
// context stays usable.  One thread, no memory traffic.
extern "C" __global__ void f4s_check_bounded_wait(unsigned int polls) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  f4s::mbar_init(&bar, 1);
  f4s::mbar_init_fence();
  f4s::mbar_expect_tx(&bar, 16);
  if (!f4s::mbar_wait_bounded(&bar, 0, polls)) atomicAdd(&f4s_wait_timeouts, 1u);
}
