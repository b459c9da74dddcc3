// Bulk-copy (TMA engine) and mbarrier helpers for sm_100a, written as inline
// PTX.  Every wait is bounded: after M5_WAIT_LIMIT failed polls the caller
// gets `false`, records an error code in the word `err` points at (a sticky
// per-translation-unit device flag read back by m5_device_error) and must
// leave its loop.
#pragma once

#include "common.cuh"

namespace m5 {

constexpr uint32_t M5_WAIT_LIMIT = 1u << 20;  // polls (each up to ~2 us of suspension) before a wait gives up
enum { M5_DEV_ERR_WAIT_TIMEOUT = 1 };

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

// Make mbarrier initialisation visible to the async (bulk copy) proxy.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// One poll; the thread may be suspended by the hardware for up to ~2 us
// while the phase is incomplete, so a waiting warp does not burn issue slots.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(2000u)
      : "memory");
  return ok != 0;
}

// One poll without a suspend-time hint: the hardware may still suspend the
// thread for a short system-defined time while the phase is incomplete.
__device__ __forceinline__ bool mbar_try_wait_fast(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait until the phase with `parity` completed; false (and error recorded) on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  for (uint32_t i = 0; i < M5_WAIT_LIMIT; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  atomicExch(err, M5_DEV_ERR_WAIT_TIMEOUT);
  return false;
}

// Named barrier among `threads` threads (a subset of the CTA, e.g. the consumer warps).
__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// 1-D bulk copy global -> this CTA's shared memory, completing `bytes` of
// transaction count on `bar`.  dst, src 16-byte aligned; bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Same, with an L2 evict-first hint (streamed weights are read once per token).
__device__ __forceinline__ void bulk_g2s_stream(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}


}  // namespace m5
