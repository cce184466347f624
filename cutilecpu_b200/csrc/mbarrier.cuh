// mbarrier.cuh — shared-memory barriers, bounded waits and 2-D TMA copies
// (inline PTX for sm_100a) used by the warp-specialised kernels (sgemm, scan).
// No copy here carries cluster multicast.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace mk {
namespace tma {

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Complete `bytes` of the current phase's transaction count without a copy:
// stands in for a copy that was never issued, so a drain can wait for a phase.
__device__ __forceinline__ void mbar_complete_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.complete_tx.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Budget of the waits that make a kernel's exit safe after an abort (copies
// and MMAs already issued must land before shared memory or TMEM is given
// back).  Fixed, so a small MK_WAIT_LIMIT_CYCLES cannot cut a drain short:
// 2^27 SM cycles is about 70 ms at 1.9 GHz, while an issued copy lands in
// microseconds.
constexpr unsigned long long kDrainCycles = 1ull << 27;

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of `bar` to complete; false on timeout (`limit` SM
// cycles) or when another role raised `abort_flag`.
__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity, unsigned long long limit,
                                             volatile int* abort_flag) {
  const long long t0 = clock64();
  uint32_t spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++spins & 63u) == 0) {
      if (*abort_flag) return false;
      if ((unsigned long long)(clock64() - t0) > limit) return false;
    }
  }
  return true;
}

// 2-D tiled TMA load global -> shared, completing on `bar` (this CTA).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(map), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

// 2-D tiled TMA store shared -> global in the current bulk group.  The box is
// clipped at the tensor's bounds; c0, c1 must be >= 0.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int c0, int c1, uint32_t src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map), "r"(c0),
               "r"(c1), "r"(src)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Wait until at most N committed bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until every committed bulk group has completed (writes visible).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Make this thread's generic-proxy shared-memory writes visible to the TMA.
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Barrier over `count` threads (a multiple of 32) on hardware barrier `id`.
__device__ __forceinline__ void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

}  // namespace tma
}  // namespace mk
