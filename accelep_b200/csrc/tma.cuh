// Bulk-copy (TMA) and mbarrier helpers in inline PTX for sm_100a.
//
// This header holds the untiled global -> shared bulk copy and the L2
// prefetch; the tiled tensor-map copies (cp.async.bulk.tensor) of the
// tensor-core product live in gemm_tc.cu. Every copy in this library has a
// CTA-local destination and no cluster multicast: it reads this GPU's own
// memory into the issuing CTA's shared memory. Waits on an mbarrier are
// bounded; a wait that runs out reports failure to its caller instead of
// spinning on.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace accel_b200 {

// Upper bound on the wait for one mbarrier phase: 2^31 SM clock cycles (about
// one second at 1.9 GHz, under two at the lowest clocks), far beyond any real
// copy or MMA latency (microseconds). The cycle counter is cheap to read,
// unlike the global timer, and is read only after a run of failed polls.
constexpr long long kWaitLimitCycles = 1ll << 31;

__device__ __forceinline__ uint64_t GlobalTimerNs() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t SmemAddr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void MbarInit(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(SmemAddr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void FenceBarrierInit() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// One arrival that also announces `bytes` of incoming transactions.
__device__ __forceinline__ void MbarArriveExpectTx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(SmemAddr(bar)), "r"(bytes) : "memory");
}

// One plain arrival.
__device__ __forceinline__ void MbarArrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(SmemAddr(bar)) : "memory");
}

// Global -> shared bulk copy completing on `bar`. dst, src and bytes must be
// multiples of 16.
__device__ __forceinline__ void BulkCopyG2S(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(SmemAddr(dst)),
      "l"(src), "r"(bytes), "r"(SmemAddr(bar))
      : "memory");
}

// The same copy with an L2 eviction policy (a createpolicy value).
__device__ __forceinline__ void BulkCopyG2SHint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          SmemAddr(dst)),
      "l"(src), "r"(bytes), "r"(SmemAddr(bar)), "l"(policy)
      : "memory");
}

// L2 policy for data read once: evicted before other lines.
__device__ __forceinline__ uint64_t EvictFirstPolicy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

// Brings [src, src + bytes) into L2 (a hint; src and bytes multiples of 16).
__device__ __forceinline__ void PrefetchL2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Non-blocking test of phase `parity`: the waiting thread is never suspended,
// so a completed phase is seen on the next poll (a suspended try_wait adds a
// wake-up delay to every hand-off of a pipeline).
__device__ __forceinline__ bool MbarTryWait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(SmemAddr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// The polling loop of MbarWait, out of line: every wait site of a kernel
// would otherwise carry its own copy of it.
static __device__ __noinline__ bool MbarWaitPoll(uint64_t* bar, uint32_t parity) {
  const long long start = clock64();
  for (;;) {
    for (int i = 0; i < 256; ++i) {
      if (MbarTryWait(bar, parity)) return true;
    }
    if (clock64() - start > kWaitLimitCycles) return false;
  }
}

// Waits for phase `parity` of `bar` to complete; false when the bound ran out.
__device__ __forceinline__ bool MbarWait(uint64_t* bar, uint32_t parity) {
  if (MbarTryWait(bar, parity)) return true;
  return MbarWaitPoll(bar, parity);
}

// The same wait with the suspending try_wait: the thread sleeps inside the
// instruction until the phase completes or a hardware time limit passes. For
// long waits of warps with nothing else to do, so that they take no issue
// slots from the warps that work meanwhile.
__device__ __forceinline__ bool MbarWaitSleep(uint64_t* bar, uint32_t parity) {
  const long long start = clock64();
  for (;;) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(SmemAddr(bar)), "r"(parity)
        : "memory");
    if (done != 0) return true;
    if (clock64() - start > kWaitLimitCycles) return false;
  }
}

}  // namespace accel_b200
