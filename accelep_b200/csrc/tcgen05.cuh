// 5th-generation tensor core (tcgen05) helpers in inline PTX for sm_100a:
// TMEM allocation, shared-memory matrix descriptors, the int8 MMA with int32
// accumulation in TMEM, commit to an mbarrier, and TMEM loads.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace accel_b200 {

// --------------------------------------------------------------------- TMEM

// One warp allocates `cols` TMEM columns (a power of two >= 32) and writes the
// base address to shared memory.
__device__ __forceinline__ void TmemAlloc(uint32_t* smem_dst, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void TmemDealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

__device__ __forceinline__ void TcFenceBeforeSync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void TcFenceAfterSync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Makes this thread's generic-proxy shared-memory writes visible to the
// tensor core (async proxy).
__device__ __forceinline__ void FenceProxyAsyncSmem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ------------------------------------------------------------- descriptors

// Shared-memory matrix descriptor (sm_100): start address, leading and stride
// byte offsets (all >> 4), descriptor version 1, 128-byte swizzle.
__device__ __forceinline__ uint64_t SmemDescSw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // version
  d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor of kind::i8 with signed int8 A and B, int32 D,
// M = 128; A stored M-contiguous (MN-major), B K-major. n: the MMA N (16..256, % 16).
__host__ __device__ constexpr uint32_t InstrDescS8(uint32_t n) {
  return (2u << 4)                 // D format: s32
         | (1u << 7)               // A format: signed 8-bit
         | (1u << 10)              // B format: signed 8-bit
         | (1u << 15)              // A major: MN
         | (0u << 16)              // B major: K
         | ((n >> 3) << 17)        // N >> 3
         | ((128u >> 4) << 24);    // M >> 4
}

// D[tmem] (+)= A[smem] x B[smem] in exact int32 arithmetic, issued by one thread.
__device__ __forceinline__ void MmaS8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                      uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once every tensor-core operation this thread issued so far
// has completed.
__device__ __forceinline__ void MmaCommit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
               : "memory");
}

// 16 consecutive 32-bit columns of this thread's TMEM lane, raw, without
// waiting: TmemWaitLoads() before the registers are read.
__device__ __forceinline__ void TmemLoad16Raw(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void TmemWaitLoads() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

}  // namespace accel_b200
