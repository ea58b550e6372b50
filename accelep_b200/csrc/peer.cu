// Rank barrier over peer memory for the fused product + all-gather of the
// N-sharded C5 product: after each rank's product kernel has stored its
// output block into every rank's Y, each rank signals every peer and waits for
// every peer's signal. Flags live in symmetric memory (one int32 per rank on
// every GPU, mapped into every process); rank r writes the next epoch into
// slot r of each peer's array with a system-scope release store and polls its
// own array with system-scope acquire loads. The epoch is a device counter
// that the kernel advances, so the same launch replays correctly from a CUDA
// graph; epochs only grow, so the flags need no reset. The wait is bounded:
// a peer that never signals sets ACCEL_B200_STATUS_COPY_TIMEOUT in *status and
// the kernel returns.
#include <cuda_runtime.h>
#include <stdint.h>

#include "accel_b200.h"
#include "common.cuh"
#include "tma.cuh"

namespace accel_b200 {
namespace {

constexpr int kMaxRanks = 8;

struct PeerFlags {
  int32_t* f[kMaxRanks];  // base of rank p's flag array (world int32)
};

__global__ void PeerBarrierKernel(PeerFlags peers, int32_t* mine, int32_t rank, int32_t world, int32_t* counter,
                                  long long limit_cycles, int32_t* status) {
  __shared__ int32_t epoch_s;
  const int p = threadIdx.x;
  if (p == 0) epoch_s = *counter + 1;
  __syncthreads();
  const int32_t epoch = epoch_s;
  if (p < world && p != rank) {
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(peers.f[p] + rank), "r"(epoch) : "memory");
    const long long start = clock64();
    for (;;) {
      int32_t v;
      asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(mine + p) : "memory");
      if (v - epoch >= 0) break;
      if (clock64() - start > limit_cycles) {
        if (status != nullptr) atomicOr(status, ACCEL_B200_STATUS_COPY_TIMEOUT);
        break;
      }
      __nanosleep(64);
    }
  }
  if (p == 0) *counter = epoch;
}

}  // namespace
}  // namespace accel_b200

using namespace accel_b200;

extern "C" {

ACCEL_B200_API int accel_b200_peer_barrier(int32_t* const* peer_flags, int32_t* my_flags, int32_t rank, int32_t world,
                                           int32_t* epoch_counter, int64_t limit_cycles, int32_t* status,
                                           void* stream) {
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world || my_flags == nullptr || peer_flags == nullptr ||
      epoch_counter == nullptr) {
    return SetError(ACCEL_B200_EINVAL, "peer_barrier: bad arguments (1..8 ranks, an epoch counter)");
  }
  PeerFlags p{};
  for (int i = 0; i < world; ++i) {
    if (i != rank && peer_flags[i] == nullptr) return SetError(ACCEL_B200_EINVAL, "peer_barrier: null peer flags");
    p.f[i] = peer_flags[i];
  }
  const long long limit = limit_cycles > 0 ? limit_cycles : kWaitLimitCycles;
  PeerBarrierKernel<<<1, 32, 0, AsStream(stream)>>>(p, my_flags, rank, world, epoch_counter, limit, status);
  return CheckLaunch("peer_barrier");
}

}  // extern "C"
