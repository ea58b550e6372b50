// Thread-block cluster helpers in inline PTX for sm_100a: the cluster-wide
// barrier and loads from a peer CTA's shared memory (distributed shared
// memory). The CTAs of a cluster are scheduled together, so a barrier that
// every CTA of the cluster reaches always completes.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "tma.cuh"

namespace accel_b200 {

// Every thread of every CTA of the cluster arrives (release) and waits
// (acquire): shared-memory writes before it are visible to the peers after it.
__device__ __forceinline__ void ClusterSync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t ClusterRank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// The same shared-memory offset in cluster CTA `rank`.
__device__ __forceinline__ uint32_t PeerAddr(const void* local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(SmemAddr(local)), "r"(rank));
  return remote;
}

__device__ __forceinline__ float4 LoadPeer4(const float* local, uint32_t rank) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(PeerAddr(local, rank))
               : "memory");
  return v;
}

__device__ __forceinline__ float LoadPeer(const float* local, uint32_t rank) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(PeerAddr(local, rank)) : "memory");
  return v;
}

__device__ __forceinline__ int32_t LoadPeerInt(const int32_t* local, uint32_t rank) {
  int32_t v;
  asm volatile("ld.shared::cluster.b32 %0, [%1];" : "=r"(v) : "r"(PeerAddr(local, rank)) : "memory");
  return v;
}

}  // namespace accel_b200
