// Shared device helpers and the launch/status plumbing of the kernel ABI.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <string>
#include <utility>

#include "accel_b200.h"
#include "status.h"

namespace accel_b200 {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kSms = 148;  // B200: 2 dies x 74 SMs

// ---------------------------------------------------------------- host side

inline cudaStream_t AsStream(void* s) { return static_cast<cudaStream_t>(s); }

inline int64_t CeilDiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Product workspaces start with a fixed region of arrival counters that the
// kernels leave zero; split-K partial sums follow it. The fixed offset keeps
// the counters of every call on the same zeroed bytes whatever the shape.
constexpr size_t kCounterRegion = 64 * 1024;
constexpr int64_t kMaxCounters = static_cast<int64_t>(kCounterRegion / sizeof(int32_t));

__host__ __device__ __forceinline__ int64_t Min64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t Max64(int64_t a, int64_t b) { return a > b ? a : b; }

// Programmatic dependent launch: kernels launched through LaunchK may start
// while the previous kernel on the stream is still running. Each such kernel
// calls PdlWait before it touches memory that an earlier kernel writes (and
// before any global write of its own); only immutable inputs (weights,
// scales, tables) are read before it. PdlTrigger lets the next kernel start.
// Off when the environment sets ACCEL_B200_PDL=0.
bool PdlEnabled();

// Launches `kernel` with an optional thread-block cluster (cx, cy, 1) and, when
// enabled, programmatic stream serialization.
template <typename... KArgs, typename... Args>
cudaError_t LaunchK(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, unsigned cx,
                    unsigned cy, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (cx * cy > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cx;
    attr[n].val.clusterDim.y = cy;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (PdlEnabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------- device side

__device__ __forceinline__ void PdlWait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void PdlTrigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float WarpSum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

__device__ __forceinline__ double WarpSum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

__device__ __forceinline__ float WarpMax(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
  return v;
}

// Exact Gelu of the reference (sim_device.cc:239): 0.5 * x * (1 + erf(x / sqrt 2)),
// every step a rounded float operation. Not inlined: the epilogues that can
// apply it are unrolled many times over, and most products never take it
// (the smaller kernels keep more of their instructions in cache).
static __device__ __noinline__ float GeluExact(float v) {
  const float e = erff(__fmul_rn(v, 0.7071067811865476f));
  return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.f, e));
}

// Output copies on other GPUs: the same element is also stored to each peer
// buffer at the same offset (peer memory mapped into this process, written
// over NVLink). Used to fuse an all-gather into a product's epilogue.
constexpr int kMaxPeers = 7;
struct PeerOut {
  float* c[kMaxPeers];
  int32_t n;
};

// Element `offset` (from the output's base) to every peer copy.
__device__ __forceinline__ void StorePeers(const PeerOut& peers, int64_t offset, float v) {
  for (int i = 0; i < peers.n; ++i) peers.c[i][offset] = v;
}

__device__ __forceinline__ void StorePeers4(const PeerOut& peers, int64_t offset, float4 v) {
  for (int i = 0; i < peers.n; ++i) *reinterpret_cast<float4*>(peers.c[i] + offset) = v;
}

// Epilogue of a product (include/accel_b200.h, accel_b200_epilogue), applied to
// one output element: act(alpha * acc + beta * bias) + residual, each step a
// rounded float operation as in sim_device.cc:227-241 and runtime.cc:336-344.
struct Epilogue {
  float alpha = 1.f;
  float beta = 0.f;
  const float* bias = nullptr;
  int64_t bias_rs = 0;
  int64_t bias_cs = 0;
  int32_t act = 0;
  const float* residual = nullptr;
  int64_t residual_ld = 0;
  double* row_sq = nullptr;  // per row and 128-column block: sum of squares of the outputs
  int64_t row_sq_ld = 0;
  int32_t flags = 0;  // ACCEL_B200_EP_TRIGGER_AFTER_WAIT
};

__device__ __forceinline__ float ApplyEpilogue(const Epilogue& ep, float acc, int64_t i, int64_t j) {
  float v = __fmul_rn(ep.alpha, acc);
  if (ep.bias != nullptr) v = __fadd_rn(v, __fmul_rn(ep.beta, ep.bias[i * ep.bias_rs + j * ep.bias_cs]));
  if (ep.act == ACCEL_B200_ACT_RELU) {
    if (v < 0.f) v = 0.f;
  } else if (ep.act == ACCEL_B200_ACT_GELU) {
    v = GeluExact(v);
  }
  if (ep.residual != nullptr) v = __fadd_rn(v, ep.residual[i * ep.residual_ld + j]);
  return v;
}

// Rotate-half RoPE of one pair (src/sim_rope.cc:16-17): x[i] and x[half + i] of a
// head with the position's cos/sin rows `c`, `s` (head_dim entries each):
//   lo = x[i] * c[i] - x[half + i] * s[i]
//   hi = x[half + i] * c[half + i] + x[i] * s[half + i]
// every step a rounded float operation, as the reference evaluates it.
__device__ __forceinline__ void RopePair(float a, float b, const float* c, const float* s, int i, int half, float* lo,
                                         float* hi) {
  *lo = __fsub_rn(__fmul_rn(a, c[i]), __fmul_rn(b, s[i]));
  *hi = __fadd_rn(__fmul_rn(b, c[half + i]), __fmul_rn(a, s[half + i]));
}

}  // namespace accel_b200
