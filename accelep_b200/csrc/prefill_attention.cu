// Causal grouped-query attention of a prefill (src/sim_attend.cc:9-46 over the
// prompt rows of many sequences, src/llama_model.cc:233), tiled.
//
// The rows of sequence b are q rows first[b] .. first[b] + count[b] - 1 at
// positions pos0[b] + i; each attends to cache rows [0, pos0[b] + i] of slot b
// (already roped and appended). The cache is head-major with rows of 64 floats
// (element (slot s, kv head g, row t, dim d) at s * seq_stride + g *
// head_stride + t * 64 + d).
//
// One CTA takes 32 query rows of one sequence and the G query heads that share
// one kv head (32 * G query vectors), and walks the 64-row key/value tiles up
// to its last row's position. Per tile: key and value rows stream into shared
// memory with cp.async (rows padded to 68 floats so 16-byte loads along a row
// hit distinct banks); scores Q.K^T are register-blocked (each thread 2G
// vectors x 4 keys, each score one fp32 fused multiply-add chain over the 64
// dimensions in order), masked causally and scaled; an online softmax
// (running max and sum per vector) rescales the weighted-value accumulators;
// P.V is register-blocked the same way (2G vectors x 4 dimensions). The sum
// divides the accumulated values once at the end (the reference divides each
// weight first; the two orders agree well inside 1e-4).
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <mutex>
#include <string>

#include "accel_b200.h"
#include "common.cuh"

namespace accel_b200 {
namespace {

constexpr int kQT = 32;       // query rows per CTA
constexpr int kKT = 64;       // key rows per tile
constexpr int kD = 64;        // head_dim
constexpr int kLd = kD + 4;   // padded shared-memory row (floats)
constexpr int kThreads = 256; // 16 x 16 thread grid

template <int G>
struct PL {
  static constexpr int kV = kQT * G;     // query vectors: v = row * G + head
  static constexpr int kVpt = kV / 16;   // vectors per thread row
  static constexpr int kPLd = kV + 4;    // P row stride: [key][vector]
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kV * kLd;
  static constexpr int kVOff = kKOff + kKT * kLd;
  static constexpr int kPOff = kVOff + kKT * kLd;
  static constexpr int kFloats = kPOff + kKT * kPLd;
  static constexpr int kBytes = kFloats * 4;
};

struct PrefillArgs {
  const float* q;
  int64_t q_stride;
  const float* k_cache;
  const float* v_cache;
  int64_t seq_stride;
  int64_t head_stride;
  float* out;
  int64_t out_stride;
  const int32_t* first;
  const int32_t* count;
  const int32_t* pos0;
  int32_t heads;
  int32_t kv_heads;
  float scale;
};

__device__ __forceinline__ void CpAsync16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void CpAsyncWaitAll() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

template <int G>
__global__ void __launch_bounds__(kThreads, 2) AttnPrefillKernel(PrefillArgs a) {
  using L = PL<G>;
  constexpr int V = L::kV, VPT = L::kVpt;
  extern __shared__ __align__(16) float sm[];
  float* qs = sm + L::kQOff;
  float* ks = sm + L::kKOff;
  float* vs = sm + L::kVOff;
  float* ps = sm + L::kPOff;
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;  // lane = tx + 16 * (ty & 1): a row of 16 tx is a half warp
  const int b = blockIdx.z, g = blockIdx.y;
  const int count = a.count[b];
  const int n_tiles = (count + kQT - 1) / kQT;
  // Longest tiles (latest rows) first.
  const int qt = n_tiles - 1 - static_cast<int>(blockIdx.x);
  if (qt < 0) return;
  const int r0 = qt * kQT;
  const int rows = min(kQT, count - r0);
  const int64_t p0 = a.pos0[b];
  const int64_t last_pos = p0 + r0 + rows - 1;
  const int64_t first_row = a.first[b] + r0;
  const float* kbase = a.k_cache + b * a.seq_stride + g * a.head_stride;
  const float* vbase = a.v_cache + b * a.seq_stride + g * a.head_stride;

  // Query vectors (zero rows past the sequence).
  for (int idx = tid; idx < V * (kD / 4); idx += kThreads) {
    const int v = idx / (kD / 4), d4 = idx % (kD / 4);
    const int row = v / G, hh = v % G;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (row < rows) {
      x = *reinterpret_cast<const float4*>(a.q + (first_row + row) * a.q_stride +
                                           static_cast<int64_t>(g * G + hh) * kD + d4 * 4);
    }
    *reinterpret_cast<float4*>(qs + v * kLd + d4 * 4) = x;
  }

  float o[VPT][4], m[VPT], l[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) o[i][c] = 0.f;
  }
  const int n_kt = static_cast<int>(last_pos / kKT) + 1;
  for (int kt = 0; kt < n_kt; ++kt) {
    const int64_t t0 = static_cast<int64_t>(kt) * kKT;
    // Key and value rows t0 .. t0 + 63; rows past last_pos are zero.
    for (int idx = tid; idx < kKT * (kD / 4); idx += kThreads) {
      const int j = idx / (kD / 4), d4 = idx % (kD / 4);
      float* kd = ks + j * kLd + d4 * 4;
      float* vd = vs + j * kLd + d4 * 4;
      if (t0 + j <= last_pos) {
        CpAsync16(kd, kbase + (t0 + j) * kD + d4 * 4);
        CpAsync16(vd, vbase + (t0 + j) * kD + d4 * 4);
      } else {
        *reinterpret_cast<float4*>(kd) = make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(vd) = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    CpAsyncWaitAll();
    __syncthreads();

    // Scores of vectors ty * VPT + i against keys tx + 16 * j.
    float s[VPT][4];
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
#pragma unroll 1
    for (int d4 = 0; d4 < kD / 4; ++d4) {
      float4 kv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) kv[j] = *reinterpret_cast<const float4*>(ks + (tx + 16 * j) * kLd + d4 * 4);
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const float4 qv = *reinterpret_cast<const float4*>(qs + (ty * VPT + i) * kLd + d4 * 4);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          s[i][j] = fmaf(qv.x, kv[j].x, s[i][j]);
          s[i][j] = fmaf(qv.y, kv[j].y, s[i][j]);
          s[i][j] = fmaf(qv.z, kv[j].z, s[i][j]);
          s[i][j] = fmaf(qv.w, kv[j].w, s[i][j]);
        }
      }
    }
    // Mask, online softmax, weights to shared memory.
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int v = ty * VPT + i;
      const int64_t pos = p0 + r0 + v / G;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t t = t0 + tx + 16 * j;
        s[i][j] = t <= pos ? s[i][j] * a.scale : -INFINITY;
        mx = fmaxf(mx, s[i][j]);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, off));
      const float m_new = fmaxf(m[i], mx);  // finite: key 0 is visible to every row
      const float corr = expf(m[i] - m_new);
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = expf(s[i][j] - m_new);
        ps[(tx + 16 * j) * L::kPLd + v] = p;
        sum += p;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) sum += __shfl_xor_sync(kFull, sum, off);
      l[i] = l[i] * corr + sum;
      m[i] = m_new;
#pragma unroll
      for (int c = 0; c < 4; ++c) o[i][c] *= corr;
    }
    __syncthreads();
    // Weighted values: vectors ty * VPT + i, dimensions tx * 4 .. + 3.
#pragma unroll 4
    for (int j = 0; j < kKT; ++j) {
      const float4 vv = *reinterpret_cast<const float4*>(vs + j * kLd + tx * 4);
      const float* pj = ps + j * L::kPLd + ty * VPT;
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const float p = pj[i];
        o[i][0] = fmaf(p, vv.x, o[i][0]);
        o[i][1] = fmaf(p, vv.y, o[i][1]);
        o[i][2] = fmaf(p, vv.z, o[i][2]);
        o[i][3] = fmaf(p, vv.w, o[i][3]);
      }
    }
    __syncthreads();  // the tiles and weights are rewritten next
  }
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = ty * VPT + i;
    const int row = v / G, hh = v % G;
    if (row < rows) {
      float* dst = a.out + (first_row + row) * a.out_stride + static_cast<int64_t>(g * G + hh) * kD + tx * 4;
      *reinterpret_cast<float4*>(dst) = make_float4(o[i][0] / l[i], o[i][1] / l[i], o[i][2] / l[i], o[i][3] / l[i]);
    }
  }
}

template <int G>
int LaunchPrefill(const PrefillArgs& a, int32_t batch, int32_t max_rows, cudaStream_t stream) {
  static std::once_flag once[16];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 15], [] {
    cudaFuncSetAttribute(AttnPrefillKernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, PL<G>::kBytes);
  });
  const dim3 grid(static_cast<unsigned>((max_rows + kQT - 1) / kQT), static_cast<unsigned>(a.kv_heads),
                  static_cast<unsigned>(batch));
  AttnPrefillKernel<G><<<grid, kThreads, PL<G>::kBytes, stream>>>(a);
  return CheckLaunch("attention_prefill");
}

}  // namespace
}  // namespace accel_b200

using namespace accel_b200;

extern "C" {

ACCEL_B200_API int accel_b200_attention_prefill(const float* q, int64_t q_stride, const float* k_cache,
                                                const float* v_cache, int64_t seq_stride, int64_t head_stride,
                                                float* out, int64_t out_stride, const int32_t* first,
                                                const int32_t* count, const int32_t* pos0, int32_t batch,
                                                int32_t max_rows, int32_t heads, int32_t kv_heads, int32_t head_dim,
                                                void* stream) {
  if (batch < 0 || max_rows < 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads != 0 || head_dim != kD ||
      q == nullptr || k_cache == nullptr || v_cache == nullptr || out == nullptr || first == nullptr ||
      count == nullptr || pos0 == nullptr) {
    return SetError(ACCEL_B200_EINVAL, "attention_prefill: bad arguments (head_dim must be 64)");
  }
  if (batch == 0 || max_rows == 0) return ClearError();
  const int group = heads / kv_heads;
  if (group > 4) return SetError(ACCEL_B200_EINVAL, "attention_prefill: more than 4 query heads per kv head");
  if (batch > 65535 || kv_heads > 65535) return SetError(ACCEL_B200_EINVAL, "attention_prefill: grid too large");
  if (q_stride % 4 != 0 || out_stride % 4 != 0 || seq_stride % 4 != 0 || head_stride % 4 != 0 ||
      (reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(k_cache) |
       reinterpret_cast<uintptr_t>(v_cache)) % 16 != 0) {
    return SetError(ACCEL_B200_EINVAL, "attention_prefill: rows must be 16-byte aligned");
  }
  PrefillArgs a{q, q_stride, k_cache, v_cache, seq_stride, head_stride, out, out_stride, first, count, pos0,
                heads, kv_heads, 1.f / sqrtf(static_cast<float>(kD))};
  cudaStream_t s = AsStream(stream);
  switch (group) {
    case 1: return LaunchPrefill<1>(a, batch, max_rows, s);
    case 2: return LaunchPrefill<2>(a, batch, max_rows, s);
    case 3: return LaunchPrefill<3>(a, batch, max_rows, s);
    default: return LaunchPrefill<4>(a, batch, max_rows, s);
  }
}

}  // extern "C"
