// Causal grouped-query attention (src/sim_attend.cc:9-46) on the device.
//
// Two kernels:
//  * AttnRowsKernel: one CTA per (query row, head), an online softmax over
//    chunks of the context. Any head_dim up to 1024, any context length.
//    It serves Device::Attention and prefill, where many query rows share
//    each key row and the key rows stay in L2.
//  * AttnDecodeKernel: split-KV ("flash decoding") for one new query row per
//    sequence with head_dim 64. One CTA per (sequence, kv head, context
//    chunk) bulk-copies the chunk's key and value rows into shared memory
//    once for all query heads that share the kv head, writes a partial
//    (max, sum, weighted values), and the last CTA of the (sequence, kv head)
//    merges the partials with the log-sum-exp rule.
//
// The reference divides each weight by the sum before the value product;
// here the sum divides the accumulated product once. The two orders agree
// well inside the 1e-4 tolerance.
#include <cuda.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <mutex>

#include "accel_b200.h"
#include "common.cuh"
#include "tma.cuh"

namespace accel_b200 {
namespace {

constexpr int kRowsThreads = 128;
constexpr int kRowsChunk = 512;
constexpr int kMaxDPerThread = 8;  // head_dim <= 8 * 128

struct RowsArgs {
  const float* q;
  int64_t q_row_stride;
  const float* k;
  const float* v;
  int64_t kv_row_stride;
  int64_t kv_head_stride;
  int64_t kv_seq_stride;
  float* out;
  int64_t out_row_stride;
  const int32_t* row_seq;  // null: every row belongs to sequence 0
  const int32_t* row_pos;  // null: row r sits at position + r
  int64_t position;
  int32_t heads;
  int32_t kv_heads;
  int32_t head_dim;
  float scale;
};

__device__ float BlockReduceMax(float v, float* red) {
  v = WarpMax(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
  for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) r = fmaxf(r, red[w]);
  return r;
}

__device__ float BlockReduceSum(float v, float* red) {
  v = WarpSum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = 0.f;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) r += red[w];
  return r;
}

__global__ void __launch_bounds__(kRowsThreads) AttnRowsKernel(RowsArgs a) {
  extern __shared__ float smem[];
  float* q_s = smem;                  // head_dim
  float* p_s = smem + a.head_dim;     // kRowsChunk
  __shared__ float red[kRowsThreads / 32];
  const int64_t r = blockIdx.x;
  const int h = blockIdx.y;
  const int D = a.head_dim;
  const int g = h / (a.heads / a.kv_heads);
  const int64_t seq = a.row_seq != nullptr ? a.row_seq[r] : 0;
  const int64_t limit = a.row_pos != nullptr ? a.row_pos[r] : a.position + r;
  const float* qrow = a.q + r * a.q_row_stride + static_cast<int64_t>(h) * D;
  const float* kbase = a.k + seq * a.kv_seq_stride + static_cast<int64_t>(g) * a.kv_head_stride;
  const float* vbase = a.v + seq * a.kv_seq_stride + static_cast<int64_t>(g) * a.kv_head_stride;
  for (int d = threadIdx.x; d < D; d += blockDim.x) q_s[d] = qrow[d];
  float acc[kMaxDPerThread];
#pragma unroll
  for (int i = 0; i < kMaxDPerThread; ++i) acc[i] = 0.f;
  float m = -INFINITY, l = 0.f;
  __syncthreads();
  for (int64_t c0 = 0; c0 <= limit; c0 += kRowsChunk) {
    const int cnt = static_cast<int>(Min64(kRowsChunk, limit + 1 - c0));
    float cmax = -INFINITY;
    for (int j = threadIdx.x; j < cnt; j += blockDim.x) {
      const float* kr = kbase + (c0 + j) * a.kv_row_stride;
      float dot = 0.f;
      for (int d = 0; d < D; ++d) dot = fmaf(q_s[d], kr[d], dot);
      const float s = dot * a.scale;
      p_s[j] = s;
      cmax = fmaxf(cmax, s);
    }
    cmax = BlockReduceMax(cmax, red);
    const float m_new = fmaxf(m, cmax);
    const float corr = (m == -INFINITY) ? 0.f : expf(m - m_new);
    float lsum = 0.f;
    for (int j = threadIdx.x; j < cnt; j += blockDim.x) {
      const float p = expf(p_s[j] - m_new);
      p_s[j] = p;
      lsum += p;
    }
    lsum = BlockReduceSum(lsum, red);  // also orders the p_s writes before the reads below
    l = l * corr + lsum;
#pragma unroll
    for (int i = 0; i < kMaxDPerThread; ++i) {
      const int d = threadIdx.x + i * kRowsThreads;
      if (d < D) {
        float s = acc[i] * corr;
        const float* vcol = vbase + c0 * a.kv_row_stride + d;
        for (int j = 0; j < cnt; ++j) s = fmaf(p_s[j], vcol[j * a.kv_row_stride], s);
        acc[i] = s;
      }
    }
    m = m_new;
    __syncthreads();
  }
  float* orow = a.out + r * a.out_row_stride + static_cast<int64_t>(h) * D;
#pragma unroll
  for (int i = 0; i < kMaxDPerThread; ++i) {
    const int d = threadIdx.x + i * kRowsThreads;
    if (d < D) orow[d] = acc[i] / l;
  }
}

// ----------------------------------------------------------- split-KV decode

constexpr int kDecD = 64;
constexpr int kDecThreads = 128;
constexpr int kMaxGroup = 8;
constexpr int kPart = kDecD + 2;  // weighted values, max, sum

struct DecodeArgs {
  const float* q;  // row b: heads * 64 floats at q + b * q_row_stride
  int64_t q_row_stride;
  const float* k;  // slot b, kv head g, row t: k + b * seq + g * head + t * row (floats)
  const float* v;
  int64_t kv_row_stride;
  int64_t kv_head_stride;
  int64_t kv_seq_stride;
  const int32_t* lens;  // context length of sequence b (new row included)
  int32_t heads;
  int32_t kv_heads;
  int32_t chunk;     // context rows per CTA
  int32_t n_chunks;  // grid.x
  float scale;
  float* part;        // [B][heads][n_chunks][kPart]
  int32_t* counters;  // [B][kv_heads]: arrivals; zero before and after a launch
  int32_t* status;    // ORs ACCEL_B200_STATUS_COPY_TIMEOUT; may be null
  float* out;
  int64_t out_row_stride;
};

// One CTA per (chunk, kv head, sequence). The chunk's key and value rows are
// pulled into shared memory by bulk copies (one copy per operand when rows
// are contiguous, else one per row), the G query heads of the kv head score
// them, and a partial (max, sum, weighted values) per head goes to the
// workspace. The last CTA of a (sequence, kv head) to arrive merges the
// partials in chunk order, so the result does not depend on arrival order.
template <int G>
__global__ void __launch_bounds__(kDecThreads) AttnDecodeKernel(DecodeArgs a) {
  extern __shared__ __align__(128) float smem[];
  const int C = a.chunk;
  float* ks = smem;               // C * 64
  float* vs = ks + C * kDecD;     // C * 64
  float* qs = vs + C * kDecD;     // G * 64
  float* ps = qs + G * kDecD;     // G * C
  __shared__ __align__(8) uint64_t bar;
  __shared__ float stat[2 * kMaxGroup];
  __shared__ int32_t last;
  const int c = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t len = a.lens[b];
  const int64_t t0 = static_cast<int64_t>(c) * C;
  const int cnt = static_cast<int>(Max64(0, Min64(C, len - t0)));
  const int h0 = g * G;
  const int64_t head_part = static_cast<int64_t>(a.n_chunks) * kPart;
  float* part_base = a.part + ((static_cast<int64_t>(b) * a.heads + h0) * a.n_chunks + c) * kPart;

  if (cnt > 0) {
    const float* kb = a.k + b * a.kv_seq_stride + g * a.kv_head_stride + t0 * a.kv_row_stride;
    const float* vb = a.v + b * a.kv_seq_stride + g * a.kv_head_stride + t0 * a.kv_row_stride;
    const bool contiguous = a.kv_row_stride == kDecD;
    if (tid == 0) {
      MbarInit(&bar, 1);
      FenceBarrierInit();
    }
    __syncthreads();
    if (tid == 0) {
      MbarArriveExpectTx(&bar, static_cast<uint32_t>(cnt) * kDecD * 4 * 2);
      if (contiguous) {
        BulkCopyG2S(ks, kb, static_cast<uint32_t>(cnt) * kDecD * 4, &bar);
        BulkCopyG2S(vs, vb, static_cast<uint32_t>(cnt) * kDecD * 4, &bar);
      }
    }
    __syncthreads();  // the expected byte count is posted before row copies land
    if (!contiguous) {
      for (int j = tid; j < cnt; j += kDecThreads) {
        BulkCopyG2S(ks + j * kDecD, kb + j * a.kv_row_stride, kDecD * 4, &bar);
        BulkCopyG2S(vs + j * kDecD, vb + j * a.kv_row_stride, kDecD * 4, &bar);
      }
    }
    const float* qrow = a.q + static_cast<int64_t>(b) * a.q_row_stride + static_cast<int64_t>(h0) * kDecD;
    for (int i = tid; i < G * kDecD; i += kDecThreads) qs[i] = qrow[i];
    __syncthreads();
    bool ok = MbarWait(&bar, 0);
    if (!ok) {
      if (a.status != nullptr) atomicOr(a.status, ACCEL_B200_STATUS_COPY_TIMEOUT);
      MbarWait(&bar, 0);  // give copies still in flight one more bounded wait
    }
    ok = __syncthreads_and(ok);
    if (ok) {
      // Scores: two threads per row, each over half of the dimensions; the
      // float4 index rotates with the row so a quarter-warp hits 32 banks.
      for (int base = 0; base < 2 * cnt; base += kDecThreads) {
        const int task = base + tid;
        const bool valid = task < 2 * cnt;  // uniform loop: every lane reaches the shuffle
        const int j = valid ? task >> 1 : 0, half = task & 1;
        float dot[G];
#pragma unroll
        for (int hh = 0; hh < G; ++hh) dot[hh] = 0.f;
        if (valid) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int d4 = half * 8 + ((i + j + 4 * half) & 7);
            const float4 kv = *reinterpret_cast<const float4*>(ks + j * kDecD + d4 * 4);
#pragma unroll
            for (int hh = 0; hh < G; ++hh) {
              const float4 qv = *reinterpret_cast<const float4*>(qs + hh * kDecD + d4 * 4);
              dot[hh] = fmaf(qv.x, kv.x, dot[hh]);
              dot[hh] = fmaf(qv.y, kv.y, dot[hh]);
              dot[hh] = fmaf(qv.z, kv.z, dot[hh]);
              dot[hh] = fmaf(qv.w, kv.w, dot[hh]);
            }
          }
        }
#pragma unroll
        for (int hh = 0; hh < G; ++hh) {
          const float other = __shfl_xor_sync(kFull, dot[hh], 1);
          if (valid && half == 0) ps[hh * C + j] = (dot[hh] + other) * a.scale;
        }
      }
      __syncthreads();
      for (int hh = warp; hh < G; hh += kDecThreads / 32) {
        float mx = -INFINITY;
        for (int j = lane; j < cnt; j += 32) mx = fmaxf(mx, ps[hh * C + j]);
        mx = WarpMax(mx);
        float sum = 0.f;
        for (int j = lane; j < cnt; j += 32) {
          const float p = expf(ps[hh * C + j] - mx);
          ps[hh * C + j] = p;
          sum += p;
        }
        sum = WarpSum(sum);
        if (lane == 0) {
          stat[2 * hh] = mx;
          stat[2 * hh + 1] = sum;
        }
      }
      __syncthreads();
      // Weighted values: thread owns dimension d for heads tid / 64, + 2, ...
      const int d = tid & (kDecD - 1);
      for (int hh = tid / kDecD; hh < G; hh += kDecThreads / kDecD) {
        float acc = 0.f;
        const float* p = ps + hh * C;
        for (int j = 0; j < cnt; ++j) acc = fmaf(p[j], vs[j * kDecD + d], acc);
        part_base[hh * head_part + d] = acc;
      }
      if (tid < G) {
        part_base[tid * head_part + kDecD] = stat[2 * tid];
        part_base[tid * head_part + kDecD + 1] = stat[2 * tid + 1];
      }
    } else if (tid < G) {
      part_base[tid * head_part + kDecD] = -INFINITY;
      part_base[tid * head_part + kDecD + 1] = 0.f;
    }
  }
  // Arrive; the last CTA of this (sequence, kv head) merges.
  __threadfence();
  __syncthreads();
  int32_t* counter = a.counters + static_cast<int64_t>(b) * a.kv_heads + g;
  if (tid == 0) last = atomicAdd(counter, 1) == static_cast<int32_t>(gridDim.x) - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  const int used = static_cast<int>((len + C - 1) / C);
  const float* pb = a.part + (static_cast<int64_t>(b) * a.heads + h0) * head_part;
  for (int task = tid; task < G * kDecD; task += kDecThreads) {
    const int hh = task / kDecD, d = task % kDecD;
    const float* ph = pb + hh * head_part;
    float mx = -INFINITY;
    for (int cc = 0; cc < used; ++cc) mx = fmaxf(mx, __ldcg(ph + cc * kPart + kDecD));
    float l = 0.f, o = 0.f;
    for (int cc = 0; cc < used; ++cc) {
      const float w = expf(__ldcg(ph + cc * kPart + kDecD) - mx);
      l = fmaf(__ldcg(ph + cc * kPart + kDecD + 1), w, l);
      o = fmaf(__ldcg(ph + cc * kPart + d), w, o);
    }
    a.out[static_cast<int64_t>(b) * a.out_row_stride + static_cast<int64_t>(h0 + hh) * kDecD + d] = o / l;
  }
  if (tid == 0) *counter = 0;
}

int LaunchRows(const RowsArgs& a, int64_t rows, cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(a.head_dim + kRowsChunk) * sizeof(float);
  if (rows > 2147483647LL || a.heads > 65535) return SetError(ACCEL_B200_EINVAL, "attention: grid too large");
  AttnRowsKernel<<<dim3(static_cast<unsigned>(rows), static_cast<unsigned>(a.heads)), kRowsThreads, smem, stream>>>(a);
  return CheckLaunch("attention_rows");
}

template <int G>
int LaunchDecode(const DecodeArgs& a, int32_t batch, cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(2 * a.chunk * kDecD + G * kDecD + G * a.chunk) * sizeof(float);
  if (smem > 48 * 1024) {
    cudaFuncSetAttribute(AttnDecodeKernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  }
  AttnDecodeKernel<G><<<dim3(a.n_chunks, a.kv_heads, batch), kDecThreads, smem, stream>>>(a);
  return CheckLaunch("attention_decode");
}

// Posts an expected byte count that no copy will ever deliver, so the
// bounded wait runs out: the status word must then carry the timeout bit and
// the context must stay usable. Used by the failure-detection test.
__global__ void WaitSelftestKernel(int32_t* status) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    MbarInit(&bar, 1);
    FenceBarrierInit();
  }
  __syncthreads();
  if (threadIdx.x == 0) MbarArriveExpectTx(&bar, 16);
  __syncthreads();
  const bool ok = MbarWait(&bar, 0);
  if (!ok && threadIdx.x == 0) atomicOr(status, ACCEL_B200_STATUS_COPY_TIMEOUT);
}

}  // namespace

// ------------------------------------------- decode attention without allocation
//
// Scratch of accel_b200_attention_decode_noalloc: a fixed array in the
// library's own device memory, so that callers who may not allocate still
// have a place for the split partials and arrival counters. Every GPU that
// loads this library holds these 4 MiB until the process exits.
constexpr size_t kNoAllocScratchBytes = static_cast<size_t>(4) << 20;
static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
struct ScratchSlot {
  unsigned long long context_id = 0;  // the CUDA context the address belongs to
  void* address = nullptr;
};
ScratchSlot g_scratch[kMaxDevices];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// The unique id of the current CUDA context (the driver's cuCtxGetId, reached
// through the runtime's entry-point query, so the library needs no libcuda at
// link time). A device reset ends the context; the next one has another id.
int CurrentContextId(unsigned long long* id) {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  if (get_current == nullptr || get_id == nullptr) {
    void* f1 = nullptr;
    void* f2 = nullptr;
    cudaDriverEntryPointQueryResult q1{}, q2{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f1, cudaEnableDefault, &q1) != cudaSuccess ||
        cudaGetDriverEntryPoint("cuCtxGetId", &f2, cudaEnableDefault, &q2) != cudaSuccess || f1 == nullptr ||
        f2 == nullptr) {
      cudaGetLastError();
      return SetError(ACCEL_B200_ECUDA, "noalloc scratch: the driver does not offer cuCtxGetId");
    }
    get_current = reinterpret_cast<CtxGetCurrentFn>(f1);
    get_id = reinterpret_cast<CtxGetIdFn>(f2);
  }
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr || get_id(ctx, id) != CUDA_SUCCESS) {
    return SetError(ACCEL_B200_ECUDA, "noalloc scratch: no current CUDA context");
  }
  return ACCEL_B200_OK;
}

// The device address of the scratch array on the current device. In host code
// g_decode_scratch names a host-side stand-in, not device memory: a kernel
// given that name would fault or read the wrong memory, so the address is
// looked up with cudaGetSymbolAddress once per device (and again after a
// device reset, which gives the device a new context) and cached.
int ScratchAddress(void** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return SetError(ACCEL_B200_ECUDA, std::string("noalloc scratch: ") + cudaGetErrorString(err));
  if (dev < 0 || dev >= kMaxDevices) return SetError(ACCEL_B200_EINVAL, "noalloc scratch: device ordinal above 63");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  ScratchSlot& slot = g_scratch[dev];
  unsigned long long ctx_id = 0;
  if (slot.address != nullptr) {
    // Cheap check that the cached address still belongs to the live context.
    const int rc = CurrentContextId(&ctx_id);
    if (rc != ACCEL_B200_OK) return rc;
    if (ctx_id == slot.context_id) {
      *out = slot.address;
      return ACCEL_B200_OK;
    }
  }
  void* ptr = nullptr;
  err = cudaGetSymbolAddress(&ptr, g_decode_scratch);  // also creates the context on first use
  if (err != cudaSuccess || ptr == nullptr) {
    cudaGetLastError();
    return SetError(ACCEL_B200_ECUDA, std::string("noalloc scratch: cudaGetSymbolAddress failed: ") +
                                          cudaGetErrorString(err));
  }
  const int rc = CurrentContextId(&ctx_id);
  if (rc != ACCEL_B200_OK) return rc;
  slot.address = ptr;
  slot.context_id = ctx_id;
  *out = ptr;
  return ACCEL_B200_OK;
}

// The argument checks of the split-KV decode attention, shared by the
// workspace and the no-allocation entry points, so that both reject a bad
// call before anything is queued on the stream.
int CheckDecodeArgs(const float* q, const float* k, const float* v, int64_t kv_row_stride, int64_t kv_head_stride,
                    int64_t kv_seq_stride, const int32_t* lens, int32_t batch, int32_t heads, int32_t kv_heads,
                    int32_t head_dim, int32_t max_len, int32_t chunk, const float* out) {
  if (batch < 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads != 0 || head_dim != kDecD || max_len <= 0 ||
      chunk <= 0 || chunk > 128 || lens == nullptr || q == nullptr || k == nullptr || v == nullptr || out == nullptr) {
    return SetError(ACCEL_B200_EINVAL, "attention_decode: bad arguments");
  }
  if (heads / kv_heads > kMaxGroup) {
    return SetError(ACCEL_B200_EINVAL, "attention_decode: more than 8 query heads per kv head");
  }
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) % 16 != 0 || kv_row_stride % 4 != 0 ||
      kv_head_stride % 4 != 0 || kv_seq_stride % 4 != 0) {
    return SetError(ACCEL_B200_EINVAL, "attention_decode: cache rows must be 16-byte aligned");
  }
  // One arrival counter per (sequence, kv head) in the workspace's fixed
  // counter region.
  if (static_cast<int64_t>(batch) * kv_heads > kMaxCounters) {
    return SetError(ACCEL_B200_EINVAL, "attention_decode: batch * kv_heads above 16384");
  }
  return ACCEL_B200_OK;
}
}  // namespace
}  // namespace accel_b200

using namespace accel_b200;

extern "C" {

ACCEL_B200_API int accel_b200_attention(const float* q, const float* k, const float* v, float* out, int64_t seq,
                                        int64_t position, int64_t heads, int64_t kv_heads, int64_t head_dim,
                                        void* stream) {
  if (kv_heads <= 0 || (heads > 0 && heads % kv_heads != 0)) {
    return SetError(ACCEL_B200_EINVAL, "Attention kv heads are out of range");
  }
  if (seq < 0 || position < 0 || heads < 0 || head_dim < 0) return SetError(ACCEL_B200_EINVAL, "attention: negative size");
  if (seq == 0 || heads == 0 || head_dim == 0) return ClearError();
  if (head_dim > kMaxDPerThread * kRowsThreads) return SetError(ACCEL_B200_EINVAL, "attention: head_dim above 1024");
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr) return SetError(ACCEL_B200_EINVAL, "attention: null pointer");
  RowsArgs a{};
  a.q = q;
  a.q_row_stride = heads * head_dim;
  a.k = k;
  a.v = v;
  a.kv_row_stride = kv_heads * head_dim;
  a.kv_head_stride = head_dim;
  a.kv_seq_stride = 0;
  a.out = out;
  a.out_row_stride = heads * head_dim;
  a.position = position;
  a.heads = static_cast<int32_t>(heads);
  a.kv_heads = static_cast<int32_t>(kv_heads);
  a.head_dim = static_cast<int32_t>(head_dim);
  a.scale = 1.f / sqrtf(static_cast<float>(head_dim));
  return LaunchRows(a, seq, AsStream(stream));
}

ACCEL_B200_API int accel_b200_attention_rows(const float* q, int64_t q_row_stride, const float* k, const float* v,
                                             int64_t kv_row_stride, int64_t kv_head_stride, int64_t kv_seq_stride,
                                             float* out,
                                             int64_t out_row_stride, const int32_t* row_seq, const int32_t* row_pos,
                                             int64_t rows, int32_t heads, int32_t kv_heads, int32_t head_dim,
                                             void* stream) {
  if (rows < 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads != 0 || head_dim <= 0 ||
      head_dim > kMaxDPerThread * kRowsThreads || row_pos == nullptr) {
    return SetError(ACCEL_B200_EINVAL, "attention_rows: bad arguments");
  }
  if (rows == 0) return ClearError();
  RowsArgs a{q, q_row_stride, k, v, kv_row_stride, kv_head_stride, kv_seq_stride, out, out_row_stride, row_seq, row_pos, 0,
             heads, kv_heads, head_dim, 1.f / sqrtf(static_cast<float>(head_dim))};
  return LaunchRows(a, rows, AsStream(stream));
}

ACCEL_B200_API size_t accel_b200_attention_decode_workspace(int32_t batch, int32_t heads, int32_t kv_heads,
                                                            int32_t max_len, int32_t chunk) {
  if (batch <= 0 || heads <= 0 || kv_heads <= 0 || max_len <= 0 || chunk <= 0) return 0;
  const int64_t chunks = (max_len + chunk - 1) / chunk;
  return kCounterRegion + static_cast<size_t>(batch) * heads * chunks * kPart * sizeof(float);
}

ACCEL_B200_API int accel_b200_attention_decode(const float* q, int64_t q_row_stride, const float* k, const float* v,
                                               int64_t kv_row_stride, int64_t kv_head_stride, int64_t kv_seq_stride,
                                               const int32_t* lens, int32_t batch, int32_t heads, int32_t kv_heads,
                                               int32_t head_dim, int32_t max_len, int32_t chunk, float* out,
                                               int64_t out_row_stride, void* workspace, size_t workspace_bytes,
                                               int32_t* status, void* stream) {
  const int rc = CheckDecodeArgs(q, k, v, kv_row_stride, kv_head_stride, kv_seq_stride, lens, batch, heads, kv_heads,
                                 head_dim, max_len, chunk, out);
  if (rc != ACCEL_B200_OK) return rc;
  if (batch == 0) return ClearError();
  const int group = heads / kv_heads;
  const size_t need = accel_b200_attention_decode_workspace(batch, heads, kv_heads, max_len, chunk);
  if (workspace == nullptr || workspace_bytes < need) return SetError(ACCEL_B200_EINVAL, "attention_decode: workspace too small");
  DecodeArgs a{};
  a.q = q;
  a.q_row_stride = q_row_stride;
  a.k = k;
  a.v = v;
  a.kv_row_stride = kv_row_stride;
  a.kv_head_stride = kv_head_stride;
  a.kv_seq_stride = kv_seq_stride;
  a.lens = lens;
  a.heads = heads;
  a.kv_heads = kv_heads;
  a.chunk = chunk;
  a.n_chunks = (max_len + chunk - 1) / chunk;
  a.scale = 1.f / sqrtf(static_cast<float>(head_dim));
  a.counters = static_cast<int32_t*>(workspace);
  a.part = reinterpret_cast<float*>(static_cast<char*>(workspace) + kCounterRegion);
  a.status = status;
  a.out = out;
  a.out_row_stride = out_row_stride;
  cudaStream_t s = AsStream(stream);
  switch (group) {
    case 1: return LaunchDecode<1>(a, batch, s);
    case 2: return LaunchDecode<2>(a, batch, s);
    case 3: return LaunchDecode<3>(a, batch, s);
    case 4: return LaunchDecode<4>(a, batch, s);
    case 5: return LaunchDecode<5>(a, batch, s);
    case 6: return LaunchDecode<6>(a, batch, s);
    case 7: return LaunchDecode<7>(a, batch, s);
    default: return LaunchDecode<8>(a, batch, s);
  }
}

ACCEL_B200_API size_t accel_b200_attention_decode_noalloc_limit(void) { return kNoAllocScratchBytes; }

ACCEL_B200_API int accel_b200_attention_decode_noalloc(const float* q, int64_t q_row_stride, const float* k,
                                                       const float* v, int64_t kv_row_stride, int64_t kv_head_stride,
                                                       int64_t kv_seq_stride, const int32_t* lens, int32_t batch,
                                                       int32_t heads, int32_t kv_heads, int32_t head_dim,
                                                       int32_t max_len, int32_t chunk, float* out,
                                                       int64_t out_row_stride, int32_t* status, void* stream) {
  // Every argument is checked before the scratch is touched: a call that
  // fails here queues nothing.
  int rc = CheckDecodeArgs(q, k, v, kv_row_stride, kv_head_stride, kv_seq_stride, lens, batch, heads, kv_heads,
                           head_dim, max_len, chunk, out);
  if (rc != ACCEL_B200_OK) return rc;
  if (batch == 0) return ClearError();
  const size_t need = accel_b200_attention_decode_workspace(batch, heads, kv_heads, max_len, chunk);
  if (need > kNoAllocScratchBytes) {
    return SetError(ACCEL_B200_EINVAL,
                    "attention_decode_noalloc: these sizes need " + std::to_string(need) +
                        " bytes of scratch, above the fixed 4 MiB (4194304 bytes); use accel_b200_attention_decode "
                        "with a caller-owned workspace");
  }
  void* scratch = nullptr;
  rc = ScratchAddress(&scratch);
  if (rc != ACCEL_B200_OK) return rc;
  // The array keeps whatever the last call left; the arrival counters (one
  // per (sequence, kv head), at most the counter region) must start at zero,
  // so they are cleared on this call's stream first.
  const size_t counter_bytes = static_cast<size_t>(batch) * kv_heads * sizeof(int32_t);
  const cudaError_t err = cudaMemsetAsync(scratch, 0, counter_bytes < kCounterRegion ? counter_bytes : kCounterRegion,
                                          AsStream(stream));
  if (err != cudaSuccess) {
    return SetError(ACCEL_B200_ECUDA, std::string("attention_decode_noalloc: ") + cudaGetErrorString(err));
  }
  return accel_b200_attention_decode(q, q_row_stride, k, v, kv_row_stride, kv_head_stride, kv_seq_stride, lens, batch,
                                     heads, kv_heads, head_dim, max_len, chunk, out, out_row_stride, scratch,
                                     kNoAllocScratchBytes, status, stream);
}

ACCEL_B200_API int accel_b200_wait_selftest(int32_t* status, void* stream) {
  if (status == nullptr) return SetError(ACCEL_B200_EINVAL, "wait_selftest: null status");
  WaitSelftestKernel<<<1, 32, 0, AsStream(stream)>>>(status);
  return CheckLaunch("wait_selftest");
}

}  // extern "C"
