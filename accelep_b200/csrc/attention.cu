// Causal grouped-query attention (src/sim_attend.cc:9-46) on the device.
//
// Two kernels:
//  * AttnRowsKernel: one CTA per (query row, head), an online softmax over
//    chunks of the context. Any head_dim up to 1024, any context length.
//    It serves Device::Attention and prefill, where many query rows share
//    each key row and the key rows stay in L2.
//  * AttnDecodeKernel + AttnCombineKernel: split-KV ("flash decoding") for
//    one new query row per sequence with head_dim 64. One CTA per
//    (sequence, kv head, context chunk) reads each key and value row of its
//    chunk once from HBM for all query heads that share the kv head, and
//    writes a partial (max, sum, weighted values) that the combine kernel
//    merges with the log-sum-exp rule.
//
// The reference divides each weight by the sum before the value product;
// here the sum divides the accumulated product once. The two orders agree
// well inside the 1e-4 tolerance.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "accel_b200.h"
#include "common.cuh"

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
  const float* kbase = a.k + seq * a.kv_seq_stride + static_cast<int64_t>(g) * D;
  const float* vbase = a.v + seq * a.kv_seq_stride + static_cast<int64_t>(g) * D;
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

struct DecodeArgs {
  const float* q;  // row b: heads * 64 floats at q + b * q_row_stride
  int64_t q_row_stride;
  const float* k;  // sequence b, row t, kv head g: k + b * kv_seq_stride + t * kv_row_stride + g * 64
  const float* v;
  int64_t kv_row_stride;
  int64_t kv_seq_stride;
  const int32_t* lens;  // context length of sequence b (new row included)
  int32_t heads;
  int32_t kv_heads;
  int32_t chunk;      // context rows per CTA
  int32_t n_chunks;   // grid.x
  float scale;
  float* part;  // [B][heads][n_chunks][kDecD + 2]: weighted values, max, sum
};

template <int G>
__global__ void __launch_bounds__(kDecThreads) AttnDecodeKernel(DecodeArgs a) {
  extern __shared__ float smem[];
  float* q_s = smem;                       // G * 64
  float* p_s = smem + G * kDecD;           // G * chunk
  float* red = p_s + G * a.chunk;          // 4 warps * G * 64 partial values
  __shared__ float stat[2 * kMaxGroup];
  const int c = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t len = a.lens[b];
  const int64_t t0 = static_cast<int64_t>(c) * a.chunk;
  const int cnt = static_cast<int>(Max64(0, Min64(a.chunk, len - t0)));
  const int h0 = g * G;
  float* part_base = a.part + ((static_cast<int64_t>(b) * a.heads + h0) * a.n_chunks + c) * (kDecD + 2);
  const int64_t part_head_stride = static_cast<int64_t>(a.n_chunks) * (kDecD + 2);
  if (cnt == 0) {
    for (int i = tid; i < G; i += blockDim.x) {
      part_base[i * part_head_stride + kDecD] = -INFINITY;
      part_base[i * part_head_stride + kDecD + 1] = 0.f;
    }
    return;
  }
  const float* qrow = a.q + static_cast<int64_t>(b) * a.q_row_stride + static_cast<int64_t>(h0) * kDecD;
  for (int i = tid; i < G * kDecD; i += blockDim.x) q_s[i] = qrow[i];
  __syncthreads();
  const float* kb = a.k + static_cast<int64_t>(b) * a.kv_seq_stride + t0 * a.kv_row_stride + static_cast<int64_t>(g) * kDecD;
  const float* vb = a.v + static_cast<int64_t>(b) * a.kv_seq_stride + t0 * a.kv_row_stride + static_cast<int64_t>(g) * kDecD;
  // Scores: one key row per thread, 16-byte loads, all G heads per row.
  for (int j = tid; j < cnt; j += blockDim.x) {
    const float4* kr = reinterpret_cast<const float4*>(kb + j * a.kv_row_stride);
    float dot[G];
#pragma unroll
    for (int hh = 0; hh < G; ++hh) dot[hh] = 0.f;
#pragma unroll
    for (int d4 = 0; d4 < kDecD / 4; ++d4) {
      const float4 kv = __ldg(kr + d4);
#pragma unroll
      for (int hh = 0; hh < G; ++hh) {
        // Every lane reads the same q words: a shared-memory broadcast.
        const float* qh = q_s + hh * kDecD + d4 * 4;
        dot[hh] = fmaf(qh[0], kv.x, dot[hh]);
        dot[hh] = fmaf(qh[1], kv.y, dot[hh]);
        dot[hh] = fmaf(qh[2], kv.z, dot[hh]);
        dot[hh] = fmaf(qh[3], kv.w, dot[hh]);
      }
    }
#pragma unroll
    for (int hh = 0; hh < G; ++hh) p_s[hh * a.chunk + j] = dot[hh] * a.scale;
  }
  __syncthreads();
  // Per head: max and exp-sum over the chunk; warp hh handles head hh.
  for (int hh = warp; hh < G; hh += kDecThreads / 32) {
    float mx = -INFINITY;
    for (int j = lane; j < cnt; j += 32) mx = fmaxf(mx, p_s[hh * a.chunk + j]);
    mx = WarpMax(mx);
    float sum = 0.f;
    for (int j = lane; j < cnt; j += 32) {
      const float p = expf(p_s[hh * a.chunk + j] - mx);
      p_s[hh * a.chunk + j] = p;
      sum += p;
    }
    sum = WarpSum(sum);
    if (lane == 0) {
      stat[2 * hh] = mx;
      stat[2 * hh + 1] = sum;
    }
  }
  __syncthreads();
  // Weighted values: warp w takes rows w, w + 4, ...; lane owns d = 2 lane, 2 lane + 1.
  float acc[G][2];
#pragma unroll
  for (int hh = 0; hh < G; ++hh) acc[hh][0] = acc[hh][1] = 0.f;
  for (int j = warp; j < cnt; j += kDecThreads / 32) {
    const float2 vv = __ldg(reinterpret_cast<const float2*>(vb + j * a.kv_row_stride) + lane);
#pragma unroll
    for (int hh = 0; hh < G; ++hh) {
      const float p = p_s[hh * a.chunk + j];
      acc[hh][0] = fmaf(p, vv.x, acc[hh][0]);
      acc[hh][1] = fmaf(p, vv.y, acc[hh][1]);
    }
  }
#pragma unroll
  for (int hh = 0; hh < G; ++hh) {
    red[(warp * G + hh) * kDecD + 2 * lane] = acc[hh][0];
    red[(warp * G + hh) * kDecD + 2 * lane + 1] = acc[hh][1];
  }
  __syncthreads();
  for (int i = tid; i < G * kDecD; i += blockDim.x) {
    const int hh = i / kDecD, d = i % kDecD;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kDecThreads / 32; ++w) s += red[(w * G + hh) * kDecD + d];
    part_base[hh * part_head_stride + d] = s;
  }
  if (tid < G) {
    part_base[tid * part_head_stride + kDecD] = stat[2 * tid];
    part_base[tid * part_head_stride + kDecD + 1] = stat[2 * tid + 1];
  }
}

// One warp per (sequence, head): merge the chunk partials.
__global__ void AttnCombineKernel(const float* __restrict__ part, const int32_t* __restrict__ lens, int32_t heads,
                                  int32_t chunk, int32_t n_chunks, float* __restrict__ out, int64_t out_row_stride,
                                  int32_t batch) {
  const int lane = threadIdx.x & 31;
  const int64_t pair = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (pair >= static_cast<int64_t>(batch) * heads) return;
  const int64_t b = pair / heads;
  const int h = static_cast<int>(pair % heads);
  const int used = static_cast<int>((static_cast<int64_t>(lens[b]) + chunk - 1) / chunk);
  const float* p = part + pair * n_chunks * (kDecD + 2);
  float mx = -INFINITY;
  for (int c = 0; c < used; ++c) mx = fmaxf(mx, p[c * (kDecD + 2) + kDecD]);
  float l = 0.f, o0 = 0.f, o1 = 0.f;
  for (int c = 0; c < used; ++c) {
    const float* pc = p + c * (kDecD + 2);
    const float w = expf(pc[kDecD] - mx);
    l = fmaf(pc[kDecD + 1], w, l);
    o0 = fmaf(pc[2 * lane], w, o0);
    o1 = fmaf(pc[2 * lane + 1], w, o1);
  }
  float* orow = out + b * out_row_stride + static_cast<int64_t>(h) * kDecD;
  orow[2 * lane] = o0 / l;
  orow[2 * lane + 1] = o1 / l;
}

int LaunchRows(const RowsArgs& a, int64_t rows, cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(a.head_dim + kRowsChunk) * sizeof(float);
  if (rows > 2147483647LL || a.heads > 65535) return SetError(ACCEL_B200_EINVAL, "attention: grid too large");
  AttnRowsKernel<<<dim3(static_cast<unsigned>(rows), static_cast<unsigned>(a.heads)), kRowsThreads, smem, stream>>>(a);
  return CheckLaunch("attention_rows");
}

template <int G>
int LaunchDecode(const DecodeArgs& a, int32_t batch, cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(G * kDecD + G * a.chunk + (kDecThreads / 32) * G * kDecD) * sizeof(float);
  AttnDecodeKernel<G><<<dim3(a.n_chunks, a.kv_heads, batch), kDecThreads, smem, stream>>>(a);
  return CheckLaunch("attention_decode");
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
                                             int64_t kv_row_stride, int64_t kv_seq_stride, float* out,
                                             int64_t out_row_stride, const int32_t* row_seq, const int32_t* row_pos,
                                             int64_t rows, int32_t heads, int32_t kv_heads, int32_t head_dim,
                                             void* stream) {
  if (rows < 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads != 0 || head_dim <= 0 ||
      head_dim > kMaxDPerThread * kRowsThreads || row_pos == nullptr) {
    return SetError(ACCEL_B200_EINVAL, "attention_rows: bad arguments");
  }
  if (rows == 0) return ClearError();
  RowsArgs a{q, q_row_stride, k, v, kv_row_stride, kv_seq_stride, out, out_row_stride, row_seq, row_pos, 0,
             heads, kv_heads, head_dim, 1.f / sqrtf(static_cast<float>(head_dim))};
  return LaunchRows(a, rows, AsStream(stream));
}

ACCEL_B200_API size_t accel_b200_attention_decode_workspace(int32_t batch, int32_t heads, int32_t max_len,
                                                            int32_t chunk) {
  if (batch <= 0 || heads <= 0 || max_len <= 0 || chunk <= 0) return 0;
  const int64_t chunks = (max_len + chunk - 1) / chunk;
  return static_cast<size_t>(batch) * heads * chunks * (kDecD + 2) * sizeof(float);
}

ACCEL_B200_API int accel_b200_attention_decode(const float* q, int64_t q_row_stride, const float* k, const float* v,
                                               int64_t kv_row_stride, int64_t kv_seq_stride, const int32_t* lens,
                                               int32_t batch, int32_t heads, int32_t kv_heads, int32_t head_dim,
                                               int32_t max_len, int32_t chunk, float* out, int64_t out_row_stride,
                                               void* workspace, size_t workspace_bytes, void* stream) {
  if (batch < 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads != 0 || head_dim != kDecD || max_len <= 0 ||
      chunk <= 0 || chunk > 1024 || lens == nullptr) {
    return SetError(ACCEL_B200_EINVAL, "attention_decode: bad arguments");
  }
  if (batch == 0) return ClearError();
  const int group = heads / kv_heads;
  if (group > kMaxGroup) return SetError(ACCEL_B200_EINVAL, "attention_decode: more than 8 query heads per kv head");
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) % 16 != 0 || kv_row_stride % 4 != 0 ||
      kv_seq_stride % 4 != 0) {
    return SetError(ACCEL_B200_EINVAL, "attention_decode: cache rows must be 16-byte aligned");
  }
  const size_t need = accel_b200_attention_decode_workspace(batch, heads, max_len, chunk);
  if (workspace == nullptr || workspace_bytes < need) return SetError(ACCEL_B200_EINVAL, "attention_decode: workspace too small");
  DecodeArgs a{};
  a.q = q;
  a.q_row_stride = q_row_stride;
  a.k = k;
  a.v = v;
  a.kv_row_stride = kv_row_stride;
  a.kv_seq_stride = kv_seq_stride;
  a.lens = lens;
  a.heads = heads;
  a.kv_heads = kv_heads;
  a.chunk = chunk;
  a.n_chunks = (max_len + chunk - 1) / chunk;
  a.scale = 1.f / sqrtf(static_cast<float>(head_dim));
  a.part = static_cast<float*>(workspace);
  cudaStream_t s = AsStream(stream);
  int rc;
  switch (group) {
    case 1: rc = LaunchDecode<1>(a, batch, s); break;
    case 2: rc = LaunchDecode<2>(a, batch, s); break;
    case 3: rc = LaunchDecode<3>(a, batch, s); break;
    case 4: rc = LaunchDecode<4>(a, batch, s); break;
    case 5: rc = LaunchDecode<5>(a, batch, s); break;
    case 6: rc = LaunchDecode<6>(a, batch, s); break;
    case 7: rc = LaunchDecode<7>(a, batch, s); break;
    default: rc = LaunchDecode<8>(a, batch, s); break;
  }
  if (rc != ACCEL_B200_OK) return rc;
  const int64_t pairs = static_cast<int64_t>(batch) * heads;
  AttnCombineKernel<<<static_cast<unsigned>(CeilDiv(pairs, 4)), 128, 0, s>>>(a.part, lens, heads, chunk, a.n_chunks, out,
                                                                             out_row_stride, batch);
  return CheckLaunch("attention_combine");
}

}  // extern "C"
