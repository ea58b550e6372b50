// Row and elementwise kernels behind the named device calls: embedding,
// RMSNorm, RoPE, cache append, SiLU-mul, residual add, the GEMM epilogue and
// transpose. All are HBM-bound; each thread moves 16-byte vectors where the
// row allows it and grids are sized in multiples of the SM count.
#include <cuda_runtime.h>
#include <stdint.h>

#include "accel_b200.h"
#include "common.cuh"

namespace accel_b200 {
namespace {

inline int GridFor(int64_t work, int block, int per_sm = 8) {
  const int64_t blocks = CeilDiv(work, block);
  const int64_t cap = static_cast<int64_t>(kSms) * per_sm;
  return static_cast<int>(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

// One CTA per output row; out-of-range ids set the status bit and skip the row
// (src/sim_embed.cc:12-15 throws there).
__global__ void EmbedKernel(const int32_t* __restrict__ ids, int64_t id_offset, const float* __restrict__ table,
                            float* __restrict__ out, int64_t seq, int64_t hidden, int64_t vocab, int32_t* status) {
  PdlTrigger();
  PdlWait();
  for (int64_t s = blockIdx.x; s < seq; s += gridDim.x) {
    const int32_t id = ids[id_offset + s];
    if (id < 0 || id >= vocab) {
      if (threadIdx.x == 0 && status != nullptr) atomicOr(status, ACCEL_B200_STATUS_BAD_TOKEN);
      continue;
    }
    const float* src = table + static_cast<int64_t>(id) * hidden;
    float* dst = out + s * hidden;
    const bool vec = (hidden % 4 == 0) && ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) % 16 == 0);
    if (vec) {
      const float4* s4 = reinterpret_cast<const float4*>(src);
      float4* d4 = reinterpret_cast<float4*>(dst);
      for (int64_t i = threadIdx.x; i < hidden / 4; i += blockDim.x) d4[i] = s4[i];
    } else {
      for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) dst[i] = src[i];
    }
  }
}

// One warp per row. Sum of squares in double (src/sim_rmsnorm.cc:11-14), one
// double reciprocal square root, float(x * inv) * w.
__global__ void RmsNormKernel(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ y,
                              int64_t rows, int64_t dim, float eps, int64_t row_offset, int64_t ldx, int64_t ldy) {
  PdlTrigger();
  PdlWait();
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const float* in = x + (row_offset + r) * ldx;
    float* out = y + r * ldy;
    double sq = 0.0;
    for (int64_t i = lane; i < dim; i += 32) {
      const double v = static_cast<double>(in[i]);
      sq += v * v;
    }
    sq = WarpSum(sq);
    const double inv = 1.0 / sqrt(sq / static_cast<double>(dim) + static_cast<double>(eps));
    for (int64_t i = lane; i < dim; i += 32) {
      out[i] = __fmul_rn(static_cast<float>(static_cast<double>(in[i]) * inv), w[i]);
    }
  }
}

// One thread per rotated pair (s, h, i < half); rounded steps as in
// src/sim_rope.cc:16-17 so the result keeps the reference's bits.
__global__ void RopeKernel(float* __restrict__ states, const float* __restrict__ cos_t,
                           const float* __restrict__ sin_t, int64_t seq, int64_t n_heads, int64_t head_dim,
                           int64_t position) {
  const int64_t half = head_dim / 2;
  const int64_t total = seq * n_heads * half;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = idx % half;
    const int64_t sh = idx / half;
    const int64_t s = sh / n_heads;
    float* row = states + sh * head_dim;
    const float* c = cos_t + (position + s) * head_dim;
    const float* sn = sin_t + (position + s) * head_dim;
    const float a = row[i];
    const float b = row[half + i];
    row[i] = __fsub_rn(__fmul_rn(a, c[i]), __fmul_rn(b, sn[i]));
    row[half + i] = __fadd_rn(__fmul_rn(b, c[half + i]), __fmul_rn(a, sn[half + i]));
  }
}

// src/sim_silu.cc:10-11.
__global__ void SiluMulKernel(float* __restrict__ gate, const float* __restrict__ up, int64_t count) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float g = gate[i];
    gate[i] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, expf(-g))), up[i]);
  }
}

__global__ void AddKernel(float* __restrict__ dest, const float* __restrict__ extra, int64_t count) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    dest[i] = __fadd_rn(dest[i], extra[i]);
  }
}

__global__ void EpilogueKernel(float* __restrict__ c, int64_t m, int64_t n, Epilogue ep) {
  const int64_t total = m * n;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = idx / n;
    const int64_t j = idx - i * n;
    c[idx] = ApplyEpilogue(ep, c[idx], i, j);
  }
}

// 32x32 tiles through shared memory (padded row avoids bank conflicts).
__global__ void TransposeKernel(const float* __restrict__ src, float* __restrict__ dst, int64_t rows, int64_t cols) {
  __shared__ float tile[32][33];
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * 32;
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * 32;
  for (int dy = threadIdx.y; dy < 32; dy += blockDim.y) {
    const int64_t r = r0 + dy, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[dy][threadIdx.x] = src[r * cols + c];
  }
  __syncthreads();
  for (int dy = threadIdx.y; dy < 32; dy += blockDim.y) {
    const int64_t c = c0 + dy, r = r0 + threadIdx.x;
    if (r < rows && c < cols) dst[c * rows + r] = tile[threadIdx.x][dy];
  }
}

// Largest |a - b| (src/llama_model.cc:168-181): a NaN difference never wins.
__global__ void MaxAbsDiffKernel(const float* __restrict__ a, const float* __restrict__ b, int64_t n, float* out) {
  __shared__ float red[32];
  float m = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float d = fabsf(a[i] - b[i]);
    if (d > m) m = d;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float y = __shfl_xor_sync(kFull, m, o);
    if (y > m) m = y;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float r = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w)
      if (red[w] > r) r = red[w];
    *out = r;
  }
}

bool BadDims(int64_t a, int64_t b = 0, int64_t c = 0, int64_t d = 0) { return a < 0 || b < 0 || c < 0 || d < 0; }

}  // namespace

// Bias strides of a rank-0..2 bias shape right-aligned against [m, n]
// (src/sim_device.cc:104-124): a size-1 axis broadcasts with stride 0.
bool BiasStrides(const int64_t* shape, int rank, int64_t m, int64_t n, int64_t* rs, int64_t* cs) {
  *rs = 0;
  *cs = 0;
  if (rank == 0) return true;
  if (rank == 1) {
    if (shape[0] != 1 && shape[0] != n) return false;
    *cs = shape[0] == 1 ? 0 : 1;
    return true;
  }
  if (rank == 2) {
    if ((shape[0] != 1 && shape[0] != m) || (shape[1] != 1 && shape[1] != n)) return false;
    *rs = shape[0] == 1 ? 0 : shape[1];
    *cs = shape[1] == 1 ? 0 : 1;
    return true;
  }
  return false;
}

// RmsNorm of `rows` rows of length dim: x rows at x + (row_offset + r) * ldx,
// output rows at y + r * ldy.
int LaunchRmsNormRows(const float* x, int64_t ldx, const float* w, float* y, int64_t ldy, int64_t rows, int64_t dim,
                      float eps, int64_t row_offset, cudaStream_t stream) {
  return CheckLaunchEx(LaunchK(RmsNormKernel, dim3(GridFor(rows, 8, 16)), dim3(256), 0, stream, 1u, 1u, x, w, y, rows,
                               dim, eps, row_offset, ldx, ldy),
                       "rmsnorm");
}

}  // namespace accel_b200

using namespace accel_b200;

extern "C" {

ACCEL_B200_API int accel_b200_embed(const int32_t* ids, int64_t id_offset, const float* table, float* out, int64_t seq,
                                    int64_t hidden, int64_t vocab, int32_t* status, void* stream) {
  if (BadDims(id_offset, seq, hidden, vocab)) return SetError(ACCEL_B200_EINVAL, "embed: negative size");
  if (seq == 0 || hidden == 0) return ClearError();
  if (ids == nullptr || table == nullptr || out == nullptr) return SetError(ACCEL_B200_EINVAL, "embed: null pointer");
  return CheckLaunchEx(LaunchK(EmbedKernel, dim3(GridFor(seq, 1, 16)), dim3(128), 0, AsStream(stream), 1u, 1u, ids,
                               id_offset, table, out, seq, hidden, vocab, status),
                       "embed");
}

ACCEL_B200_API int accel_b200_rmsnorm(const float* x, const float* weight, float* y, int64_t rows, int64_t dim,
                                      float eps, int64_t row_offset, void* stream) {
  if (BadDims(rows, dim, row_offset)) return SetError(ACCEL_B200_EINVAL, "rmsnorm: negative size");
  if (rows == 0 || dim == 0) return ClearError();
  if (x == nullptr || weight == nullptr || y == nullptr) return SetError(ACCEL_B200_EINVAL, "rmsnorm: null pointer");
  return LaunchRmsNormRows(x, dim, weight, y, dim, rows, dim, eps, row_offset, AsStream(stream));
}

ACCEL_B200_API int accel_b200_rope(float* states, const float* cos_table, const float* sin_table, int64_t seq,
                                   int64_t n_heads, int64_t head_dim, int64_t position, void* stream) {
  if (BadDims(seq, n_heads, head_dim, position)) return SetError(ACCEL_B200_EINVAL, "rope: negative size");
  const int64_t work = seq * n_heads * (head_dim / 2);
  if (work == 0) return ClearError();
  if (states == nullptr || cos_table == nullptr || sin_table == nullptr)
    return SetError(ACCEL_B200_EINVAL, "rope: null pointer");
  RopeKernel<<<GridFor(work, 256), 256, 0, AsStream(stream)>>>(states, cos_table, sin_table, seq, n_heads, head_dim,
                                                               position);
  return CheckLaunch("rope");
}

ACCEL_B200_API int accel_b200_append_cache(const float* src, float* cache, int64_t seq, int64_t position,
                                           int64_t n_heads, int64_t head_dim, void* stream) {
  if (BadDims(seq, position, n_heads, head_dim)) return SetError(ACCEL_B200_EINVAL, "append_cache: negative size");
  const int64_t row = n_heads * head_dim;
  const size_t bytes = static_cast<size_t>(seq * row) * sizeof(float);
  if (bytes == 0) return ClearError();
  if (src == nullptr || cache == nullptr) return SetError(ACCEL_B200_EINVAL, "append_cache: null pointer");
  const cudaError_t err = cudaMemcpyAsync(cache + position * row, src, bytes, cudaMemcpyDeviceToDevice, AsStream(stream));
  if (err != cudaSuccess) return SetError(ACCEL_B200_ECUDA, std::string("append_cache: ") + cudaGetErrorString(err));
  return ClearError();
}

ACCEL_B200_API int accel_b200_silu_mul(float* gate, const float* up, int64_t count, void* stream) {
  if (count < 0) return SetError(ACCEL_B200_EINVAL, "silu_mul: negative size");
  if (count == 0) return ClearError();
  if (gate == nullptr || up == nullptr) return SetError(ACCEL_B200_EINVAL, "silu_mul: null pointer");
  SiluMulKernel<<<GridFor(count, 256), 256, 0, AsStream(stream)>>>(gate, up, count);
  return CheckLaunch("silu_mul");
}

ACCEL_B200_API int accel_b200_residual_add(float* dest, const float* extra, int64_t count, void* stream) {
  if (count < 0) return SetError(ACCEL_B200_EINVAL, "residual_add: negative size");
  if (count == 0) return ClearError();
  if (dest == nullptr || extra == nullptr) return SetError(ACCEL_B200_EINVAL, "residual_add: null pointer");
  AddKernel<<<GridFor(count, 256), 256, 0, AsStream(stream)>>>(dest, extra, count);
  return CheckLaunch("residual_add");
}

ACCEL_B200_API int accel_b200_gemm_epilogue(float* c, int64_t m, int64_t n, float alpha, const float* bias,
                                            const int64_t* bias_shape, int32_t bias_rank, float beta, int32_t act,
                                            void* stream) {
  if (BadDims(m, n)) return SetError(ACCEL_B200_EINVAL, "gemm_epilogue: negative size");
  Epilogue ep;
  ep.alpha = alpha;
  ep.beta = beta;
  ep.act = act;
  if (bias != nullptr) {
    if (bias_rank < 0 || bias_rank > 2 || (bias_rank > 0 && bias_shape == nullptr) ||
        !BiasStrides(bias_shape, bias_rank, m, n, &ep.bias_rs, &ep.bias_cs)) {
      return SetError(ACCEL_B200_EINVAL, "gemm_epilogue: bias shape does not broadcast");
    }
    ep.bias = bias;
  }
  if (m * n == 0) return ClearError();
  if (c == nullptr) return SetError(ACCEL_B200_EINVAL, "gemm_epilogue: null output");
  EpilogueKernel<<<GridFor(m * n, 256), 256, 0, AsStream(stream)>>>(c, m, n, ep);
  return CheckLaunch("gemm_epilogue");
}

ACCEL_B200_API int accel_b200_transpose(const float* src, float* dst, int64_t rows, int64_t cols, void* stream) {
  if (BadDims(rows, cols)) return SetError(ACCEL_B200_EINVAL, "transpose: negative size");
  if (rows == 0 || cols == 0) return ClearError();
  if (src == nullptr || dst == nullptr) return SetError(ACCEL_B200_EINVAL, "transpose: null pointer");
  if (CeilDiv(rows, 32) > 65535) return SetError(ACCEL_B200_EINVAL, "transpose: too many rows");
  const dim3 grid(static_cast<unsigned>(CeilDiv(cols, 32)), static_cast<unsigned>(CeilDiv(rows, 32)));
  TransposeKernel<<<grid, dim3(32, 8), 0, AsStream(stream)>>>(src, dst, rows, cols);
  return CheckLaunch("transpose");
}

ACCEL_B200_API int accel_b200_max_abs_diff(const float* a, const float* b, int64_t n, float* out, void* stream) {
  if (n < 0 || a == nullptr || b == nullptr || out == nullptr) return SetError(ACCEL_B200_EINVAL, "max_abs_diff: bad arguments");
  MaxAbsDiffKernel<<<1, 1024, 0, AsStream(stream)>>>(a, b, n, out);
  return CheckLaunch("max_abs_diff");
}

}  // extern "C"
