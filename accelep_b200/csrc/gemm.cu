// Products with the weight in the reference's device layout: B is [k, n]
// row-major (n contiguous), as SimDevice stores a MatMul right-hand side and
// an int8 QuantPlane.
//
//  * MatMulExactKernel: Device::MatMul. Each output is a k-ascending chain of
//    rounded products and rounded adds, exactly PackedMatMul's arithmetic
//    (src/sim_device.cc:346-357), so the result has the reference's bits.
//  * GemmKnKernel<W, MT, VEC>: the fast path for fp32 and int8 weights with
//    small M (decode). A thread owns MT rows x VEC adjacent columns; a warp
//    reads 32 x VEC contiguous weight elements of one k row per step (16-byte
//    loads where alignment allows); the A rows of the current k slice sit in
//    shared memory as [k][MT] so one 16-byte load feeds four rows. int8
//    weights are dequantized in registers, element by element, to the
//    reference's value (float(q) - zero) * scale (src/sim_device.cc:406-424).
//    K is split across CTAs until the grid covers the SMs; split partials go
//    to a workspace and a second kernel sums them in split order
//    (deterministic) and applies the fused epilogue.
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "accel_b200.h"
#include "common.cuh"

namespace accel_b200 {
namespace {

constexpr int kGemmThreads = 128;
constexpr int kKc = 16;  // k rows staged per step; also the split granularity

struct GemmArgs {
  const float* a;
  int64_t lda;
  const void* w;  // float or int8, [k, n], row stride n
  const float* scale;
  const int8_t* zero;
  int32_t axis;  // int8 only: -1 one value, 0 per k row, 1 per column
  float* c;
  int64_t ldc;
  int64_t m, k, n;
  int64_t k_per_split;
  float* part;  // splits > 1: [splits][m][n]
  Epilogue ep;
};

template <typename W, int VEC>
struct WeightVec;

template <int VEC>
struct WeightVec<float, VEC> {
  static __device__ __forceinline__ void Load(const GemmArgs& g, int64_t kk, int64_t j, bool fast, float (&out)[VEC]) {
    const float* row = static_cast<const float*>(g.w) + kk * g.n + j;
    if (fast) {
#pragma unroll
      for (int v = 0; v < VEC; v += 4) {
        const float4 x = __ldg(reinterpret_cast<const float4*>(row + v));
        out[v] = x.x;
        out[v + 1] = x.y;
        out[v + 2] = x.z;
        out[v + 3] = x.w;
      }
    } else {
#pragma unroll
      for (int v = 0; v < VEC; ++v) out[v] = (j + v < g.n) ? __ldg(row + v) : 0.f;
    }
  }
};

template <int VEC>
struct WeightVec<int8_t, VEC> {
  static __device__ __forceinline__ void Load(const GemmArgs& g, int64_t kk, int64_t j, bool fast, float (&out)[VEC]) {
    const int8_t* row = static_cast<const int8_t*>(g.w) + kk * g.n + j;
    int8_t raw[VEC];
    if (fast) {
      if constexpr (VEC == 16) {
        const int4 x = __ldg(reinterpret_cast<const int4*>(row));
        *reinterpret_cast<int4*>(raw) = x;
      } else if constexpr (VEC == 8) {
        const int2 x = __ldg(reinterpret_cast<const int2*>(row));
        *reinterpret_cast<int2*>(raw) = x;
      } else if constexpr (VEC == 4) {
        const int x = __ldg(reinterpret_cast<const int*>(row));
        *reinterpret_cast<int*>(raw) = x;
      } else {
#pragma unroll
        for (int v = 0; v < VEC; ++v) raw[v] = row[v];
      }
    } else {
#pragma unroll
      for (int v = 0; v < VEC; ++v) raw[v] = (j + v < g.n) ? row[v] : 0;
    }
    // Dequantize like DequantAt: (float(q) - zero) * scale, one rounding.
    if (g.axis == 0) {
      const float sc = __ldg(g.scale + kk);
      const float zp = g.zero != nullptr ? static_cast<float>(g.zero[kk]) : 0.f;
#pragma unroll
      for (int v = 0; v < VEC; ++v) out[v] = __fmul_rn(static_cast<float>(raw[v]) - zp, sc);
    } else {
#pragma unroll
      for (int v = 0; v < VEC; ++v) out[v] = static_cast<float>(raw[v]);
    }
  }
};

// Column-indexed dequantization factors (axis 1 or one value), held per thread.
template <typename W, int VEC>
__device__ __forceinline__ void ColumnFactors(const GemmArgs& g, int64_t j, float (&sc)[VEC], float (&zp)[VEC]) {
#pragma unroll
  for (int v = 0; v < VEC; ++v) {
    sc[v] = 1.f;
    zp[v] = 0.f;
  }
  if constexpr (sizeof(W) == 1) {
    if (g.axis == 1) {
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        const bool ok = j + v < g.n;
        sc[v] = ok ? __ldg(g.scale + j + v) : 0.f;
        zp[v] = (ok && g.zero != nullptr) ? static_cast<float>(g.zero[j + v]) : 0.f;
      }
    } else if (g.axis < 0) {
      const float s0 = __ldg(g.scale);
      const float z0 = g.zero != nullptr ? static_cast<float>(g.zero[0]) : 0.f;
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        sc[v] = s0;
        zp[v] = z0;
      }
    }
  }
}

template <typename W, int MT, int VEC>
__global__ void __launch_bounds__(kGemmThreads) GemmKnKernel(GemmArgs g) {
  static_assert(sizeof(W) == 1 || VEC % 4 == 0, "fp32 rows load in float4 groups");
  constexpr int MTP = (MT + 3) / 4 * 4;  // A staging row padded to a float4
  __shared__ __align__(16) float a_s[kKc][MTP];
  const int64_t j = (static_cast<int64_t>(blockIdx.x) * kGemmThreads + threadIdx.x) * VEC;
  const int64_t row0 = static_cast<int64_t>(blockIdx.z) * MT;
  const int64_t kb = static_cast<int64_t>(blockIdx.y) * g.k_per_split;
  const int64_t ke = Min64(g.k, kb + g.k_per_split);
  const bool active = j < g.n;
  const bool fast = active && (j + VEC <= g.n) && (g.n % VEC == 0) &&
                    (reinterpret_cast<uintptr_t>(g.w) % (VEC * sizeof(W)) == 0);
  float sc[VEC], zp[VEC];
  if (active) ColumnFactors<W, VEC>(g, j, sc, zp);
  const bool col_dequant = sizeof(W) == 1 && g.axis != 0;
  float acc[MT][VEC];
#pragma unroll
  for (int r = 0; r < MT; ++r)
#pragma unroll
    for (int v = 0; v < VEC; ++v) acc[r][v] = 0.f;

  for (int64_t k0 = kb; k0 < ke; k0 += kKc) {
    const int kn = static_cast<int>(Min64(kKc, ke - k0));
    __syncthreads();
    for (int idx = threadIdx.x; idx < kKc * MTP; idx += kGemmThreads) {
      const int kk = idx / MTP, r = idx % MTP;
      const int64_t row = row0 + r;
      a_s[kk][r] = (kk < kn && r < MT && row < g.m) ? g.a[row * g.lda + k0 + kk] : 0.f;
    }
    __syncthreads();
    if (!active) continue;
#pragma unroll 4
    for (int kk = 0; kk < kn; ++kk) {
      float wv[VEC];
      WeightVec<W, VEC>::Load(g, k0 + kk, j, fast, wv);
      if (col_dequant) {
#pragma unroll
        for (int v = 0; v < VEC; ++v) wv[v] = __fmul_rn(wv[v] - zp[v], sc[v]);
      }
#pragma unroll
      for (int r4 = 0; r4 < MTP; r4 += 4) {
        const float4 av = *reinterpret_cast<const float4*>(&a_s[kk][r4]);
        const float ar[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (r4 + q < MT) {
#pragma unroll
            for (int v = 0; v < VEC; ++v) acc[r4 + q][v] = fmaf(ar[q], wv[v], acc[r4 + q][v]);
          }
        }
      }
    }
  }
  if (!active) return;
  const bool split = gridDim.y > 1;
#pragma unroll
  for (int r = 0; r < MT; ++r) {
    const int64_t row = row0 + r;
    if (row >= g.m) break;
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      if (j + v >= g.n) break;
      if (split) {
        g.part[(static_cast<int64_t>(blockIdx.y) * g.m + row) * g.n + j + v] = acc[r][v];
      } else {
        g.c[row * g.ldc + j + v] = ApplyEpilogue(g.ep, acc[r][v], row, j + v);
      }
    }
  }
}

__global__ void SplitReduceKernel(const float* __restrict__ part, int splits, int64_t m, int64_t n, float* c,
                                  int64_t ldc, Epilogue ep) {
  const int64_t total = m * n;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float s = 0.f;
    for (int p = 0; p < splits; ++p) s += part[p * total + idx];
    const int64_t i = idx / n, jj = idx - i * n;
    c[i * ldc + jj] = ApplyEpilogue(ep, s, i, jj);
  }
}

// Device::MatMul. One thread per output element; k-ascending chain with the
// reference's rounding. Coalesced along n.
__global__ void MatMulExactKernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ c,
                                  int64_t m, int64_t k, int64_t n) {
  const int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (j >= n) return;
  for (int64_t i = blockIdx.y; i < m; i += gridDim.y) {
    const float* arow = a + i * k;
    float acc = 0.f;
    for (int64_t kk = 0; kk < k; ++kk) acc = __fadd_rn(acc, __fmul_rn(__ldg(arow + kk), __ldg(b + kk * n + j)));
    c[i * n + j] = acc;
  }
}

struct Plan {
  int mt, vec;
  int64_t col_blocks, row_blocks, splits, k_per_split;
};

Plan MakePlan(bool int8, int64_t m, int64_t k, int64_t n) {
  Plan p{};
  if (m <= 1) {
    p.mt = 1;
    p.vec = int8 ? 16 : 4;
  } else if (m <= 2) {
    p.mt = 2;
    p.vec = int8 ? 16 : 4;
  } else if (m <= 4) {
    p.mt = 4;
    p.vec = int8 ? 8 : 4;
  } else if (m <= 8) {
    p.mt = 8;
    p.vec = int8 ? 8 : 4;
  } else {
    p.mt = 16;
    p.vec = 4;
  }
  p.col_blocks = CeilDiv(n, static_cast<int64_t>(kGemmThreads) * p.vec);
  p.row_blocks = CeilDiv(m, p.mt);
  const int64_t base = p.col_blocks * p.row_blocks;
  const int64_t want = CeilDiv(static_cast<int64_t>(kSms) * 4, base);
  const int64_t max_splits = CeilDiv(k, kKc);
  p.splits = want < 1 ? 1 : (want > max_splits ? max_splits : want);
  p.k_per_split = CeilDiv(CeilDiv(k, p.splits), kKc) * kKc;
  p.splits = k == 0 ? 1 : CeilDiv(k, p.k_per_split);
  return p;
}

template <typename W, int MT, int VEC>
void LaunchKn(const GemmArgs& g, const Plan& p, cudaStream_t s) {
  GemmKnKernel<W, MT, VEC><<<dim3(static_cast<unsigned>(p.col_blocks), static_cast<unsigned>(p.splits),
                                  static_cast<unsigned>(p.row_blocks)),
                             kGemmThreads, 0, s>>>(g);
}

template <typename W>
int RunGemm(GemmArgs g, cudaStream_t s, void* workspace, size_t workspace_bytes) {
  const bool int8 = sizeof(W) == 1;
  const Plan p = MakePlan(int8, g.m, g.k, g.n);
  if (p.row_blocks > 65535 || p.splits > 65535) return SetError(ACCEL_B200_EINVAL, "matmul: grid too large");
  g.k_per_split = p.k_per_split;
  if (p.splits > 1) {
    const size_t need = kCounterRegion + static_cast<size_t>(p.splits) * g.m * g.n * sizeof(float);
    if (workspace == nullptr || workspace_bytes < need) return SetError(ACCEL_B200_EINVAL, "matmul: workspace too small");
    g.part = reinterpret_cast<float*>(static_cast<char*>(workspace) + kCounterRegion);
  }
  switch (p.mt * 100 + p.vec) {
    case 116: LaunchKn<W, 1, 16>(g, p, s); break;
    case 104: LaunchKn<W, 1, 4>(g, p, s); break;
    case 216: LaunchKn<W, 2, 16>(g, p, s); break;
    case 204: LaunchKn<W, 2, 4>(g, p, s); break;
    case 408: LaunchKn<W, 4, 8>(g, p, s); break;
    case 404: LaunchKn<W, 4, 4>(g, p, s); break;
    case 808: LaunchKn<W, 8, 8>(g, p, s); break;
    case 804: LaunchKn<W, 8, 4>(g, p, s); break;
    default: LaunchKn<W, 16, 4>(g, p, s); break;
  }
  int rc = CheckLaunch("matmul_kn");
  if (rc != ACCEL_B200_OK || p.splits == 1) return rc;
  const int64_t total = g.m * g.n;
  const int grid = static_cast<int>(Min64(CeilDiv(total, 256), static_cast<int64_t>(kSms) * 8));
  SplitReduceKernel<<<grid, 256, 0, s>>>(g.part, static_cast<int>(p.splits), g.m, g.n, g.c, g.ldc, g.ep);
  return CheckLaunch("matmul_split_reduce");
}

size_t WorkspaceFor(bool int8, int64_t m, int64_t k, int64_t n) {
  if (m <= 0 || k <= 0 || n <= 0) return 0;
  const Plan p = MakePlan(int8, m, k, n);
  return p.splits > 1 ? kCounterRegion + static_cast<size_t>(p.splits) * m * n * sizeof(float) : 0;
}

bool ToEpilogue(const accel_b200_epilogue* in, Epilogue* out) {
  *out = Epilogue{};
  if (in == nullptr) return true;
  out->alpha = in->alpha;
  out->beta = in->beta;
  out->bias = in->bias;
  out->bias_rs = in->bias_row_stride;
  out->bias_cs = in->bias_col_stride;
  out->act = in->act;
  out->residual = in->residual;
  out->residual_ld = in->residual_ld;
  out->row_sq = in->row_sq;
  out->row_sq_ld = in->row_sq_ld;
  out->flags = in->flags;
  return in->act >= 0 && in->act <= 2 && (in->flags & ~ACCEL_B200_EP_TRIGGER_AFTER_WAIT) == 0;
}

// Zero-size products still define C: an empty sum is 0 before the epilogue.
__global__ void EmptySumKernel(float* c, int64_t ldc, int64_t m, int64_t n, Epilogue ep) {
  const int64_t total = m * n;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = idx / n, j = idx - i * n;
    c[i * ldc + j] = ApplyEpilogue(ep, 0.f, i, j);
  }
}

int EmptySum(float* c, int64_t ldc, int64_t m, int64_t n, const Epilogue& ep, cudaStream_t s) {
  const int grid = static_cast<int>(Min64(CeilDiv(m * n, 256), static_cast<int64_t>(kSms) * 8));
  EmptySumKernel<<<grid, 256, 0, s>>>(c, ldc, m, n, ep);
  return CheckLaunch("matmul_empty_k");
}

}  // namespace

// Tensor-core path (gemm_tc.cu).
bool TcEligible(const float* a, int64_t lda, const int8_t* w, int32_t axis, const int8_t* zero, int64_t m, int64_t k,
                int64_t n);
size_t TcWorkspace(int64_t m, int64_t k, int64_t n);
int RunTc(const float* a, const float* up, int64_t lda, const float* gamma, float eps, const int8_t* w,
          const float* scale, bool scalar_scale, float* c, int64_t ldc, int64_t m, int64_t k, int64_t n,
          const Epilogue& ep, void* workspace, size_t workspace_bytes, int32_t* status, cudaStream_t stream,
          const PeerOut* peers, const double* sq_in, int64_t sq_ld, int32_t sq_n, bool silu_pairs);
int LaunchRmsNormRows(const float* x, int64_t ldx, const float* w, float* y, int64_t ldy, int64_t rows, int64_t dim,
                      float eps, int64_t row_offset, cudaStream_t stream);
int LaunchSiluMulRows(const float* gate_up, int64_t ld, float* out, int64_t ldo, int64_t rows, int64_t inter,
                      cudaStream_t stream);

// GEMV for m <= 8 (gemv.cu).
bool GemvEligible(const float* a, int64_t lda, const int8_t* w, int32_t axis, const int8_t* zero, int64_t m,
                  int64_t k, int64_t n);
int RunGemv(const float* a, int64_t lda, const int8_t* w, const float* scale, bool scalar_scale, float* c,
            int64_t ldc, int64_t m, int64_t k, int64_t n, const Epilogue& ep, cudaStream_t stream,
            const PeerOut* peers);

namespace {
// 0: by shape (GEMV for m <= 8, tensor cores above), 1: CUDA cores,
// 2: tensor cores where eligible, 3: GEMV where eligible. Per thread: a
// choice made on one thread never changes the products another thread runs.
thread_local int g_q8_path = 0;

bool UseTc(const float* a, int64_t lda, const int8_t* w, int32_t axis, const int8_t* zero, int64_t m, int64_t k,
           int64_t n) {
  const int path = g_q8_path;
  if (path == 1 || path == 3) return false;
  return TcEligible(a, lda, w, axis, zero, m, k, n);
}

bool UseGemv(const float* a, int64_t lda, const int8_t* w, int32_t axis, const int8_t* zero, int64_t m, int64_t k,
             int64_t n) {
  const int path = g_q8_path;
  if (path == 1 || path == 2) return false;
  return GemvEligible(a, lda, w, axis, zero, m, k, n);
}
}  // namespace
}  // namespace accel_b200

namespace accel_b200 {
namespace {
int MatMulQ8(const float* a, int64_t lda, const accel_b200_q8_plane* b, float* c, int64_t ldc, int64_t m, int64_t k,
             int64_t n, const accel_b200_epilogue* ep, void* workspace, size_t workspace_bytes, void* stream,
             const PeerOut* peers) {
  if (m < 0 || k < 0 || n < 0 || b == nullptr) return SetError(ACCEL_B200_EINVAL, "quantized MatMul is out of range");
  if (b->axis < -1 || b->axis > 1 || b->offset < 0) return SetError(ACCEL_B200_EINVAL, "quantized MatMul: bad plane axis");
  GemmArgs g{};
  if (!ToEpilogue(ep, &g.ep)) return SetError(ACCEL_B200_EINVAL, "quantized MatMul: bad activation or flags");
  if (m == 0 || n == 0) return ClearError();
  if (c == nullptr || ldc < n) return SetError(ACCEL_B200_EINVAL, "quantized MatMul: bad output");
  const bool with_peers = peers != nullptr && peers->n > 0;
  if (k == 0 && !with_peers) return EmptySum(c, ldc, m, n, g.ep, AsStream(stream));
  if (a == nullptr || lda < k || b->q == nullptr || b->scale == nullptr) {
    return SetError(ACCEL_B200_EINVAL, "quantized MatMul is missing an operand");
  }
  const int8_t* w = b->q + b->offset;
  if (UseGemv(a, lda, w, b->axis, b->zero, m, k, n)) {
    return RunGemv(a, lda, w, b->scale, b->axis < 0, c, ldc, m, k, n, g.ep, AsStream(stream), peers);
  }
  if (UseTc(a, lda, w, b->axis, b->zero, m, k, n)) {
    return RunTc(a, nullptr, lda, nullptr, 0.f, w, b->scale, b->axis < 0, c, ldc, m, k, n, g.ep, workspace,
                 workspace_bytes, nullptr, AsStream(stream), peers, nullptr, 0, 0, false);
  }
  if (with_peers || g.ep.row_sq != nullptr) {
    return SetError(ACCEL_B200_EINVAL,
                    "matmul_q8: peer outputs and row sums of squares need the GEMV or tensor-core path "
                    "(per-column or single scale, no zero points, 16-byte aligned rows, k % 8 == 0 and n % 16 == 0 "
                    "above m = 8)");
  }
  g.a = a;
  g.lda = lda;
  g.w = w;
  g.scale = b->scale;
  g.zero = b->zero;
  g.axis = b->axis;
  g.c = c;
  g.ldc = ldc;
  g.m = m;
  g.k = k;
  g.n = n;
  return RunGemm<int8_t>(g, AsStream(stream), workspace, workspace_bytes);
}
}  // namespace
}  // namespace accel_b200

using namespace accel_b200;

extern "C" {

ACCEL_B200_API int accel_b200_matmul(const float* a, const float* b, float* c, int64_t m, int64_t k, int64_t n,
                                     void* stream) {
  if (m < 0 || k < 0 || n < 0) return SetError(ACCEL_B200_EINVAL, "MatMul is out of range");
  if (m == 0 || n == 0) return ClearError();
  if (c == nullptr || (k > 0 && (a == nullptr || b == nullptr))) return SetError(ACCEL_B200_EINVAL, "MatMul: null pointer");
  MatMulExactKernel<<<dim3(static_cast<unsigned>(CeilDiv(n, 128)), static_cast<unsigned>(m < 65535 ? m : 65535)), 128, 0,
                      AsStream(stream)>>>(a, b, c, m, k, n);
  return CheckLaunch("matmul_exact");
}

ACCEL_B200_API size_t accel_b200_matmul_q8_workspace(int64_t m, int64_t k, int64_t n) {
  // Enough for either path, so the caller need not know which one runs.
  const size_t simt = WorkspaceFor(true, m, k, n);
  const size_t tc = (m > 0 && k > 0 && n > 0) ? TcWorkspace(m, k, n) : 0;
  return simt > tc ? simt : tc;
}

ACCEL_B200_API int accel_b200_set_q8_path(int32_t path) {
  if (path < 0 || path > 3) {
    return SetError(ACCEL_B200_EINVAL, "set_q8_path: 0 (by shape), 1 (CUDA cores), 2 (tensor cores), 3 (GEMV)");
  }
  g_q8_path = path;
  return ClearError();
}

ACCEL_B200_API size_t accel_b200_matmul_f32_workspace(int64_t m, int64_t k, int64_t n) {
  return WorkspaceFor(false, m, k, n);
}


ACCEL_B200_API int accel_b200_matmul_q8(const float* a, int64_t lda, const accel_b200_q8_plane* b, float* c,
                                        int64_t ldc, int64_t m, int64_t k, int64_t n,
                                        const accel_b200_epilogue* ep, void* workspace, size_t workspace_bytes,
                                        void* stream) {
  return MatMulQ8(a, lda, b, c, ldc, m, k, n, ep, workspace, workspace_bytes, stream, nullptr);
}

ACCEL_B200_API int accel_b200_matmul_q8_peers(const float* a, int64_t lda, const accel_b200_q8_plane* b, float* c,
                                              int64_t ldc, int64_t m, int64_t k, int64_t n, float* const* peers,
                                              int32_t n_peers, const accel_b200_epilogue* ep, void* workspace,
                                              size_t workspace_bytes, void* stream) {
  if (n_peers < 0 || n_peers > kMaxPeers || (n_peers > 0 && peers == nullptr)) {
    return SetError(ACCEL_B200_EINVAL, "matmul_q8_peers: 0 to 7 peer outputs");
  }
  PeerOut p{};
  p.n = n_peers;
  for (int i = 0; i < n_peers; ++i) {
    if (peers[i] == nullptr) return SetError(ACCEL_B200_EINVAL, "matmul_q8_peers: null peer output");
    p.c[i] = peers[i];
  }
  return MatMulQ8(a, lda, b, c, ldc, m, k, n, ep, workspace, workspace_bytes, stream, &p);
}

ACCEL_B200_API size_t accel_b200_matmul_q8_silu_workspace(int64_t m, int64_t inter, int64_t n) {
  // The product's workspace, then room for the SiluMul rows when the product
  // runs on the CUDA cores (which read A from memory).
  const size_t base = (accel_b200_matmul_q8_workspace(m, inter, n) + 255) / 256 * 256;
  return base + static_cast<size_t>(m > 0 ? m : 0) * static_cast<size_t>(inter > 0 ? inter : 0) * sizeof(float);
}

ACCEL_B200_API int accel_b200_matmul_q8_silu(const float* gate_up, int64_t ld, int64_t inter,
                                             const accel_b200_q8_plane* b, float* c, int64_t ldc, int64_t m,
                                             int64_t n, const accel_b200_epilogue* ep, void* workspace,
                                             size_t workspace_bytes, void* stream) {
  if (m < 0 || inter < 0 || n < 0 || b == nullptr || ld < 2 * inter) {
    return SetError(ACCEL_B200_EINVAL, "quantized MatMul (SiluMul rows) is out of range");
  }
  if (b->axis < -1 || b->axis > 1 || b->offset < 0) return SetError(ACCEL_B200_EINVAL, "quantized MatMul: bad plane axis");
  Epilogue e{};
  if (!ToEpilogue(ep, &e)) return SetError(ACCEL_B200_EINVAL, "quantized MatMul: bad activation or flags");
  if (m == 0 || n == 0) return ClearError();
  if (c == nullptr || ldc < n) return SetError(ACCEL_B200_EINVAL, "quantized MatMul: bad output");
  if (inter == 0) return EmptySum(c, ldc, m, n, e, AsStream(stream));
  if (gate_up == nullptr || b->q == nullptr || b->scale == nullptr) {
    return SetError(ACCEL_B200_EINVAL, "quantized MatMul is missing an operand");
  }
  const size_t need = accel_b200_matmul_q8_silu_workspace(m, inter, n);
  if (workspace == nullptr || workspace_bytes < need) return SetError(ACCEL_B200_EINVAL, "matmul_q8_silu: workspace too small");
  const int8_t* w = b->q + b->offset;
  const float* up = gate_up + inter;
  if (inter % 4 == 0 && UseTc(gate_up, ld, w, b->axis, b->zero, m, inter, n) &&
      reinterpret_cast<uintptr_t>(up) % 16 == 0) {
    return RunTc(gate_up, up, ld, nullptr, 0.f, w, b->scale, b->axis < 0, c, ldc, m, inter, n, e, workspace,
                 workspace_bytes, nullptr, AsStream(stream), nullptr, nullptr, 0, 0, false);
  }
  // CUDA cores: SiluMul rows into the workspace's tail, then the product.
  const size_t base = need - static_cast<size_t>(m) * inter * sizeof(float);
  float* act = reinterpret_cast<float*>(static_cast<char*>(workspace) + base);
  const int rc = LaunchSiluMulRows(gate_up, ld, act, inter, m, inter, AsStream(stream));
  if (rc != ACCEL_B200_OK) return rc;
  return accel_b200_matmul_q8(act, inter, b, c, ldc, m, inter, n, ep, workspace, base, stream);
}

ACCEL_B200_API size_t accel_b200_matmul_q8_rmsnorm_workspace(int64_t m, int64_t k, int64_t n) {
  // The product's workspace, then room for the normalized rows when the
  // product runs on the CUDA cores.
  const size_t base = (accel_b200_matmul_q8_workspace(m, k, n) + 255) / 256 * 256;
  return base + static_cast<size_t>(m > 0 ? m : 0) * static_cast<size_t>(k > 0 ? k : 0) * sizeof(float);
}

static int MatMulQ8RmsNorm(const float* x, int64_t ldx, const double* sq, int64_t sq_ld, int32_t sq_n,
                           const float* gamma, float eps, const accel_b200_q8_plane* b, float* c, int64_t ldc,
                           int64_t m, int64_t k, int64_t n, const accel_b200_epilogue* ep, void* workspace,
                           size_t workspace_bytes, void* stream) {
  if (m < 0 || k < 0 || n < 0 || b == nullptr || ldx < k) {
    return SetError(ACCEL_B200_EINVAL, "quantized MatMul (RmsNorm rows) is out of range");
  }
  if (b->axis < -1 || b->axis > 1 || b->offset < 0) return SetError(ACCEL_B200_EINVAL, "quantized MatMul: bad plane axis");
  Epilogue e{};
  if (!ToEpilogue(ep, &e)) return SetError(ACCEL_B200_EINVAL, "quantized MatMul: bad activation or flags");
  if (m == 0 || n == 0) return ClearError();
  if (c == nullptr || ldc < n) return SetError(ACCEL_B200_EINVAL, "quantized MatMul: bad output");
  if (k == 0) return EmptySum(c, ldc, m, n, e, AsStream(stream));
  if (x == nullptr || gamma == nullptr || b->q == nullptr || b->scale == nullptr) {
    return SetError(ACCEL_B200_EINVAL, "quantized MatMul is missing an operand");
  }
  const size_t need = accel_b200_matmul_q8_rmsnorm_workspace(m, k, n);
  if (workspace == nullptr || workspace_bytes < need) {
    return SetError(ACCEL_B200_EINVAL, "matmul_q8_rmsnorm: workspace too small");
  }
  const int8_t* w = b->q + b->offset;
  if (UseTc(x, ldx, w, b->axis, b->zero, m, k, n) && reinterpret_cast<uintptr_t>(gamma) % 16 == 0) {
    return RunTc(x, nullptr, ldx, gamma, eps, w, b->scale, b->axis < 0, c, ldc, m, k, n, e, workspace,
                 workspace_bytes, nullptr, AsStream(stream), nullptr, sq, sq_ld, sq_n, false);
  }
  // CUDA cores: RmsNorm rows into the workspace's tail, then the product.
  const size_t base = need - static_cast<size_t>(m) * k * sizeof(float);
  float* act = reinterpret_cast<float*>(static_cast<char*>(workspace) + base);
  const int rc = LaunchRmsNormRows(x, ldx, gamma, act, k, m, k, eps, 0, AsStream(stream));
  if (rc != ACCEL_B200_OK) return rc;
  return accel_b200_matmul_q8(act, k, b, c, ldc, m, k, n, ep, workspace, base, stream);
}

ACCEL_B200_API int accel_b200_matmul_q8_rmsnorm(const float* x, int64_t ldx, const float* gamma, float eps,
                                                const accel_b200_q8_plane* b, float* c, int64_t ldc, int64_t m,
                                                int64_t k, int64_t n, const accel_b200_epilogue* ep, void* workspace,
                                                size_t workspace_bytes, void* stream) {
  return MatMulQ8RmsNorm(x, ldx, nullptr, 0, 0, gamma, eps, b, c, ldc, m, k, n, ep, workspace, workspace_bytes,
                         stream);
}

ACCEL_B200_API int accel_b200_matmul_q8_rmsnorm_stats(const float* x, int64_t ldx, const double* row_sq,
                                                      int64_t row_sq_ld, int32_t row_sq_n, const float* gamma,
                                                      float eps, const accel_b200_q8_plane* b, float* c, int64_t ldc,
                                                      int64_t m, int64_t k, int64_t n, const accel_b200_epilogue* ep,
                                                      void* workspace, size_t workspace_bytes, void* stream) {
  if (row_sq == nullptr || row_sq_n <= 0 || row_sq_ld < row_sq_n) {
    return SetError(ACCEL_B200_EINVAL, "matmul_q8_rmsnorm_stats: bad row sums of squares");
  }
  return MatMulQ8RmsNorm(x, ldx, row_sq, row_sq_ld, row_sq_n, gamma, eps, b, c, ldc, m, k, n, ep, workspace,
                         workspace_bytes, stream);
}

ACCEL_B200_API int accel_b200_matmul_q8_rmsnorm_silu_pairs(const float* x, int64_t ldx, const double* row_sq,
                                                           int64_t row_sq_ld, int32_t row_sq_n, const float* gamma,
                                                           float eps, const accel_b200_q8_plane* b, float* c,
                                                           int64_t ldc, int64_t m, int64_t k, int64_t n,
                                                           void* workspace, size_t workspace_bytes, void* stream) {
  if (m < 0 || k <= 0 || n <= 0 || n % 128 != 0 || b == nullptr || ldx < k || ldc < n / 2) {
    return SetError(ACCEL_B200_EINVAL, "matmul_q8_rmsnorm_silu_pairs: out of range (n must be a multiple of 128)");
  }
  if (row_sq != nullptr && (row_sq_n <= 0 || row_sq_ld < row_sq_n)) {
    return SetError(ACCEL_B200_EINVAL, "matmul_q8_rmsnorm_silu_pairs: bad row sums of squares");
  }
  if (m == 0) return ClearError();
  if (x == nullptr || gamma == nullptr || c == nullptr || b->q == nullptr || b->scale == nullptr) {
    return SetError(ACCEL_B200_EINVAL, "matmul_q8_rmsnorm_silu_pairs is missing an operand");
  }
  const int8_t* w = b->q + b->offset;
  if (b->offset < 0 || !TcEligible(x, ldx, w, b->axis, b->zero, m, k, n) ||
      reinterpret_cast<uintptr_t>(gamma) % 16 != 0) {
    return SetError(ACCEL_B200_EINVAL,
                    "matmul_q8_rmsnorm_silu_pairs: needs the tensor-core path (per-column or single scale, no zero "
                    "points, k % 8 == 0, 16-byte aligned rows and gamma)");
  }
  if (workspace == nullptr || workspace_bytes < accel_b200_matmul_q8_rmsnorm_workspace(m, k, n)) {
    return SetError(ACCEL_B200_EINVAL, "matmul_q8_rmsnorm_silu_pairs: workspace too small");
  }
  Epilogue e{};
  return RunTc(x, nullptr, ldx, gamma, eps, w, b->scale, b->axis < 0, c, ldc, m, k, n, e, workspace, workspace_bytes,
               nullptr, AsStream(stream), nullptr, row_sq, row_sq_ld, row_sq_n, true);
}

ACCEL_B200_API int accel_b200_matmul_f32(const float* a, int64_t lda, const float* b, float* c, int64_t ldc, int64_t m,
                                         int64_t k, int64_t n, const accel_b200_epilogue* ep, void* workspace,
                                         size_t workspace_bytes, void* stream) {
  if (m < 0 || k < 0 || n < 0) return SetError(ACCEL_B200_EINVAL, "MatMul is out of range");
  GemmArgs g{};
  if (!ToEpilogue(ep, &g.ep)) return SetError(ACCEL_B200_EINVAL, "MatMul: bad activation or flags");
  if (m == 0 || n == 0) return ClearError();
  if (c == nullptr || ldc < n) return SetError(ACCEL_B200_EINVAL, "MatMul: bad output");
  if (k == 0) return EmptySum(c, ldc, m, n, g.ep, AsStream(stream));
  if (a == nullptr || b == nullptr || lda < k) return SetError(ACCEL_B200_EINVAL, "MatMul is missing an operand");
  if (g.ep.row_sq != nullptr) return SetError(ACCEL_B200_EINVAL, "MatMul: row sums of squares need int8 weights");
  g.a = a;
  g.lda = lda;
  g.w = b;
  g.c = c;
  g.ldc = ldc;
  g.m = m;
  g.k = k;
  g.n = n;
  g.axis = -1;
  return RunGemm<float>(g, AsStream(stream), workspace, workspace_bytes);
}

}  // extern "C"
