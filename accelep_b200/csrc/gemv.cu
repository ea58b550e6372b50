// int8-weight GEMV for few rows (M <= 8): the decode-sized product
// C[m, n] = epilogue(scale[n] * sum_k A[m, k] * q[k, n]) with q int8 [k, n]
// (n contiguous, the reference's QuantPlane layout) and a per-column or single
// scale (src/sim_device.cc:541-602, the epilogue of src/runtime.cc:332-344).
//
// The weights are read once, at HBM speed: lane l of a warp owns CPL
// adjacent columns (16-, 8- or 4-byte loads, a warp reads 32 * CPL contiguous
// bytes of a k row) and keeps 8 k rows of loads in flight. int8 -> fp32 is
// exact (byte permute under the exponent of 2^23 + 128, then one fp32
// subtract); each output accumulates fp32 fused multiply-adds over its k
// slice, and the column scale multiplies the sum once, as the tensor-core
// path does. The A rows are read as warp-wide broadcasts.
//
// K is split: the 8 warps of a CTA take 8 consecutive k slices of the same
// column strip, and up to 8 CTAs of one thread-block cluster take 8 more
// each. The slices are summed warp by warp in shared memory, then rank by
// rank through distributed shared memory, always in the same order, so the
// result does not depend on scheduling. One launch, no workspace.
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string>

#include "accel_b200.h"
#include "cluster.cuh"
#include "common.cuh"

namespace accel_b200 {
namespace {

constexpr int kGvWarps = 8;
constexpr int kGvThreads = kGvWarps * 32;
constexpr int kGvUnroll = 8;  // k rows per load batch

struct GemvArgs {
  const float* a;
  int64_t lda;
  const int8_t* w;
  const float* scale;
  int32_t scalar_scale;
  float* c;
  int64_t ldc;
  int64_t m, k, n;
  int64_t k_per_slice;  // multiple of kGvUnroll
  int32_t vec_store;
  Epilogue ep;
  PeerOut peers;  // copies of C on other GPUs (n = 0: none)
};

template <int CPL>
struct WRow;
template <>
struct WRow<16> {
  uint4 v;
  __device__ __forceinline__ void Load(const int8_t* p) { v = __ldg(reinterpret_cast<const uint4*>(p)); }
  __device__ __forceinline__ uint32_t Word(int i) const { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }
};
template <>
struct WRow<8> {
  uint2 v;
  __device__ __forceinline__ void Load(const int8_t* p) { v = __ldg(reinterpret_cast<const uint2*>(p)); }
  __device__ __forceinline__ uint32_t Word(int i) const { return i == 0 ? v.x : v.y; }
};
template <>
struct WRow<4> {
  uint32_t v;
  __device__ __forceinline__ void Load(const int8_t* p) { v = __ldg(reinterpret_cast<const uint32_t*>(p)); }
  __device__ __forceinline__ uint32_t Word(int) const { return v; }
};

// Four int8 in a word -> four exact floats: XOR 0x80 gives q + 128, a byte
// permute places it under the fp32 exponent of 2^23 (the float 2^23 + 128 +
// q), and subtracting 2^23 + 128 leaves q.
__device__ __forceinline__ void Int8x4ToF32(uint32_t w, float* f) {
  const uint32_t u = w ^ 0x80808080u;
  f[0] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650)) - 8388736.0f;
  f[1] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7651)) - 8388736.0f;
  f[2] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7652)) - 8388736.0f;
  f[3] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7653)) - 8388736.0f;
}

template <int MT, int CPL>
__global__ void __launch_bounds__(kGvThreads) Q8GemvKernel(GemvArgs g) {
  constexpr int SW = 32 * CPL;  // columns per CTA
  extern __shared__ __align__(16) float red[];  // [kGvWarps][MT][SW], then the CTA sum [MT][SW]
  float* cta_sum = red + kGvWarps * MT * SW;
  // The next kernel may launch at once, or (TRIGGER_AFTER_WAIT) only after
  // this CTA has waited for the previous kernel.
  const bool late = (g.ep.flags & ACCEL_B200_EP_TRIGGER_AFTER_WAIT) != 0;
  if (!late) PdlTrigger();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rank = static_cast<int>(blockIdx.y), splits = static_cast<int>(gridDim.y);
  const int64_t strip0 = static_cast<int64_t>(blockIdx.x) * SW;
  const int64_t col0 = strip0 + lane * CPL;
  const int64_t row0 = static_cast<int64_t>(blockIdx.z) * MT;
  const int rows = static_cast<int>(Min64(MT, g.m - row0));
  const int64_t kb = static_cast<int64_t>(rank * kGvWarps + warp) * g.k_per_slice;
  const int64_t ke = Min64(g.k, kb + g.k_per_slice);
  float acc[MT][CPL];
#pragma unroll
  for (int r = 0; r < MT; ++r)
#pragma unroll
    for (int c = 0; c < CPL; ++c) acc[r][c] = 0.f;
  PdlWait();  // A comes from an earlier kernel
  if (late) PdlTrigger();
  if (col0 < g.n) {
    // Two register buffers: the loads of batch i + 1 are in flight while batch
    // i is converted and accumulated.
    const int8_t* wp = g.w + kb * g.n + col0;
    WRow<CPL> wa[kGvUnroll], wb[kGvUnroll];
    float xa[MT][kGvUnroll], xb[MT][kGvUnroll];
    auto load = [&](int64_t k, WRow<CPL>(&wr)[kGvUnroll], float(&x)[MT][kGvUnroll]) {
      const int nk = static_cast<int>(Min64(kGvUnroll, ke - k));
      const int8_t* p = wp + (k - kb) * g.n;
#pragma unroll
      for (int u = 0; u < kGvUnroll; ++u) {
        if (u < nk) {
          wr[u].Load(p + u * g.n);
        } else {
          wr[u].v = {};
        }
      }
#pragma unroll
      for (int r = 0; r < MT; ++r) {
        const float* ar = g.a + (row0 + (r < rows ? r : 0)) * g.lda + k;
        if (nk == kGvUnroll) {
          const float4 x0 = __ldg(reinterpret_cast<const float4*>(ar));
          const float4 x1 = __ldg(reinterpret_cast<const float4*>(ar + 4));
          x[r][0] = x0.x; x[r][1] = x0.y; x[r][2] = x0.z; x[r][3] = x0.w;
          x[r][4] = x1.x; x[r][5] = x1.y; x[r][6] = x1.z; x[r][7] = x1.w;
        } else {
#pragma unroll
          for (int u = 0; u < kGvUnroll; ++u) x[r][u] = u < nk ? __ldg(ar + u) : 0.f;
        }
        if (r >= rows) {
#pragma unroll
          for (int u = 0; u < kGvUnroll; ++u) x[r][u] = 0.f;
        }
      }
    };
    auto compute = [&](const WRow<CPL>(&wr)[kGvUnroll], const float(&x)[MT][kGvUnroll]) {
#pragma unroll
      for (int u = 0; u < kGvUnroll; ++u) {
        float q[CPL];
#pragma unroll
        for (int i = 0; i < CPL / 4; ++i) Int8x4ToF32(wr[u].Word(i), q + 4 * i);
#pragma unroll
        for (int r = 0; r < MT; ++r)
#pragma unroll
          for (int c = 0; c < CPL; ++c) acc[r][c] = fmaf(x[r][u], q[c], acc[r][c]);
      }
    };
    // Rows past the slice load as zero weights and zero A, adding nothing.
    int64_t k = kb;
    if (k < ke) load(k, wa, xa);
    while (k < ke) {
      if (k + kGvUnroll < ke) load(k + kGvUnroll, wb, xb);
      compute(wa, xa);
      k += kGvUnroll;
      if (k >= ke) break;
      if (k + kGvUnroll < ke) load(k + kGvUnroll, wa, xa);
      compute(wb, xb);
      k += kGvUnroll;
    }
  }
  // Warp partials -> shared memory; the CTA sums them warp by warp in order.
#pragma unroll
  for (int r = 0; r < MT; ++r)
#pragma unroll
    for (int c = 0; c < CPL; c += 4)
      *reinterpret_cast<float4*>(red + (warp * MT + r) * SW + lane * CPL + c) =
          make_float4(acc[r][c], acc[r][c + 1], acc[r][c + 2], acc[r][c + 3]);
  __syncthreads();
  for (int e = tid * 4; e < MT * SW; e += kGvThreads * 4) {
    float4 s = *reinterpret_cast<const float4*>(red + e);
#pragma unroll
    for (int w = 1; w < kGvWarps; ++w) {
      const float4 v = *reinterpret_cast<const float4*>(red + w * MT * SW + e);
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
    *reinterpret_cast<float4*>(cta_sum + e) = s;
  }
  if (splits > 1) {
    ClusterSync();  // every rank's CTA sum is complete
  } else {
    __syncthreads();
  }
  // Rank `rank` finishes groups of four outputs rank, rank + splits, ...: the
  // CTA sums of ranks 0, 1, ... added in order, then scale and epilogue.
  for (int grp = rank * kGvThreads + tid; grp < MT * SW / 4; grp += splits * kGvThreads) {
    const int r = grp / (SW / 4), cl = (grp % (SW / 4)) * 4;
    const int64_t col = strip0 + cl;
    float4 s;
    if (splits > 1) {
      s = LoadPeer4(cta_sum + r * SW + cl, 0u);
      for (int p = 1; p < splits; ++p) {
        const float4 v = LoadPeer4(cta_sum + r * SW + cl, static_cast<uint32_t>(p));
        s.x += v.x;
        s.y += v.y;
        s.z += v.z;
        s.w += v.w;
      }
    } else {
      s = *reinterpret_cast<const float4*>(cta_sum + r * SW + cl);
    }
    double sq = 0.0;
    if (r < rows && col < g.n) {
      const int64_t row = row0 + r;
      const float v[4] = {s.x, s.y, s.z, s.w};
      float o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float scq = g.scalar_scale ? __ldg(g.scale) : (col + q < g.n ? __ldg(g.scale + col + q) : 0.f);
        o[q] = ApplyEpilogue(g.ep, __fmul_rn(v[q], scq), row, col + q);
      }
      const int64_t off = row * g.ldc + col;
      float* dst = g.c + off;
      if (g.vec_store && col + 4 <= g.n) {
        *reinterpret_cast<float4*>(dst) = make_float4(o[0], o[1], o[2], o[3]);
        StorePeers4(g.peers, off, make_float4(o[0], o[1], o[2], o[3]));
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (col + q < g.n) {
            dst[q] = o[q];
            StorePeers(g.peers, off + q, o[q]);
          }
        }
      }
      if (g.ep.row_sq != nullptr) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (col + q < g.n) {
            const double dv = static_cast<double>(o[q]);
            sq = fma(dv, dv, sq);  // one fused multiply-add, as every kernel that writes row sums does
          }
        }
      }
    }
    if (g.ep.row_sq != nullptr) {
      // The 32 lanes of a warp hold 32 consecutive groups: one 128-column
      // block of row r (SW is a multiple of 128).
      sq = WarpSum(sq);
      if (lane == 0 && r < rows) g.ep.row_sq[(row0 + r) * g.ep.row_sq_ld + col / 128] = sq;
    }
  }
  if (g.peers.n > 0) __threadfence_system();  // peer copies land before the kernel completes
  if (splits > 1) ClusterSync();  // no CTA leaves while a peer may still read its sum
}

struct GvPlan {
  int mt, cpl, splits;
  int64_t strips, row_tiles, k_per_slice;
};

GvPlan MakeGvPlan(int64_t m, int64_t k, int64_t n) {
  GvPlan p{};
  p.mt = m <= 1 ? 1 : m <= 2 ? 2 : m <= 4 ? 4 : 8;
  // Widest loads that still give about one CTA per SM once K is split 8 ways.
  const int max_cpl = p.mt <= 4 ? 16 : 8;
  p.cpl = max_cpl;
  while (p.cpl > 4 && CeilDiv(n, 32 * p.cpl) * 8 < kSms) p.cpl /= 2;
  if (n % p.cpl != 0) p.cpl = 4;
  p.strips = CeilDiv(n, 32 * p.cpl);
  p.row_tiles = CeilDiv(m, p.mt);
  const int64_t base = p.strips * p.row_tiles;
  // Cluster ranks: enough CTAs for about two per SM, each warp >= 64 k rows.
  int64_t splits = CeilDiv(2 * kSms, base);
  splits = Min64(splits, Max64(1, k / (kGvWarps * 64)));
  p.splits = static_cast<int>(Max64(1, Min64(splits, 8)));
  p.k_per_slice = CeilDiv(CeilDiv(k, static_cast<int64_t>(p.splits) * kGvWarps), kGvUnroll) * kGvUnroll;
  return p;
}

template <int MT, int CPL>
int LaunchGv(const GemvArgs& g, const GvPlan& p, cudaStream_t s) {
  constexpr size_t smem = static_cast<size_t>(kGvWarps + 1) * MT * 32 * CPL * sizeof(float);
  static std::once_flag once[16];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 15], [] {
    cudaFuncSetAttribute(Q8GemvKernel<MT, CPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  });
  const dim3 grid(static_cast<unsigned>(p.strips), static_cast<unsigned>(p.splits),
                  static_cast<unsigned>(p.row_tiles));
  return CheckLaunchEx(LaunchK(Q8GemvKernel<MT, CPL>, grid, dim3(kGvThreads), smem, s, 1u,
                               static_cast<unsigned>(p.splits), g),
                       "matmul_q8_gemv");
}

}  // namespace

// Whether the GEMV takes this product: m <= 8, a per-column or single scale
// without zero points, n a multiple of 4, 16-byte aligned A rows and weights.
bool GemvEligible(const float* a, int64_t lda, const int8_t* w, int32_t axis, const int8_t* zero, int64_t m,
                  int64_t k, int64_t n) {
  if (zero != nullptr || (axis != 1 && axis != -1)) return false;
  if (m <= 0 || m > 8 || k <= 0 || n <= 0 || n % 4 != 0 || lda % 4 != 0) return false;
  if (reinterpret_cast<uintptr_t>(a) % 16 != 0 || reinterpret_cast<uintptr_t>(w) % 16 != 0) return false;
  return CeilDiv(n, 128) <= 2147483647LL;
}

int RunGemv(const float* a, int64_t lda, const int8_t* w, const float* scale, bool scalar_scale, float* c,
            int64_t ldc, int64_t m, int64_t k, int64_t n, const Epilogue& ep, cudaStream_t stream,
            const PeerOut* peers) {
  const GvPlan p = MakeGvPlan(m, k, n);
  GemvArgs g{};
  g.a = a;
  g.lda = lda;
  g.w = w;
  g.scale = scale;
  g.scalar_scale = scalar_scale ? 1 : 0;
  g.c = c;
  g.ldc = ldc;
  g.m = m;
  g.k = k;
  g.n = n;
  g.k_per_slice = p.k_per_slice;
  g.vec_store = (reinterpret_cast<uintptr_t>(c) % 16 == 0 && ldc % 4 == 0) ? 1 : 0;
  g.ep = ep;
  g.peers = peers != nullptr ? *peers : PeerOut{};
  for (int i = 0; i < g.peers.n; ++i) {
    if (reinterpret_cast<uintptr_t>(g.peers.c[i]) % 16 != 0) g.vec_store = 0;
  }
  switch (p.mt * 100 + p.cpl) {
    case 116: return LaunchGv<1, 16>(g, p, stream);
    case 108: return LaunchGv<1, 8>(g, p, stream);
    case 104: return LaunchGv<1, 4>(g, p, stream);
    case 216: return LaunchGv<2, 16>(g, p, stream);
    case 208: return LaunchGv<2, 8>(g, p, stream);
    case 204: return LaunchGv<2, 4>(g, p, stream);
    case 416: return LaunchGv<4, 16>(g, p, stream);
    case 408: return LaunchGv<4, 8>(g, p, stream);
    case 404: return LaunchGv<4, 4>(g, p, stream);
    case 808: return LaunchGv<8, 8>(g, p, stream);
    default: return LaunchGv<8, 4>(g, p, stream);
  }
}

}  // namespace accel_b200
