// int8-weight product on the 5th-generation tensor cores (tcgen05).
//
// C[m, n] = epilogue(scale[n] * sum_k A[m, k] * q[k, n]) with A fp32 [m, k] and q
// int8 [k, n] (n contiguous: the reference's QuantPlane layout) and a
// per-column (or single) scale: src/sim_device.cc:541-602 and the epilogue of
// src/runtime.cc:332-344.
//
// Operand preparation happens in shared memory, per 64-deep k block:
//  * q: int8 -> bf16 is exact (|q| <= 128 needs 8 significant bits), stored
//    n-contiguous ("MN-major") in the 128-byte-swizzled canonical layout.
//  * A: each fp32 value is split into three bf16 terms hi + mid + lo (each
//    the rounded remainder of the previous), which carry the 24-bit fp32
//    significand; products with the exact bf16 weight are exact, so three
//    MMAs accumulating in fp32 reproduce the fp32 product to within the fp32
//    accumulation error.
// The MMA is issued "swapped": its M = 128 runs over output features (the
// weight tile) and its N = R over activation rows, so decode with 32 rows is a
// full-width MMA. D lives in TMEM (R fp32 columns); four warps read it back
// with tcgen05.ld, one output feature per thread, and store rows coalesced.
// K can be split across CTAs; each split writes a partial tile and the last
// CTA of a tile sums the partials in split order, so the result does not
// depend on arrival order.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "accel_b200.h"
#include "common.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace accel_b200 {

namespace {

constexpr int kTcThreads = 128;
constexpr int kBk = 64;                     // k per block: 128 bytes of bf16, one swizzle row
constexpr int kBn = 128;                    // output features per tile (MMA M)
constexpr int kATile = kBn * kBk * 2;       // 16 KB
constexpr int kMmaK = 16;                   // k per bf16 MMA

struct TcArgs {
  const float* a;
  int64_t lda;
  const int8_t* w;
  const float* scale;
  int32_t scalar_scale;
  float* c;
  int64_t ldc;
  int64_t m, k, n;
  int32_t kb_total;
  int32_t kb_per_split;
  float* part;        // [splits][m][n] raw sums, splits > 1
  int32_t* counters;  // [row tiles][feature tiles]; zero before and after
  int32_t* status;
  Epilogue ep;
};

template <int R>
struct TcLayout {
  static constexpr int kBTile = R * kBk * 2;  // one bf16 term of the activations
  static constexpr int kStage = kATile + 3 * kBTile;
  static constexpr int kSmem = 2 * kStage + 1024;  // + slack to 1024-align the base
};

__device__ __forceinline__ uint32_t PackBf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Weight block [64 k x 128 n] -> bf16, n-contiguous, 128-byte swizzle. Atom
// (k / 8, n / 64) of 8 k rows x 128 bytes sits at (k/8) * 2048 + (n/64) * 1024;
// the 16-byte chunk (n % 64) / 8 of row k % 8 is stored at chunk ^ (k % 8).
__device__ __forceinline__ void LoadWeightBlock(const TcArgs& g, uint8_t* a_tile, int64_t k0, int64_t n0, int tid) {
#pragma unroll
  for (int pass = 0; pass < 4; ++pass) {
    const int idx = pass * kTcThreads + tid;
    const int kl = idx >> 3;
    const int nl = (idx & 7) * 16;
    const int64_t gk = k0 + kl, gn = n0 + nl;
    int8_t q[16];
    if (gk < g.k && gn + 16 <= g.n) {
      *reinterpret_cast<int4*>(q) = __ldg(reinterpret_cast<const int4*>(g.w + gk * g.n + gn));
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) q[i] = (gk < g.k && gn + i < g.n) ? g.w[gk * g.n + gn + i] : 0;
    }
    uint32_t packed[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) packed[i] = PackBf16(static_cast<float>(q[2 * i]), static_cast<float>(q[2 * i + 1]));
    const int row = kl & 7;
    uint8_t* atom = a_tile + (kl >> 3) * 2048 + (nl >> 6) * 1024 + row * 128;
    const int chunk = (nl & 63) >> 3;
    *reinterpret_cast<uint4*>(atom + (((chunk) ^ row) << 4)) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    *reinterpret_cast<uint4*>(atom + (((chunk + 1) ^ row) << 4)) = make_uint4(packed[4], packed[5], packed[6], packed[7]);
  }
}

// Activation block [R rows x 64 k] -> three bf16 terms, k-contiguous, 128-byte
// swizzle: row r at (r / 8) * 1024 + (r % 8) * 128, chunk (k / 8) ^ (r % 8).
template <int R>
__device__ __forceinline__ void LoadActBlock(const TcArgs& g, uint8_t* b_tiles, int64_t row0, int64_t k0, int tid) {
  constexpr int kBTile = TcLayout<R>::kBTile;
#pragma unroll
  for (int pass = 0; pass < R / 8; ++pass) {
    const int idx = pass * kTcThreads + tid;
    const int rl = idx >> 4;
    const int kl = (idx & 15) * 4;
    const int64_t gr = row0 + rl, gk = k0 + kl;
    float x[4];
    if (gr < g.m && gk + 4 <= g.k) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(g.a + gr * g.lda + gk));
      x[0] = v.x;
      x[1] = v.y;
      x[2] = v.z;
      x[3] = v.w;
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) x[i] = (gr < g.m && gk + i < g.k) ? g.a[gr * g.lda + gk + i] : 0.f;
    }
    float hi[4], mid[4], lo[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      hi[i] = __bfloat162float(__float2bfloat16_rn(x[i]));
      const float r1 = x[i] - hi[i];
      mid[i] = __bfloat162float(__float2bfloat16_rn(r1));
      lo[i] = r1 - mid[i];
    }
    const int row = rl & 7;
    const int off = (rl >> 3) * 1024 + row * 128 + ((((kl >> 3) ^ row)) << 4) + (kl & 7) * 2;
    *reinterpret_cast<uint2*>(b_tiles + off) = make_uint2(PackBf16(hi[0], hi[1]), PackBf16(hi[2], hi[3]));
    *reinterpret_cast<uint2*>(b_tiles + kBTile + off) = make_uint2(PackBf16(mid[0], mid[1]), PackBf16(mid[2], mid[3]));
    *reinterpret_cast<uint2*>(b_tiles + 2 * kBTile + off) = make_uint2(PackBf16(lo[0], lo[1]), PackBf16(lo[2], lo[3]));
  }
}

template <int R>
__global__ void __launch_bounds__(kTcThreads, 1) Q8GemmTcKernel(TcArgs g) {
  using L = TcLayout<R>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t mma_bar[2];
  __shared__ uint32_t tmem_base_s;
  __shared__ int32_t last_s;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t raw_addr = SmemAddr(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023) & ~1023u) - raw_addr);
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * kBn;
  const int64_t row0 = static_cast<int64_t>(blockIdx.z) * R;
  const int kb_begin = blockIdx.y * g.kb_per_split;
  const int kb_end = min(g.kb_total, kb_begin + g.kb_per_split);
  const int nkb = max(0, kb_end - kb_begin);
  constexpr uint32_t kCols = R < 32 ? 32 : R;
  constexpr uint32_t kIdesc = InstrDescBf16(R, true);

  if (warp == 0) TmemAlloc(&tmem_base_s, kCols);
  if (tid == 0) {
    MbarInit(&mma_bar[0], 1);
    MbarInit(&mma_bar[1], 1);
    FenceBarrierInit();
  }
  TcFenceBeforeSync();
  __syncthreads();
  TcFenceAfterSync();
  const uint32_t tmem = tmem_base_s;
  bool ok = true;

  for (int i = 0; i < nkb; ++i) {
    const int s = i & 1;
    uint8_t* stage = smem + s * L::kStage;
    if (i >= 2) ok &= MbarWait(&mma_bar[s], ((i >> 1) - 1) & 1);  // the MMAs that read this stage are done
    const int64_t k0 = static_cast<int64_t>(kb_begin + i) * kBk;
    LoadWeightBlock(g, stage, k0, n0, tid);
    LoadActBlock<R>(g, stage + kATile, row0, k0, tid);
    FenceProxyAsyncSmem();
    __syncthreads();
    if (tid == 0) {
      TcFenceAfterSync();
      const uint32_t a_addr = SmemAddr(stage);
      const uint32_t b_addr = a_addr + kATile;
#pragma unroll
      for (int ks = 0; ks < kBk / kMmaK; ++ks) {
        // A: two k atoms (16 k) per MMA, 4096 bytes; n atoms 1024 apart (LBO),
        // k atoms 2048 apart (SBO). B: 32 bytes of k per MMA inside the
        // swizzled row; 8-row groups 1024 apart (SBO).
        const uint64_t adesc = SmemDescSw128(a_addr + ks * 4096, 1024, 2048);
#pragma unroll
        for (int part = 0; part < 3; ++part) {
          const uint64_t bdesc = SmemDescSw128(b_addr + part * L::kBTile + ks * 32, 16, 1024);
          MmaBf16(tmem, adesc, bdesc, kIdesc, (i | ks | part) != 0);
        }
      }
      MmaCommit(&mma_bar[s]);
    }
  }
  if (nkb > 0) ok &= MbarWait(&mma_bar[(nkb - 1) & 1], ((nkb - 1) >> 1) & 1);
  if (!__syncthreads_and(ok)) {
    // A wait ran out: report it, give the tensor core one more bounded wait
    // before the TMEM is released, and leave the output untouched.
    if (tid == 0 && g.status != nullptr) atomicOr(g.status, ACCEL_B200_STATUS_COPY_TIMEOUT);
    if (nkb > 0) MbarWait(&mma_bar[(nkb - 1) & 1], ((nkb - 1) >> 1) & 1);
    TcFenceBeforeSync();
    __syncthreads();
    if (warp == 0) TmemDealloc(tmem, kCols);
    return;
  }
  TcFenceAfterSync();

  const int64_t gn = n0 + warp * 32 + lane;
  const bool col_ok = gn < g.n;
  const float sc = g.scalar_scale ? __ldg(g.scale) : (col_ok ? __ldg(g.scale + gn) : 0.f);
  const bool split = gridDim.y > 1;
#pragma unroll
  for (int c0 = 0; c0 < R; c0 += 32) {
    float v[32];
    if (nkb > 0) {
      TmemLoad32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + c0, v);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = 0.f;
    }
    if (!col_ok) continue;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int64_t row = row0 + c0 + j;
      if (row >= g.m) break;
      if (split) {
        g.part[(static_cast<int64_t>(blockIdx.y) * g.m + row) * g.n + gn] = v[j];
      } else {
        g.c[row * g.ldc + gn] = ApplyEpilogue(g.ep, __fmul_rn(v[j], sc), row, gn);
      }
    }
  }
  TcFenceBeforeSync();
  __syncthreads();
  if (warp == 0) TmemDealloc(tmem, kCols);
  if (!split) return;

  // Split K: the last CTA of this tile sums the partials in split order.
  __threadfence();
  __syncthreads();
  int32_t* counter = g.counters + static_cast<int64_t>(blockIdx.z) * gridDim.x + blockIdx.x;
  if (tid == 0) last_s = atomicAdd(counter, 1) == static_cast<int32_t>(gridDim.y) - 1;
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  const int64_t rows = Min64(R, g.m - row0);
  const int64_t cols = Min64(kBn, g.n - n0);
  for (int64_t idx = tid; idx < rows * cols; idx += kTcThreads) {
    const int64_t row = row0 + idx / cols, col = n0 + idx % cols;
    float sum = 0.f;
    for (int p = 0; p < static_cast<int>(gridDim.y); ++p) sum += __ldcg(g.part + (p * g.m + row) * g.n + col);
    const float s2 = g.scalar_scale ? __ldg(g.scale) : __ldg(g.scale + col);
    g.c[row * g.ldc + col] = ApplyEpilogue(g.ep, __fmul_rn(sum, s2), row, col);
  }
  if (tid == 0) *counter = 0;
}

struct TcPlan {
  int r;
  int64_t feature_tiles, row_tiles;
  int32_t kb_total, kb_per_split, splits;
  size_t counter_bytes, part_bytes;
};

TcPlan MakeTcPlan(int64_t m, int64_t k, int64_t n) {
  TcPlan p{};
  p.r = m <= 32 ? 32 : (m <= 64 ? 64 : 128);
  p.feature_tiles = CeilDiv(n, kBn);
  p.row_tiles = CeilDiv(m, p.r);
  p.kb_total = static_cast<int32_t>(CeilDiv(k, kBk));
  const int64_t base = p.feature_tiles * p.row_tiles;
  int64_t want = CeilDiv(2 * kSms, base);
  if (want > p.kb_total) want = p.kb_total;
  if (want < 1 || base > kMaxCounters) want = 1;  // split K needs one counter per tile
  p.kb_per_split = static_cast<int32_t>(CeilDiv(p.kb_total, want));
  p.splits = static_cast<int32_t>(CeilDiv(p.kb_total, p.kb_per_split));
  p.counter_bytes = kCounterRegion;
  p.part_bytes = p.splits > 1 ? static_cast<size_t>(p.splits) * m * n * sizeof(float) : 0;
  return p;
}

template <int R>
int LaunchTc(const TcArgs& g, const TcPlan& p, cudaStream_t s) {
  static std::once_flag once[16];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 15], [] {
    cudaFuncSetAttribute(Q8GemmTcKernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcLayout<R>::kSmem);
  });
  Q8GemmTcKernel<R><<<dim3(static_cast<unsigned>(p.feature_tiles), static_cast<unsigned>(p.splits),
                           static_cast<unsigned>(p.row_tiles)),
                      kTcThreads, TcLayout<R>::kSmem, s>>>(g);
  return CheckLaunch("matmul_q8_tc");
}

}  // namespace

// Whether the tensor-core path takes this product: a per-column or single
// scale without zero points, 16-byte aligned rows of A and of the weight.
bool TcEligible(const float* a, int64_t lda, const int8_t* w, int32_t axis, const int8_t* zero, int64_t m, int64_t k,
                int64_t n) {
  if (zero != nullptr || (axis != 1 && axis != -1)) return false;
  if (m <= 0 || k <= 0 || n <= 0 || n % 16 != 0 || lda % 4 != 0) return false;
  if (reinterpret_cast<uintptr_t>(a) % 16 != 0 || reinterpret_cast<uintptr_t>(w) % 16 != 0) return false;
  const int64_t row_tiles = CeilDiv(m, m <= 32 ? 32 : (m <= 64 ? 64 : 128));
  return row_tiles <= 65535 && CeilDiv(n, kBn) <= 2147483647LL;
}

size_t TcWorkspace(int64_t m, int64_t k, int64_t n) {
  const TcPlan p = MakeTcPlan(m, k, n);
  return p.counter_bytes + p.part_bytes;
}

int RunTc(const float* a, int64_t lda, const int8_t* w, const float* scale, bool scalar_scale, float* c, int64_t ldc,
          int64_t m, int64_t k, int64_t n, const Epilogue& ep, void* workspace, size_t workspace_bytes,
          int32_t* status, cudaStream_t stream) {
  const TcPlan p = MakeTcPlan(m, k, n);
  if (workspace == nullptr || workspace_bytes < p.counter_bytes + p.part_bytes) {
    return SetError(ACCEL_B200_EINVAL, "matmul_q8: workspace too small");
  }
  TcArgs g{};
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
  g.kb_total = p.kb_total;
  g.kb_per_split = p.kb_per_split;
  g.counters = static_cast<int32_t*>(workspace);
  g.part = p.part_bytes > 0 ? reinterpret_cast<float*>(static_cast<char*>(workspace) + p.counter_bytes) : nullptr;
  g.status = status;
  g.ep = ep;
  switch (p.r) {
    case 32: return LaunchTc<32>(g, p, stream);
    case 64: return LaunchTc<64>(g, p, stream);
    default: return LaunchTc<128>(g, p, stream);
  }
}

}  // namespace accel_b200
