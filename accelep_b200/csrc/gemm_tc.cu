// int8-weight product on the 5th-generation tensor cores (tcgen05), fed by TMA.
//
// C[m, n] = epilogue(scale[n] * sum_k A[m, k] * q[k, n]) with A fp32 [m, k], q int8
// [k, n] (n contiguous: the reference's QuantPlane layout) and a per-column
// (or single) scale: src/sim_device.cc:541-602 and the epilogue of
// src/runtime.cc:332-344. A may also be SiluMul of a fused gate|up row
// (src/sim_silu.cc:8-13 then the down projection, src/llama_model.cc:239-240).
//
// Arithmetic. int8 -> bf16 is exact (|q| <= 128 needs 8 significant bits).
// Each fp32 activation is split into three bf16 planes hi + mid + lo (each the
// rounded remainder of the previous); together they carry the 24-bit fp32
// significand, every product with the bf16 weight is exact, and the planes
// accumulate separately in fp32 in TMEM. The MMA is issued "swapped": M = 128
// runs over output features and N over activation rows (all three planes in
// one MMA of N = 3R when 3R <= 256), so decode with 32 rows is a full-width MMA.
//
// Activation operand, by mode:
//   planes  (m > 64): a separate pass writes the three planes [3][m][k] to the
//           workspace; TMA loads them with 128-byte swizzle, which is already
//           the MMA's K-major canonical layout.
//   fp32    (m <= 64): TMA loads the fp32 tile [R rows x 64 k]; the converter
//           warps split it into the planes in shared memory.
//   silu    (m <= 64): TMA loads the gate and up tiles; the converter warps form
//           silu(g) * u exactly as SiluMul rounds it and split the result.
//
// Pipeline (one CTA = one 128-feature x R-row tile over a range of 64-deep k
// blocks; 6 warps):
//   warp 0  producer: per k block one TMA of the raw int8 weight block
//           [64 k x 128 n] and the activation load(s) of the mode; a ring of
//           stages.
//   warps 2-5 converters: int8 -> bf16 (integer and fp32-add bit arithmetic,
//           exact) into the MMA's n-contiguous swizzled layout (two buffers),
//           and the split of fp32 activations; afterwards the epilogue:
//           tcgen05.ld of the accumulator into a shared tile, then scale,
//           fused epilogue and coalesced row stores.
//   warp 1  MMA issuer (one thread): 4 k steps per block, then tcgen05.commit
//           to the barriers that free the stage and the buffer.
// K can be split across the CTAs of one thread-block cluster (up to 8); each
// keeps its partial tile in shared memory and the cluster sums the tiles in
// rank order through distributed shared memory, so the result is
// deterministic and no partial sums go to global memory.
//
// Launch overlap: the kernel is launched with programmatic stream
// serialization. Before griddepcontrol.wait it only sets up barriers and TMEM
// and loads weights (immutable); activations, residuals and the output are
// touched after it. Every mbarrier wait is bounded (tma.cuh).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string>

#include "accel_b200.h"
#include "cluster.cuh"
#include "common.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace accel_b200 {

namespace {

constexpr int kBk = 64;                // k per block: 128 bytes of bf16, one swizzle row
constexpr int kBn = 128;               // output features per tile (MMA M)
constexpr int kMmaK = 16;              // k per bf16 MMA
constexpr int kWRaw = kBk * kBn;       // raw int8 weight block, 8 KiB
constexpr int kWConv = kBk * kBn * 2;  // converted bf16 weight block, 16 KiB
constexpr int kConvBufs = 2;
constexpr int kConvWarps = 4;
constexpr int kThreads = (2 + kConvWarps) * 32;
constexpr int kMaxStages = 4;

enum AMode : int { kAPlanes = 0, kAF32 = 1, kASilu = 2, kANorm = 3 };

template <int R, int S, int M>
struct Tc {
  static constexpr int kXBytes = 3 * R * kBk * 2;  // three bf16 planes (MMA operand)
  static constexpr int kXRaw = M == kAPlanes ? 0 : (M == kASilu ? 2 : 1) * R * kBk * 4;  // fp32 tiles
  static constexpr int kXLoad = M == kAPlanes ? kXBytes : kXRaw;  // bytes the activation TMA delivers
  static constexpr int kStage = kXBytes + kWRaw + kXRaw;          // planes first: 1024-aligned
  static constexpr int kStages = S;
  static constexpr int kTile = R * kBn * 4;  // fp32 accumulator tile, staged in stage memory
  static constexpr int kStageArea = kStages * kStage > kTile ? kStages * kStage : kTile;
  static constexpr int kSmem = kStageArea + kConvBufs * kWConv + 1024;
  static_assert(kStages <= kMaxStages, "stage count");
  static_assert(kStage % 1024 == 0, "stage alignment");
  static_assert(kSmem <= 227 * 1024, "shared memory");
};

struct TcArgs {
  const float* a;      // fp32 A rows (norm mode: the whole rows are read for their RMS)
  int64_t lda;
  const float* gamma;  // norm mode: RmsNorm weights [k]
  float eps;
  const double* sq_in;  // norm mode, optional: per row, sq_n partial sums of squares (stride sq_ld)
  int64_t sq_ld;
  int32_t sq_n;
  int64_t m, k, n;
  int32_t kb_total;
  int32_t kb_per_split;
  const float* scale;
  int32_t scalar_scale;
  float* c;
  int64_t ldc;
  int32_t* status;
  int32_t vec_store;  // c and ldc allow 16-byte row stores
  Epilogue ep;
  PeerOut peers;  // copies of C on other GPUs (n = 0: none)
};

__device__ __forceinline__ void TmaLoad2D(void* dst, const CUtensorMap* map, int32_t x, int32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          SmemAddr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(SmemAddr(bar))
      : "memory");
}

__device__ __forceinline__ void TmaLoad3D(void* dst, const CUtensorMap* map, int32_t x, int32_t y, int32_t z,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          SmemAddr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(SmemAddr(bar))
      : "memory");
}

__device__ __forceinline__ void TmemLoadCols(uint32_t taddr, float (&v)[32]) { TmemLoad32(taddr, v); }
__device__ __forceinline__ void TmemLoadCols(uint32_t taddr, float (&v)[16]) { TmemLoad16(taddr, v); }

__device__ __forceinline__ uint32_t PackBf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Four int8 in a word -> two bf16x2 words, exactly and with full-rate integer
// and fp32 adds only: XOR 0x80 turns each byte into q + 128 (offset binary);
// a byte permute places it under the fp32 exponent of 2^23, so the float is
// 2^23 + 128 + q; subtracting 2^23 + 128 leaves q exactly, and an integer-valued
// float of at most 8 significant bits has a zero low half, so its top 16 bits
// are the bf16 encoding.
__device__ __forceinline__ void Int8x4ToBf16(uint32_t w, uint32_t* lo, uint32_t* hi) {
  const uint32_t u = w ^ 0x80808080u;
  const float f0 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650)) - 8388736.0f;
  const float f1 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7651)) - 8388736.0f;
  const float f2 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7652)) - 8388736.0f;
  const float f3 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7653)) - 8388736.0f;
  *lo = __byte_perm(__float_as_uint(f0), __float_as_uint(f1), 0x7632);
  *hi = __byte_perm(__float_as_uint(f2), __float_as_uint(f3), 0x7632);
}

// Raw weight block [64 k][128 n] int8 (dense rows of 128 bytes) -> bf16 in the
// n-contiguous 128-byte-swizzled layout: atom (k / 8, n / 64) of 8 k rows x 128
// bytes at (k / 8) * 2048 + (n / 64) * 1024; 16-byte chunk (n % 64) / 8 of row
// k % 8 stored at chunk ^ (k % 8).
__device__ __forceinline__ void ConvertWeightBlock(const uint8_t* raw, uint8_t* conv, int ct) {
#pragma unroll
  for (int pass = 0; pass < 4; ++pass) {
    const int idx = pass * (kConvWarps * 32) + ct;
    const int kl = idx >> 3;
    const int nl = (idx & 7) * 16;
    const uint4 q = *reinterpret_cast<const uint4*>(raw + kl * kBn + nl);
    uint32_t p[8];
    Int8x4ToBf16(q.x, &p[0], &p[1]);
    Int8x4ToBf16(q.y, &p[2], &p[3]);
    Int8x4ToBf16(q.z, &p[4], &p[5]);
    Int8x4ToBf16(q.w, &p[6], &p[7]);
    const int row = kl & 7;
    uint8_t* atom = conv + (kl >> 3) * 2048 + (nl >> 6) * 1024 + row * 128;
    const int chunk = (nl & 63) >> 3;
    *reinterpret_cast<uint4*>(atom + ((chunk ^ row) << 4)) = make_uint4(p[0], p[1], p[2], p[3]);
    *reinterpret_cast<uint4*>(atom + (((chunk + 1) ^ row) << 4)) = make_uint4(p[4], p[5], p[6], p[7]);
  }
}

// hi = bf16(x), mid = bf16(x - hi), lo = bf16(x - hi - mid).
__device__ __forceinline__ void Split3(float x, float* hi, float* mid, float* lo) {
  *hi = __bfloat162float(__float2bfloat16_rn(x));
  const float r1 = x - *hi;
  *mid = __bfloat162float(__float2bfloat16_rn(r1));
  *lo = r1 - *mid;
}

// SiluMul of one element as src/sim_silu.cc:8-13 rounds it.
__device__ __forceinline__ float SiluMul(float g, float u) {
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, expf(-g))), u);
}

// fp32 activation tile(s) [R rows][64 k] (rows of 256 bytes) -> the three bf16
// planes in the K-major 128-byte-swizzled layout the planes TMA would write:
// plane p, row r at p * R * 128 + r * 128, 16-byte chunk j stored at
// j ^ (r % 8). Each thread takes four consecutive k of one row per pass.
// Rows at or past `valid` are skipped: their planes stay zero. Norm mode: the
// element is RmsNorm'd first, float(double(x) * inv[row]) * gamma[k], as
// RmsNormKernel rounds it (gamma points at this block's first k; `kvalid` k
// of the block lie inside the matrix).
template <int R, int M>
__device__ __forceinline__ void SplitTile(const uint8_t* raw, uint8_t* planes, int ct, int valid,
                                          const float* gamma, int kvalid, const double* inv) {
#pragma unroll
  for (int pass = 0; pass < R * 16 / (kConvWarps * 32); ++pass) {
    const int idx = pass * (kConvWarps * 32) + ct;
    const int row = idx >> 4, k4 = idx & 15;
    if (pass * (kConvWarps * 32) >= valid * 16) break;  // uniform across the CTA
    if (row >= valid) continue;
    float x[4];
    const float4 v = *reinterpret_cast<const float4*>(raw + row * 256 + k4 * 16);
    if constexpr (M == kASilu) {
      const float4 u = *reinterpret_cast<const float4*>(raw + R * 256 + row * 256 + k4 * 16);
      x[0] = SiluMul(v.x, u.x);
      x[1] = SiluMul(v.y, u.y);
      x[2] = SiluMul(v.z, u.z);
      x[3] = SiluMul(v.w, u.w);
    } else if constexpr (M == kANorm) {
      const float4 w = k4 * 4 < kvalid ? __ldg(reinterpret_cast<const float4*>(gamma + k4 * 4))
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
      const double iv = inv[row];
      x[0] = __fmul_rn(static_cast<float>(static_cast<double>(v.x) * iv), w.x);
      x[1] = __fmul_rn(static_cast<float>(static_cast<double>(v.y) * iv), w.y);
      x[2] = __fmul_rn(static_cast<float>(static_cast<double>(v.z) * iv), w.z);
      x[3] = __fmul_rn(static_cast<float>(static_cast<double>(v.w) * iv), w.w);
    } else {
      x[0] = v.x;
      x[1] = v.y;
      x[2] = v.z;
      x[3] = v.w;
    }
    float h[4], md[4], lo[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) Split3(x[j], &h[j], &md[j], &lo[j]);
    const int off = row * 128 + (((k4 >> 1) ^ (row & 7)) << 4) + (k4 & 1) * 8;
    *reinterpret_cast<uint2*>(planes + off) = make_uint2(PackBf16(h[0], h[1]), PackBf16(h[2], h[3]));
    *reinterpret_cast<uint2*>(planes + R * 128 + off) = make_uint2(PackBf16(md[0], md[1]), PackBf16(md[2], md[3]));
    *reinterpret_cast<uint2*>(planes + 2 * R * 128 + off) = make_uint2(PackBf16(lo[0], lo[1]), PackBf16(lo[2], lo[3]));
  }
}

// 1 / sqrt(mean(x^2) + eps) of a row in double, summed exactly as
// RmsNormKernel sums it (lane-strided partial sums, then a butterfly), so the
// normalized values are bit-identical to that kernel's.
__device__ __forceinline__ double RowInverseRms(const float* in, int64_t dim, float eps, int lane) {
  double sq = 0.0;
#pragma unroll 6
  for (int64_t i = lane; i < dim; i += 32) {
    const double v = static_cast<double>(in[i]);
    sq += v * v;
  }
  sq = WarpSum(sq);
  return 1.0 / sqrt(sq / static_cast<double>(dim) + static_cast<double>(eps));
}

// The same inverse RMS for rows [0, valid) of a tile, all rows at once: four
// converter threads per row (ct = 4 * row + q) and the same arithmetic order.
// RmsNormKernel's lane l sums x[l + 32 i] over i ascending and the 32 partial
// sums combine in a butterfly (xor 16, 8, 4, 2, 1; each level a + b in either
// order, which is exact-commutative). Here thread q holds the partials of
// lanes 8q .. 8q + 7, so levels 16 and 8 are shuffles with threads q ^ 2 and
// q ^ 1 and levels 4, 2, 1 stay inside the thread. dim % 8 == 0.
template <int R>
__device__ __forceinline__ void TileInverseRms(const float* a, int64_t lda, int64_t row0, int valid, int64_t dim,
                                               float eps, int ct, double* inv) {
  for (int base = 0; base < R; base += kConvWarps * 8) {
    const int r = base + (ct >> 2), q = ct & 3;
    double s[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j] = 0.0;
    if (r < valid) {
      const float* in = a + (row0 + r) * lda + 8 * q;
#pragma unroll 9
      for (int64_t i0 = 0; i0 + 8 * q < dim; i0 += 32) {
        const float4 x0 = __ldg(reinterpret_cast<const float4*>(in + i0));
        const float4 x1 = __ldg(reinterpret_cast<const float4*>(in + i0 + 4));
        const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const double v = static_cast<double>(xs[j]);
          s[j] += v * v;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j] += __shfl_xor_sync(kFull, s[j], 2);  // lane l ^ 16
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j] += __shfl_xor_sync(kFull, s[j], 1);  // lane l ^ 8
    const double u0 = s[0] + s[4], u1 = s[1] + s[5], u2 = s[2] + s[6], u3 = s[3] + s[7];  // l ^ 4
    const double sum = (u0 + u2) + (u1 + u3);                                             // l ^ 2, l ^ 1
    if (r < valid && q == 0) inv[r] = 1.0 / sqrt(sum / static_cast<double>(dim) + static_cast<double>(eps));
  }
}

// R = 16 planes kernels (long weight streams, m <= 16) run three CTAs per SM.
template <int R, int kStagesT, int M>
__global__ void __launch_bounds__(kThreads, (R == 16 && M == kAPlanes) ? 3 : 1)
    Q8GemmTcKernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx,
                   const __grid_constant__ CUtensorMap tu, TcArgs g) {
  using L = Tc<R, kStagesT, M>;
  constexpr int S = L::kStages;
  // The three activation planes are 3R consecutive K-major rows in shared
  // memory: one MMA with N = 3R covers all of them when 3R <= 256 and reads the
  // weight operand once; D column p * R + r then holds plane p of row r.
  constexpr bool kOneMma = 3 * R <= 256;
  constexpr uint32_t kCols = 3 * R <= 64 ? 64 : (3 * R <= 128 ? 128 : (3 * R <= 256 ? 256 : 512));
  constexpr uint32_t kIdesc = InstrDescBf16(kOneMma ? 3 * R : R, true);
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_w[kMaxStages], full_x[kMaxStages], empty[kMaxStages], cfull[kConvBufs],
      cempty[kConvBufs], accf;
  __shared__ uint32_t tmem_s;
  __shared__ double inv_s[M == kANorm ? R : 1];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t raw_addr = SmemAddr(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023) & ~1023u) - raw_addr);
  uint8_t* conv_base = smem + L::kStageArea;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * kBn;
  const int64_t row0 = static_cast<int64_t>(blockIdx.z) * R;
  const int kb_begin = blockIdx.y * g.kb_per_split;
  const int nkb = max(0, min(g.kb_total, kb_begin + g.kb_per_split) - kb_begin);

  PdlTrigger();
  if (warp == 1) TmemAlloc(&tmem_s, kCols);
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      MbarInit(&full_w[s], 1);
      MbarInit(&full_x[s], 1);
      MbarInit(&empty[s], 1 + kConvWarps);
    }
    for (int c = 0; c < kConvBufs; ++c) {
      MbarInit(&cfull[c], kConvWarps);
      MbarInit(&cempty[c], 1);
    }
    MbarInit(&accf, 1);
    FenceBarrierInit();
  }
  TcFenceBeforeSync();
  __syncthreads();
  TcFenceAfterSync();
  const uint32_t tmem = tmem_s;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tw)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tx)) : "memory");
      // Weights of the first stages before the wait: they are immutable.
      const int pre = min(S, nkb);
      for (int i = 0; i < pre; ++i) {
        MbarArriveExpectTx(&full_w[i], kWRaw);
        TmaLoad2D(smem + i * L::kStage + L::kXBytes, &tw, static_cast<int32_t>(n0), (kb_begin + i) * kBk, &full_w[i]);
      }
      PdlWait();
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S;
        uint8_t* stage = smem + s * L::kStage;
        const int32_t k0 = (kb_begin + i) * kBk;
        if (i >= S) {
          ok &= MbarWait(&empty[s], ((i / S) & 1) ^ 1);
          MbarArriveExpectTx(&full_w[s], kWRaw);
          TmaLoad2D(stage + L::kXBytes, &tw, static_cast<int32_t>(n0), k0, &full_w[s]);
        }
        MbarArriveExpectTx(&full_x[s], L::kXLoad);
        if constexpr (M == kAPlanes) {
          TmaLoad3D(stage, &tx, k0, static_cast<int32_t>(row0), 0, &full_x[s]);
        } else {
          uint8_t* xraw = stage + L::kXBytes + kWRaw;
          TmaLoad2D(xraw, &tx, k0, static_cast<int32_t>(row0), &full_x[s]);
          if constexpr (M == kASilu) TmaLoad2D(xraw + R * 256, &tu, k0, static_cast<int32_t>(row0), &full_x[s]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S, c = i % kConvBufs;
        if constexpr (M == kAPlanes) ok &= MbarWait(&full_x[s], (i / S) & 1);
        ok &= MbarWait(&cfull[c], (i / kConvBufs) & 1);
        TcFenceAfterSync();
        const uint32_t a_addr = SmemAddr(conv_base + c * kWConv);
        const uint32_t b_addr = SmemAddr(smem + s * L::kStage);
#pragma unroll
        for (int ks = 0; ks < kBk / kMmaK; ++ks) {
          // A (weights, n-contiguous): 16 k = two k atoms = 4096 bytes per step;
          // n atoms 1024 apart (LBO), k atoms 2048 apart (SBO). B (planes,
          // k-contiguous): 32 bytes of k per step inside the swizzled row;
          // 8-row groups 1024 apart (SBO); planes R * 128 bytes apart.
          const uint64_t adesc = SmemDescSw128(a_addr + ks * 4096, 1024, 2048);
          if constexpr (kOneMma) {
            MmaBf16(tmem, adesc, SmemDescSw128(b_addr + ks * 32, 16, 1024), kIdesc, (i | ks) != 0);
          } else {
#pragma unroll
            for (int p = 0; p < 3; ++p) {
              const uint64_t bdesc = SmemDescSw128(b_addr + p * R * 128 + ks * 32, 16, 1024);
              MmaBf16(tmem + p * R, adesc, bdesc, kIdesc, (i | ks) != 0);
            }
          }
        }
        MmaCommit(&empty[s]);
        MmaCommit(&cempty[c]);
      }
      if (nkb > 0) MmaCommit(&accf);
    }
  } else {
    const int ct = tid - 64;
    const int valid = static_cast<int>(Min64(R, g.m - row0));
    if constexpr (M != kAPlanes) {
      // Rows past the matrix: zero planes in every stage, written once.
      if (valid < R) {
        for (int s = 0; s < S; ++s) {
          uint8_t* planes = smem + s * L::kStage;
          for (int idx = ct; idx < 3 * (R - valid) * 8; idx += kConvWarps * 32) {
            const int p = idx / ((R - valid) * 8), rem = idx % ((R - valid) * 8);
            *reinterpret_cast<uint4*>(planes + p * R * 128 + (valid + rem / 8) * 128 + (rem % 8) * 16) =
                make_uint4(0, 0, 0, 0);
          }
        }
      }
    }
    // The first weight blocks (one per conversion buffer) are converted before
    // anything waits for the activations: the weights are immutable, so this
    // overlaps the previous kernel, and after the activations land only the
    // split stands between them and the MMA.
    const int pre = min(kConvBufs, nkb);
    for (int i = 0; i < pre; ++i) {
      ok &= MbarWait(&full_w[i % S], (i / S) & 1);
      ConvertWeightBlock(smem + (i % S) * L::kStage + L::kXBytes, conv_base + i * kWConv, ct);
    }
    if constexpr (M == kANorm) {
      // Row RMS of the valid rows: from the producer's sums of squares when
      // given, else from the whole rows of A.
      PdlWait();
      if (g.sq_in != nullptr) {
        if (ct < valid) {
          const double* p = g.sq_in + (row0 + ct) * g.sq_ld;
          double sum = 0.0;
          for (int t = 0; t < g.sq_n; ++t) sum += p[t];
          inv_s[ct] = 1.0 / sqrt(sum / static_cast<double>(g.k) + static_cast<double>(g.eps));
        }
      } else {
        TileInverseRms<R>(g.a, g.lda, row0, valid, g.k, g.eps, ct, inv_s);
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kConvWarps * 32) : "memory");  // converter warps only
    }
    for (int i = 0; i < nkb; ++i) {
      const int s = i % S, c = i % kConvBufs;
      uint8_t* stage = smem + s * L::kStage;
      if (i >= pre) {
        ok &= MbarWait(&full_w[s], (i / S) & 1);
        ok &= MbarWait(&cempty[c], ((i / kConvBufs) & 1) ^ 1);
        ConvertWeightBlock(stage + L::kXBytes, conv_base + c * kWConv, ct);
      }
      if constexpr (M != kAPlanes) {
        ok &= MbarWait(&full_x[s], (i / S) & 1);
        const int64_t k0 = static_cast<int64_t>(kb_begin + i) * kBk;
        SplitTile<R, M>(stage + L::kXBytes + kWRaw, stage, ct, valid, M == kANorm ? g.gamma + k0 : nullptr,
                        static_cast<int>(Min64(kBk, g.k - k0)), inv_s);
      }
      FenceProxyAsyncSmem();
      __syncwarp();
      if (lane == 0) {
        MbarArrive(&cfull[c]);
        MbarArrive(&empty[s]);
      }
    }
    if (nkb > 0) ok &= MbarWait(&accf, 0);
  }
  // Every thread past this point may read the residual or write the output.
  PdlWait();
  const bool cta_ok = __syncthreads_and(ok);
  if (!cta_ok) {
    // A wait ran out: report it and let the tensor core finish (bounded). The
    // CTA still takes part in the cluster barriers below, so that no peer
    // waits for it. Unsplit, its tile is not written; split, its partial tile
    // is NaN, so the tile it feeds is NaN.
    if (tid == 0 && g.status != nullptr) atomicOr(g.status, ACCEL_B200_STATUS_COPY_TIMEOUT);
    if (nkb > 0) MbarWait(&accf, 0);
  }
  TcFenceAfterSync();
  // Split K runs as one thread-block cluster along grid y; every CTA of the
  // cluster holds its partial tile in shared memory and the cluster sums the
  // tiles in rank order (deterministic) through distributed shared memory.
  const int splits = static_cast<int>(gridDim.y);
  const int64_t rows = Min64(R, g.m - row0);
  const int64_t cols = Min64(kBn, g.n - n0);
  float* tile = reinterpret_cast<float*>(smem);  // [R][128] fp32; the stage memory is idle now
  if (warp >= 2) {
    const int quarter = warp & 3;  // TMEM lanes 32 * quarter .. +31
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    constexpr int kChunk = R < 32 ? R : 32;  // TMEM columns per load
#pragma unroll 1
    for (int c0 = 0; c0 < R; c0 += kChunk) {
      float v[kChunk];
      if (nkb > 0 && cta_ok) {
        // hi + mid + lo, each accumulated separately over K.
        float w[kChunk];
        TmemLoadCols(lane_base + c0, v);
        TmemLoadCols(lane_base + R + c0, w);
#pragma unroll
        for (int j = 0; j < kChunk; ++j) v[j] += w[j];
        TmemLoadCols(lane_base + 2 * R + c0, w);
#pragma unroll
        for (int j = 0; j < kChunk; ++j) v[j] += w[j];
      } else {
#pragma unroll
        for (int j = 0; j < kChunk; ++j) v[j] = cta_ok ? 0.f : __int_as_float(0x7fc00000);
      }
#pragma unroll
      for (int j = 0; j < kChunk; ++j) tile[(c0 + j) * kBn + quarter * 32 + lane] = v[j];
    }
  }
  TcFenceBeforeSync();
  __syncthreads();
  if (warp == 1) TmemDealloc(tmem, kCols);
  if (splits == 1) {
    // Thread t < 128 owns column t of the tile for every row.
    if (cta_ok && tid < cols) {
      const int64_t col = n0 + tid;
      const float sc = g.scalar_scale ? __ldg(g.scale) : __ldg(g.scale + col);
      if (g.peers.n == 0 && g.ep.row_sq == nullptr) {
        // The common case, kept free of the optional outputs (a loop over peers
        // inside this loop measured 30% slower on prefill-sized tiles).
#pragma unroll 4
        for (int64_t r = 0; r < rows; ++r) {
          const int64_t row = row0 + r;
          g.c[row * g.ldc + col] = ApplyEpilogue(g.ep, __fmul_rn(tile[r * kBn + tid], sc), row, col);
        }
      } else {
        for (int64_t r = 0; r < rows; ++r) {
          const int64_t row = row0 + r;
          const float o = ApplyEpilogue(g.ep, __fmul_rn(tile[r * kBn + tid], sc), row, col);
          g.c[row * g.ldc + col] = o;
          StorePeers(g.peers, row * g.ldc + col, o);
          if (g.ep.row_sq != nullptr) tile[r * kBn + tid] = o;
        }
      }
    }
    if (g.peers.n > 0) __threadfence_system();
    if (g.ep.row_sq != nullptr) {
      // Sums of squares of this tile's outputs per row: warp w of the first
      // four takes rows w, w + 4, ...; lane l the columns 4l .. 4l + 3.
      __syncthreads();
      if (tid < 128 && cta_ok) {
        for (int r = warp; r < rows; r += 4) {
          double sq = 0.0;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if (lane * 4 + q < cols) {
              const double v = static_cast<double>(tile[r * kBn + lane * 4 + q]);
              sq += v * v;
            }
          }
          sq = WarpSum(sq);
          if (lane == 0) g.ep.row_sq[(row0 + r) * g.ep.row_sq_ld + n0 / kBn] = sq;
        }
      }
    }
    return;
  }
  // Rank `rank` sums rows [rank * rpr, +rpr) of the tile over the cluster; a
  // thread owns one group of four columns (tid % 32) in rows tid / 32, + 6, ...
  const int rank = static_cast<int>(blockIdx.y);  // cluster (1, splits, 1): rank = y
  const int rpr = (static_cast<int>(rows) + splits - 1) / splits;
  const int c4 = (tid & 31) * 4;
  const int r_begin = rank * rpr + (tid >> 5);
  const int r_end = min(static_cast<int>(rows), (rank + 1) * rpr);
  constexpr int kMaxJ = (R / 2 + kThreads / 32 - 1) / (kThreads / 32);  // rows per thread (splits >= 2)
  float sc[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    sc[j] = (c4 + j < cols) ? (g.scalar_scale ? __ldg(g.scale) : __ldg(g.scale + n0 + c4 + j)) : 0.f;
  }
  ClusterSync();  // every partial tile of the cluster is complete
  float4 sum[kMaxJ];
  if (c4 < cols) {
#pragma unroll
    for (int j = 0; j < kMaxJ; ++j) {
      const int r = r_begin + j * (kThreads / 32);
      if (r < r_end) {
        // Summed over ranks 0, 1, ... in order: the result does not depend on
        // which rank finished first.
        const float* src = tile + r * kBn + c4;
        float4 part[8];
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (q < splits) part[q] = LoadPeer4(src, static_cast<uint32_t>(q));
        float4 acc = part[0];
#pragma unroll
        for (int q = 1; q < 8; ++q) {
          if (q < splits) {
            acc.x += part[q].x;
            acc.y += part[q].y;
            acc.z += part[q].z;
            acc.w += part[q].w;
          }
        }
        sum[j] = acc;
      }
    }
  }
  // This CTA has read what it needs from its peers: arrive now, and wait for
  // the peers' reads of this CTA's tile only before leaving.
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
#pragma unroll
  for (int j = 0; j < kMaxJ; ++j) {
    const int r = r_begin + j * (kThreads / 32);  // the same for the 32 lanes of a warp
    if (r < r_end) {
      double sq = 0.0;
      if (c4 < cols) {
        const int64_t row = row0 + r;
        const float v[4] = {sum[j].x, sum[j].y, sum[j].z, sum[j].w};
        float o[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) o[q] = ApplyEpilogue(g.ep, __fmul_rn(v[q], sc[q]), row, n0 + c4 + q);
        if (g.ep.row_sq != nullptr) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if (c4 + q < cols) {
              const double dv = static_cast<double>(o[q]);
              sq += dv * dv;
            }
          }
        }
        const int64_t off = row * g.ldc + n0 + c4;
        float* dst = g.c + off;
        if (g.vec_store && c4 + 4 <= cols) {
          *reinterpret_cast<float4*>(dst) = make_float4(o[0], o[1], o[2], o[3]);
          StorePeers4(g.peers, off, make_float4(o[0], o[1], o[2], o[3]));
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if (c4 + q < cols) {
              dst[q] = o[q];
              StorePeers(g.peers, off + q, o[q]);
            }
          }
        }
      }
      if (g.ep.row_sq != nullptr) {  // the warp holds the row's 128 columns of this tile
        sq = WarpSum(sq);
        if (lane == 0) g.ep.row_sq[(row0 + r) * g.ep.row_sq_ld + n0 / kBn] = sq;
      }
    }
  }
  if (g.peers.n > 0) __threadfence_system();  // peer copies land before the kernel completes
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");  // peers are done with this tile
}

// fp32 [m, k] (row stride lda) -> three bf16 planes [3][m][k] (Split3). With
// `up` set, the element is SiluMul(a[r][i], up[r][i]) first.
__global__ void SplitPlanesKernel(const float* __restrict__ a, const float* __restrict__ up, int64_t lda, int64_t m,
                                  int64_t k, __nv_bfloat16* __restrict__ planes) {
  PdlTrigger();
  PdlWait();
  const int64_t quads = k / 4;
  const int64_t total = m * quads;
  const int64_t plane = m * k;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = idx / quads, q = idx - r * quads;
    const float4 v = __ldg(reinterpret_cast<const float4*>(a + r * lda + q * 4));
    float x[4] = {v.x, v.y, v.z, v.w};
    if (up != nullptr) {
      const float4 u = __ldg(reinterpret_cast<const float4*>(up + r * lda + q * 4));
      x[0] = SiluMul(x[0], u.x);
      x[1] = SiluMul(x[1], u.y);
      x[2] = SiluMul(x[2], u.z);
      x[3] = SiluMul(x[3], u.w);
    }
    float hi[4], mid[4], lo[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) Split3(x[i], &hi[i], &mid[i], &lo[i]);
    const int64_t off = r * k + q * 4;
    *reinterpret_cast<uint2*>(planes + off) = make_uint2(PackBf16(hi[0], hi[1]), PackBf16(hi[2], hi[3]));
    *reinterpret_cast<uint2*>(planes + plane + off) = make_uint2(PackBf16(mid[0], mid[1]), PackBf16(mid[2], mid[3]));
    *reinterpret_cast<uint2*>(planes + 2 * plane + off) = make_uint2(PackBf16(lo[0], lo[1]), PackBf16(lo[2], lo[3]));
  }
}

// RmsNorm rows then split: one warp per row computes the row's inverse RMS as
// RmsNormKernel does and writes the three planes of float(double(x) * inv) * w.
__global__ void SplitPlanesNormKernel(const float* __restrict__ a, int64_t lda, const float* __restrict__ gamma,
                                      float eps, int64_t m, int64_t k, __nv_bfloat16* __restrict__ planes) {
  PdlTrigger();
  PdlWait();
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t plane = m * k;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < m; r += warps) {
    const float* in = a + r * lda;
    const double iv = RowInverseRms(in, k, eps, lane);
    for (int64_t q = lane; q < k / 4; q += 32) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(in + q * 4));
      const float4 w = __ldg(reinterpret_cast<const float4*>(gamma + q * 4));
      const float x[4] = {__fmul_rn(static_cast<float>(static_cast<double>(v.x) * iv), w.x),
                          __fmul_rn(static_cast<float>(static_cast<double>(v.y) * iv), w.y),
                          __fmul_rn(static_cast<float>(static_cast<double>(v.z) * iv), w.z),
                          __fmul_rn(static_cast<float>(static_cast<double>(v.w) * iv), w.w)};
      float hi[4], mid[4], lo[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) Split3(x[i], &hi[i], &mid[i], &lo[i]);
      const int64_t off = r * k + q * 4;
      *reinterpret_cast<uint2*>(planes + off) = make_uint2(PackBf16(hi[0], hi[1]), PackBf16(hi[2], hi[3]));
      *reinterpret_cast<uint2*>(planes + plane + off) =
          make_uint2(PackBf16(mid[0], mid[1]), PackBf16(mid[2], mid[3]));
      *reinterpret_cast<uint2*>(planes + 2 * plane + off) =
          make_uint2(PackBf16(lo[0], lo[1]), PackBf16(lo[2], lo[3]));
    }
  }
}

struct TcPlan {
  int r;
  int mode;  // AMode
  int stages;
  int64_t feature_tiles, row_tiles;
  int32_t kb_total, kb_per_split, splits;
  size_t planes_bytes;
};

// Stages that fit the shared memory of one CTA (at most 4).
template <int R, int M>
constexpr int MaxStages() {
  constexpr int stage = 3 * R * kBk * 2 + kWRaw + (M == kAPlanes ? 0 : (M == kASilu ? 2 : 1) * R * kBk * 4);
  return stage * 4 + kConvBufs * kWConv + 1024 <= 227 * 1024 ? 4 : 3;
}

// Activation rows per tile (the MMA's N is three times this).
int64_t TileRows(int64_t m) { return m <= 16 ? 16 : (m <= 32 ? 32 : (m <= 64 ? 64 : 128)); }

TcPlan MakeTcPlan(int64_t m, int64_t k, int64_t n, bool silu, bool norm) {
  TcPlan p{};
  p.r = static_cast<int>(TileRows(m));
  p.feature_tiles = CeilDiv(n, kBn);
  p.row_tiles = CeilDiv(m, p.r);
  p.kb_total = static_cast<int32_t>(CeilDiv(k, kBk));
  // When the tile grid is smaller than the GPU, split K across a cluster of up
  // to 8 CTAs, aiming at about two CTAs per SM and at least two k blocks per
  // CTA (a CTA's hand-offs per k block, not bandwidth, bound small products).
  const int64_t base = p.feature_tiles * p.row_tiles;
  int64_t splits = 1;
  if (base < kSms && p.kb_total > 1) {
    // R = 16 tiles run three CTAs per SM: the largest split whose grid fits
    // in one wave of them.
    splits = Min64(CeilDiv(p.kb_total, 2), p.r == 16 ? (3 * kSms) / base : CeilDiv(2 * kSms, base));
    if (splits > 8) splits = 8;
  }
  p.kb_per_split = static_cast<int32_t>(CeilDiv(p.kb_total, splits));
  p.splits = static_cast<int32_t>(CeilDiv(p.kb_total, p.kb_per_split));
  p.stages = p.kb_per_split <= 2 ? 2 : 4;  // 4: as many as fit (MaxStages, or fewer for more CTAs per SM)
  // Splitting fp32 tiles in the kernel saves the planes pass (one launch) but
  // adds converter work to every k block: worth it for CTAs that walk few
  // blocks (latency-bound decode products), not for long weight streams.
  p.mode = p.r == 128 || p.kb_per_split > 4 ? kAPlanes : (silu ? kASilu : (norm ? kANorm : kAF32));
  p.planes_bytes = p.mode == kAPlanes ? (static_cast<size_t>(3) * m * k * 2 + 1023) / 1024 * 1024 : 0;
  return p;
}

PFN_cuTensorMapEncodeTiled_v12000 EncodeFn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      ptr = nullptr;
    }
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }();
  return fn;
}

template <int R, int ST, int M>
int LaunchTc(const CUtensorMap& tw, const CUtensorMap& tx, const CUtensorMap& tu, const TcArgs& g, const TcPlan& p,
             cudaStream_t s) {
  using L = Tc<R, ST, M>;
  static std::once_flag once[16];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 15], [] {
    cudaFuncSetAttribute(Q8GemmTcKernel<R, ST, M>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmem);
  });
  const dim3 grid(static_cast<unsigned>(p.feature_tiles), static_cast<unsigned>(p.splits),
                  static_cast<unsigned>(p.row_tiles));
  return CheckLaunchEx(LaunchK(Q8GemmTcKernel<R, ST, M>, grid, dim3(kThreads), L::kSmem, s, 1u,
                               static_cast<unsigned>(p.splits), tw, tx, tu, g),
                       "matmul_q8_tc");
}

template <int R, int M>
int LaunchTcStages(const CUtensorMap& tw, const CUtensorMap& tx, const CUtensorMap& tu, const TcArgs& g,
                   const TcPlan& p, cudaStream_t s) {
  if (p.stages == 2) return LaunchTc<R, 2, M>(tw, tx, tu, g, p, s);
  // Long weight streams with few rows (planes mode): fewer stages leave room
  // for more CTAs per SM, and so more converter warps per SM: two at R = 32
  // with three stages, three at R = 16 with two.
  if constexpr (R == 16 && M == kAPlanes) {
    return LaunchTc<R, 2, M>(tw, tx, tu, g, p, s);
  } else if constexpr (R == 32 && M == kAPlanes) {
    return LaunchTc<R, 3, M>(tw, tx, tu, g, p, s);
  } else {
    return LaunchTc<R, MaxStages<R, M>(), M>(tw, tx, tu, g, p, s);
  }
}

// In-kernel split modes run at R <= 64 (the plan takes planes at R = 128).
template <int M>
int LaunchTcRows(const CUtensorMap& tw, const CUtensorMap& tx, const CUtensorMap& tu, const TcArgs& g,
                 const TcPlan& p, cudaStream_t s) {
  switch (p.r) {
    case 16: return LaunchTcStages<16, M>(tw, tx, tu, g, p, s);
    case 32: return LaunchTcStages<32, M>(tw, tx, tu, g, p, s);
    default: return LaunchTcStages<64, M>(tw, tx, tu, g, p, s);
  }
}

bool Encode2D(CUtensorMap* map, CUtensorMapDataType type, const void* base, uint64_t inner, uint64_t outer,
              uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return EncodeFn()(map, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// Whether the tensor-core path takes this product: a per-column or single
// scale without zero points; weight rows a multiple of 16 bytes and
// activation rows a multiple of 8 elements (TMA strides); 16-byte aligned.
bool TcEligible(const float* a, int64_t lda, const int8_t* w, int32_t axis, const int8_t* zero, int64_t m, int64_t k,
                int64_t n) {
  if (zero != nullptr || (axis != 1 && axis != -1)) return false;
  if (m <= 0 || k <= 0 || n <= 0 || n % 16 != 0 || k % 8 != 0 || lda % 4 != 0) return false;
  if (reinterpret_cast<uintptr_t>(a) % 16 != 0 || reinterpret_cast<uintptr_t>(w) % 16 != 0) return false;
  if (k > (int64_t{1} << 31) - 1 || n > (int64_t{1} << 31) - 1 || m > (int64_t{1} << 31) - 1) return false;
  return CeilDiv(m, TileRows(m)) <= 65535 && EncodeFn() != nullptr;
}

size_t TcWorkspace(int64_t m, int64_t k, int64_t n) {
  const TcPlan p = MakeTcPlan(m, k, n, false, false);
  return kCounterRegion + p.planes_bytes;
}

// a: fp32 rows (lda); with `up` set, the product's A is SiluMul(a, up) (same
// row stride); with `gamma` set, A is RmsNorm(a) with weights gamma [k] and
// eps (a's rows are whole rows of length k). The caller checked TcEligible
// for a (and up).
int RunTc(const float* a, const float* up, int64_t lda, const float* gamma, float eps, const int8_t* w,
          const float* scale, bool scalar_scale, float* c, int64_t ldc, int64_t m, int64_t k, int64_t n,
          const Epilogue& ep, void* workspace, size_t workspace_bytes, int32_t* status, cudaStream_t stream,
          const PeerOut* peers, const double* sq_in, int64_t sq_ld, int32_t sq_n) {
  const TcPlan p = MakeTcPlan(m, k, n, up != nullptr, gamma != nullptr);
  if (p.planes_bytes > 0 && (workspace == nullptr || workspace_bytes < kCounterRegion + p.planes_bytes)) {
    return SetError(ACCEL_B200_EINVAL, "matmul_q8: workspace too small");
  }
  CUtensorMap tw{}, tx{}, tu{};
  if (!Encode2D(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, n, k, n, kBn, kBk, CU_TENSOR_MAP_SWIZZLE_NONE)) {
    return SetError(ACCEL_B200_EINVAL, "matmul_q8: weight tensor map rejected");
  }
  if (p.mode == kAPlanes) {
    auto* planes = reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(workspace) + kCounterRegion);
    const int64_t total = m * (k / 4);
    const int64_t blocks = CeilDiv(total, 256);
    const int grid = static_cast<int>(blocks < kSms * 16 ? blocks : kSms * 16);
    const int rc =
        gamma != nullptr
            ? CheckLaunchEx(LaunchK(SplitPlanesNormKernel, dim3(static_cast<unsigned>(Min64(CeilDiv(m, 8), kSms * 16))),
                                    dim3(256), 0, stream, 1u, 1u, a, lda, gamma, eps, m, k, planes),
                            "matmul_q8_split_norm")
            : CheckLaunchEx(LaunchK(SplitPlanesKernel, dim3(grid), dim3(256), 0, stream, 1u, 1u, a, up, lda, m, k,
                                    planes),
                            "matmul_q8_split");
    if (rc != ACCEL_B200_OK) return rc;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(m), 3};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(k) * 2, static_cast<cuuint64_t>(m) * k * 2};
    const cuuint32_t box[3] = {kBk, static_cast<cuuint32_t>(p.r), 3};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (EncodeFn()(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, planes, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      return SetError(ACCEL_B200_EINVAL, "matmul_q8: activation tensor map rejected");
    }
  } else {
    // fp32 tiles [R rows x 64 k]; rows and k beyond the matrix read as zero.
    const uint64_t row_bytes = static_cast<uint64_t>(lda) * 4;
    if (!Encode2D(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a, k, m, row_bytes, kBk, p.r, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        (up != nullptr &&
         !Encode2D(&tu, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, up, k, m, row_bytes, kBk, p.r, CU_TENSOR_MAP_SWIZZLE_NONE))) {
      return SetError(ACCEL_B200_EINVAL, "matmul_q8: activation tensor map rejected");
    }
    if (up == nullptr) tu = tx;
  }
  TcArgs g{};
  g.a = a;
  g.lda = lda;
  g.gamma = gamma;
  g.eps = eps;
  g.sq_in = sq_in;
  g.sq_ld = sq_ld;
  g.sq_n = sq_n;
  g.m = m;
  g.k = k;
  g.n = n;
  g.kb_total = p.kb_total;
  g.kb_per_split = p.kb_per_split;
  g.scale = scale;
  g.scalar_scale = scalar_scale ? 1 : 0;
  g.c = c;
  g.ldc = ldc;
  g.status = status;
  g.vec_store = (reinterpret_cast<uintptr_t>(c) % 16 == 0 && ldc % 4 == 0) ? 1 : 0;
  g.ep = ep;
  g.peers = peers != nullptr ? *peers : PeerOut{};
  for (int i = 0; i < g.peers.n; ++i) {
    if (reinterpret_cast<uintptr_t>(g.peers.c[i]) % 16 != 0) g.vec_store = 0;
  }
  if (p.mode == kAPlanes) {
    switch (p.r) {
      case 16: return LaunchTcStages<16, kAPlanes>(tw, tx, tu, g, p, stream);
      case 32: return LaunchTcStages<32, kAPlanes>(tw, tx, tu, g, p, stream);
      case 64: return LaunchTcStages<64, kAPlanes>(tw, tx, tu, g, p, stream);
      default: return LaunchTcStages<128, kAPlanes>(tw, tx, tu, g, p, stream);
    }
  }
  if (p.mode == kASilu) return LaunchTcRows<kASilu>(tw, tx, tu, g, p, stream);
  if (p.mode == kANorm) return LaunchTcRows<kANorm>(tw, tx, tu, g, p, stream);
  return LaunchTcRows<kAF32>(tw, tx, tu, g, p, stream);
}

}  // namespace accel_b200
