// int8-weight product on the 5th-generation tensor cores (tcgen05), fed by TMA.
//
// C[m, n] = epilogue(scale[n] * sum_k A[m, k] * q[k, n]) with A fp32 [m, k], q int8
// [k, n] (n contiguous: the reference's QuantPlane layout) and a per-column
// (or single) scale: src/sim_device.cc:541-602 and the epilogue of
// src/runtime.cc:332-344. A may also be SiluMul of a fused gate|up row
// (src/sim_silu.cc:8-13 then the down projection, src/llama_model.cc:239-240)
// or RmsNorm of a row (src/sim_rmsnorm.cc, then the q|k|v, gate|up and LM-head
// products of src/llama_model.cc).
//
// Arithmetic: exact integer dot products. The weights stay int8: TMA writes
// the raw block with 128-byte swizzle, which is the MMA's MN-major canonical
// layout, and kind::i8 MMAs consume it directly (no conversion). Each
// activation row segment (the k range one CTA of a split-K cluster walks; the
// whole row without a split) is put in 30-bit fixed point against its largest
// magnitude: with e the
// smallest exponent such that every |y| < 2^e, X = rint(y * 2^(30 - e)), so an
// element keeps 24 significant bits when |y| >= 2^(e - 7) and an absolute error
// of at most 2^(e - 31) otherwise. X is written as four balanced base-256 digits
// (int8, X = d0 2^24 + d1 2^16 + d2 2^8 + d3), the four digit planes are the
// MMA's B operand, and the tensor core sums w * d exactly in int32 (|sum| <
// 2^31 for up to 1023 * 128 k per CTA). The epilogue recombines the planes in int64,
// rounds once to fp32 and scales by 2^(e - 30): the result is the correctly
// rounded dot product of the weights with the fixed-point row, which is no
// further from the exact product than the reference's own fp32 accumulation.
// A row holding Inf or NaN yields NaN outputs.
//
// The MMA is issued "swapped": M = 128 runs over output features and N over
// activation rows times digit planes (N = 4R, at most 256), so decode with 32
// rows is a full-width MMA.
//
// Activation operand, by mode:
//   planes  (m > 64, or more than two k blocks per CTA): a separate pass
//           forms each row segment (plain, SiluMul or RmsNorm), finds its
//           exponent and writes the digit planes [4][m][kp] and the exponents
//           [segments][m] to the workspace; TMA loads [4][R][128 k] tiles with
//           128-byte swizzle, already the MMA's K-major canonical layout.
//   in-kernel (up to two k blocks per CTA, R <= 64): the converter warps
//           load the CTA's fp32 rows (gate and up for SiluMul) straight into
//           registers (R <= 32; at R = 64 TMA loads them as [R x 128 k]
//           tiles into shared memory first), form them (SiluMul exactly as
//           SiluMul rounds it, RmsNorm exactly as RmsNormKernel rounds it),
//           find the exponents over the range and write the digit planes
//           into shared memory.
//
// Pipeline (one CTA = one 128-feature x R-row tile over a range of 128-deep k
// blocks; 6 or 10 warps):
//   warp 0  producer: per k block one TMA of the int8 weight block [128 k x
//           128 n] and one of the digit tile (planes) or the fp32 tile(s)
//           (in-kernel, R = 64); a ring of stages.
//   warp 1  MMA issuer (one thread): 4 k steps of 32 per block, then
//           tcgen05.commit to the barrier that frees the stage.
//   warps 2.. converters (eight in-kernel, four in planes mode): the
//           in-kernel operand, then the epilogue: tcgen05.ld of the
//           accumulators into a shared fp32 tile, then scale, fused epilogue
//           and coalesced row stores.
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
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string>

#include "accel_b200.h"
#include "cluster.cuh"
#include "common.cuh"
#include "fixed_point.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace accel_b200 {

namespace {

constexpr int kBk = 128;                // k per block: one 128-byte swizzle row of int8
constexpr int kBn = 128;                // output features per tile (MMA M)
constexpr int kMmaK = 32;               // k per int8 MMA
constexpr int kWBytes = kBk * kBn;      // int8 weight block, 16 KiB
constexpr int kMaxBlocksPerCta = 1023;  // |w d| <= 2^14, so 1023 * 128 k of them sum below 2^31
constexpr int kInKernelBlocks = 2;      // k blocks of a CTA that forms its own operand
// Converter warps: eight where they form the operand (latency-bound decode
// products: more threads shorten the operand and epilogue work) and where the
// tile has 64 or more rows (the epilogue's work per thread); four for long
// weight streams with few rows (R = 16 runs three CTAs per SM).
template <int R, int M>
constexpr int ConvWarps() { return (M == 0 && R < 64) ? 4 : 8; }
template <int R, int M>
constexpr int Threads() { return (2 + ConvWarps<R, M>()) * 32; }

// Operand modes. The kernel is instantiated for kAPlanes and for kAIn (the
// in-kernel operand), whose form — plain, SiluMul or RmsNorm rows — is a
// runtime argument (TcArgs::amode): one kernel body serves every decode
// product, so the code the SMs fetch for one product is warm for the next.
enum AMode : int { kAPlanes = 0, kAF32 = 1, kASilu = 2, kANorm = 3, kAIn = 4 };

template <int R, int S, int M>
struct Tc {
  static constexpr int kXBytes = kDigits * R * kBk;  // digit planes of one k block (MMA B operand)
  static constexpr int kStage = kXBytes + kWBytes;   // digits, then the weight block; 1024-aligned
  static constexpr int kStages = S;
  // fp32 tiles per k block (A, and up for SiluMul): in-kernel operands of
  // more than 32 rows only (smaller tiles load their rows into registers).
  static constexpr int kYTiles = (M == kAPlanes || R <= 32) ? 0 : 2;
  static constexpr int kYTile = R * kBk * 4;                                  // one fp32 tile [R][128 k]
  static constexpr int kYBytes = kYTiles * kInKernelBlocks * kYTile;
  static constexpr int kTile = R * kBn * 4;  // fp32 accumulator tile, over the stages after the main loop
  static constexpr int kArea = S * kStage + kYBytes;
  static constexpr int kSmem = (kArea > kTile ? kArea : kTile) + 1024;
  static_assert(M == kAPlanes || S == kInKernelBlocks, "in-kernel operand: one stage per k block");
  static_assert(kStage % 1024 == 0, "stage alignment");
  static_assert(kSmem <= 227 * 1024, "shared memory");
};

struct TcArgs {
  int32_t amode;       // kAIn: how the operand rows are formed (kAF32, kASilu or kANorm)
  const float* a;      // fp32 A rows (norm mode: the whole rows are read for their RMS)
  const float* up;     // silu mode: the up rows (row stride lda)
  int64_t lda;
  const float* gamma;  // norm mode: RmsNorm weights [k]
  float eps;
  const double* sq_in;  // norm mode, optional: per row, sq_n partial sums of squares (stride sq_ld)
  int64_t sq_ld;
  int32_t sq_n;
  const int32_t* row_exp;  // planes mode: [segment (grid y)][m] fixed-point exponents
  int64_t m, k, n;
  int32_t kb_total;
  int32_t kb_per_split;
  const float* scale;
  int32_t scalar_scale;
  float* c;
  int64_t ldc;
  int32_t* status;
  int32_t vec_store;   // c and ldc allow 16-byte row stores
  int32_t silu_pairs;  // gate|up columns in 64-column pairs; C = SiluMul(gate, up), n / 2 columns
  int32_t res_vec;     // the epilogue's residual allows 16-byte row loads
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

// SiluMul of one element as src/sim_silu.cc:8-13 rounds it.
__device__ __forceinline__ float SiluMul(float g, float u) {
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, expf(-g))), u);
}

// A gate|up product in 64-column pairs (TcArgs::silu_pairs: a 128-column
// tile holds 64 gate columns, then the 64 up columns of the same outputs):
// lanes l and l + 16 of a warp hold gate and up of the same output columns
// (4l .. 4l + 3 of the tile), and lane l < 16 stores SiluMul of the pairs, as
// SiluMul rounds it, at output columns n0 / 2 + 4l .. + 3 of the row.
__device__ __forceinline__ void StoreSiluPairs(float* c, int64_t ldc, bool vec, int64_t row, int64_t n0, int lane,
                                               float4 acc, const float (&sc)[4]) {
  const float o[4] = {__fmul_rn(acc.x, sc[0]), __fmul_rn(acc.y, sc[1]), __fmul_rn(acc.z, sc[2]),
                      __fmul_rn(acc.w, sc[3])};
  float u[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) u[q] = __shfl_xor_sync(kFull, o[q], 16);
  if (lane < 16) {
    float* dst = c + row * ldc + n0 / 2 + 4 * lane;
    const float4 y = make_float4(SiluMul(o[0], u[0]), SiluMul(o[1], u[1]), SiluMul(o[2], u[2]), SiluMul(o[3], u[3]));
    if (vec) {
      *reinterpret_cast<float4*>(dst) = y;
    } else {
      dst[0] = y.x;
      dst[1] = y.y;
      dst[2] = y.z;
      dst[3] = y.w;
    }
  }
}

// Element quad q (k = 4q .. 4q + 3) of a row as the mode forms it.
template <int M>
__device__ __forceinline__ float4 FormQuad(const float* a, const float* up, const float* gamma, double inv, int64_t q) {
  const float4 v = __ldg(reinterpret_cast<const float4*>(a) + q);
  if constexpr (M == kASilu) {
    const float4 u = __ldg(reinterpret_cast<const float4*>(up) + q);
    return make_float4(SiluMul(v.x, u.x), SiluMul(v.y, u.y), SiluMul(v.z, u.z), SiluMul(v.w, u.w));
  } else if constexpr (M == kANorm) {
    const float4 g = __ldg(reinterpret_cast<const float4*>(gamma) + q);
    return make_float4(__fmul_rn(static_cast<float>(static_cast<double>(v.x) * inv), g.x),
                       __fmul_rn(static_cast<float>(static_cast<double>(v.y) * inv), g.y),
                       __fmul_rn(static_cast<float>(static_cast<double>(v.z) * inv), g.z),
                       __fmul_rn(static_cast<float>(static_cast<double>(v.w) * inv), g.w));
  } else {
    return v;
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
template <int R, int CW>
__device__ __noinline__ void TileInverseRms(const float* a, int64_t lda, int64_t row0, int valid, int64_t dim,
                                               float eps, int ct, double* inv) {
  for (int base = 0; base < R; base += CW * 8) {
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

// In-kernel operand: the fp32 rows of the CTA's k blocks (rows past the
// matrix and k past K read as zero) are formed as the mode does, the
// exponents over the range found (exp_s, every row of the tile), and the
// digit planes of block b written into stage b: plane p, row r at (p R + r) *
// 128, the 16-byte chunk j of a row stored at j ^ (r % 8) (the TMA's 128-byte
// swizzle). Converter warp w takes block w % nkb, rows w / nkb, + CW / nkb,
// ...; lane l the quad k = 4l .. 4l + 3 of the block. Tiles of up to 32 rows
// load their quads from global memory (row0 + r of A, and of up for SiluMul)
// straight into registers, all of a warp's loads issued back to back, and
// keep the formed rows there between the maxima and the digits; 64-row tiles
// read the tiles TMA placed in shared memory (block b at ytiles + b * tiles *
// R * 128 floats: A, then up for SiluMul; rows of 128 k), write the formed
// rows back in place and read them again.
template <int R, int CW>
__device__ __forceinline__ void BuildDigits(const TcArgs& g, int nkb, int64_t k0, const double* inv, float* ytiles,
                                            uint32_t* amax, int32_t* exp_s, uint8_t* stages, int stage_bytes,
                                            int ct, int64_t row0) {
  const int mode = g.amode;
  const int kTiles = mode == kASilu ? 2 : 1;
  const int w = ct >> 5, lane = ct & 31;
  const int b = w % nkb, r0 = w / nkb, rstep = CW / nkb;
  const int kb = 4 * lane;  // k offset inside the block
  float* y_at = ytiles + b * kTiles * R * kBk + kb;
  float4 gam = make_float4(0.f, 0.f, 0.f, 0.f);
  if (mode == kANorm) {
    if (k0 + b * kBk + kb < g.k) gam = __ldg(reinterpret_cast<const float4*>(g.gamma + k0 + b * kBk + kb));
  }
  const auto form = [&](float4 v, int r) {
    if (mode == kASilu) {
      const float4 u = *reinterpret_cast<const float4*>(y_at + R * kBk + r * kBk);
      return make_float4(SiluMul(v.x, u.x), SiluMul(v.y, u.y), SiluMul(v.z, u.z), SiluMul(v.w, u.w));
    } else if (mode == kANorm) {
      const double iv = inv[r];
      return make_float4(__fmul_rn(static_cast<float>(static_cast<double>(v.x) * iv), gam.x),
                         __fmul_rn(static_cast<float>(static_cast<double>(v.y) * iv), gam.y),
                         __fmul_rn(static_cast<float>(static_cast<double>(v.z) * iv), gam.z),
                         __fmul_rn(static_cast<float>(static_cast<double>(v.w) * iv), gam.w));
    } else {
      return v;
    }
  };
  const auto row_exponent = [&](int r) {
    return RowExponent(nkb > 1 ? max(amax[2 * r], amax[2 * r + 1]) : amax[2 * r]);
  };
  uint8_t* xs = stages + b * stage_bytes;
  const int chunk = kb >> 4, byte = kb & 15;
  const auto store_digits = [&](float4 y, int r, int32_t e) {
    uint32_t d[kDigits] = {0u, 0u, 0u, 0u};
    if (e != kBadRow) FourDigits(y, FixScale(e), d);
    const int off = (((chunk ^ (r & 7)) << 4) | byte) + r * kBk;
#pragma unroll
    for (int p = 0; p < kDigits; ++p) *reinterpret_cast<uint32_t*>(xs + p * R * kBk + off) = d[p];
  };
  if constexpr (R <= 32) {
    // At most R * 2 / CW rows per warp (nkb <= 2); r is the same for the
    // whole warp, so the shuffles below see every lane.
    constexpr int kRows = (R * kInKernelBlocks + CW - 1) / CW;
    float4 y[kRows];
    const int64_t kk = k0 + b * kBk + kb;
    const bool kin = kk < g.k;
#pragma unroll
    for (int i = 0; i < kRows; ++i) {
      const int r = r0 + i * rstep;
      const int64_t row = row0 + r;
      y[i] = (r < R && row < g.m && kin) ? __ldg(reinterpret_cast<const float4*>(g.a + row * g.lda + kk))
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (mode == kASilu) {
#pragma unroll
      for (int i = 0; i < kRows; ++i) {
        const int r = r0 + i * rstep;
        const int64_t row = row0 + r;
        const float4 u = (r < R && row < g.m && kin) ? __ldg(reinterpret_cast<const float4*>(g.up + row * g.lda + kk))
                                                     : make_float4(0.f, 0.f, 0.f, 0.f);
        y[i] = make_float4(SiluMul(y[i].x, u.x), SiluMul(y[i].y, u.y), SiluMul(y[i].z, u.z), SiluMul(y[i].w, u.w));
      }
    } else {
#pragma unroll
      for (int i = 0; i < kRows; ++i) {
        const int r = r0 + i * rstep;
        if (r < R) y[i] = form(y[i], r);
      }
    }
    uint32_t m[kRows];
#pragma unroll
    for (int i = 0; i < kRows; ++i) m[i] = __reduce_max_sync(kFull, AbsMaxBits(y[i]));
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < kRows; ++i) {
        const int r = r0 + i * rstep;
        if (r < R) amax[2 * r + b] = m[i];
      }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(CW * 32) : "memory");  // converter warps only
    if (ct < R) exp_s[ct] = row_exponent(ct);
#pragma unroll
    for (int i = 0; i < kRows; ++i) {
      const int r = r0 + i * rstep;
      if (r < R) store_digits(y[i], r, row_exponent(r));
    }
  } else {
#pragma unroll 4
    for (int r = r0; r < R; r += rstep) {
      float4* at = reinterpret_cast<float4*>(y_at + r * kBk);
      const float4 y = form(*at, r);
      if (mode != kAF32) *at = y;
      const uint32_t m = __reduce_max_sync(kFull, AbsMaxBits(y));
      if (lane == 0) amax[2 * r + b] = m;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(CW * 32) : "memory");  // converter warps only
    if (ct < R) exp_s[ct] = row_exponent(ct);
#pragma unroll 4
    for (int r = r0; r < R; r += rstep) store_digits(*reinterpret_cast<const float4*>(y_at + r * kBk), r, row_exponent(r));
  }
}

// Planes-mode kernels run several CTAs per SM (three at R = 16, two above:
// long weight streams, prefill), which the register budget must allow.
template <int R, int M>
constexpr int MinBlocks() { return M != kAPlanes ? 1 : (R == 16 ? 3 : 2); }

// The epilogue of an unsplit tile: rows of the shared-memory tile through the
// fused epilogue to C (and the peer copies, the row sums). Warp w takes rows
// w, w + kWarpsN, ...; lane l the columns c4 .. c4 + 3.
template <int kWarpsN>
__device__ __forceinline__ void StoreUnsplitBody(const TcArgs& g, const float* tile, int64_t rows, int warp, int lane,
                                                 int c4, const float (&sc)[4], int64_t cols, int64_t row0,
                                                 int64_t n0) {
  if (g.silu_pairs) {
    for (int r = warp; r < rows; r += kWarpsN) {
      StoreSiluPairs(g.c, g.ldc, g.vec_store, row0 + r, n0, lane,
                     *reinterpret_cast<const float4*>(tile + r * kBn + c4), sc);
    }
  } else if (g.peers.n == 0 && g.ep.row_sq == nullptr && g.vec_store && cols == kBn) {
    // The common case, kept free of the optional outputs.
#pragma unroll 2
    for (int r = warp; r < rows; r += kWarpsN) {
      const int64_t row = row0 + r;
      const float4 v = *reinterpret_cast<const float4*>(tile + r * kBn + c4);
      *reinterpret_cast<float4*>(g.c + row * g.ldc + n0 + c4) =
          make_float4(ApplyEpilogue(g.ep, __fmul_rn(v.x, sc[0]), row, n0 + c4),
                      ApplyEpilogue(g.ep, __fmul_rn(v.y, sc[1]), row, n0 + c4 + 1),
                      ApplyEpilogue(g.ep, __fmul_rn(v.z, sc[2]), row, n0 + c4 + 2),
                      ApplyEpilogue(g.ep, __fmul_rn(v.w, sc[3]), row, n0 + c4 + 3));
    }
  } else {
    for (int r = warp; r < rows; r += kWarpsN) {
      const int64_t row = row0 + r;
      double sq = 0.0;
      if (c4 < cols) {
        const float4 v = *reinterpret_cast<const float4*>(tile + r * kBn + c4);
        const float in[4] = {v.x, v.y, v.z, v.w};
        float o[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) o[q] = ApplyEpilogue(g.ep, __fmul_rn(in[q], sc[q]), row, n0 + c4 + q);
        if (g.ep.row_sq != nullptr) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if (c4 + q < cols) {
              const double dv = static_cast<double>(o[q]);
              sq = fma(dv, dv, sq);  // one fused multiply-add, as every kernel that writes row sums does
            }
          }
        }
        const int64_t off = row * g.ldc + n0 + c4;
        if (g.vec_store && c4 + 4 <= cols) {
          *reinterpret_cast<float4*>(g.c + off) = make_float4(o[0], o[1], o[2], o[3]);
          StorePeers4(g.peers, off, make_float4(o[0], o[1], o[2], o[3]));
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if (c4 + q < cols) {
              g.c[off + q] = o[q];
              StorePeers(g.peers, off + q, o[q]);
            }
          }
        }
      }
      if (g.ep.row_sq != nullptr) {  // the warp holds the row's columns of this tile
        sq = WarpSum(sq);
        if (lane == 0) g.ep.row_sq[row * g.ep.row_sq_ld + n0 / kBn] = sq;
      }
    }
  }
  if (g.peers.n > 0) __threadfence_system();  // peer copies land before the kernel completes
}

// The same, out of line: the in-kernel (decode) products split K and never
// take it, and their kernel keeps fewer instructions in cache without it.
template <int kWarpsN>
__device__ __noinline__ void StoreUnsplitCold(TcArgs g, const float* tile, int64_t rows, int warp, int lane, int c4,
                                              float4 scv, int64_t cols, int64_t row0, int64_t n0) {
  const float sc[4] = {scv.x, scv.y, scv.z, scv.w};
  StoreUnsplitBody<kWarpsN>(g, tile, rows, warp, lane, c4, sc, cols, row0, n0);
}

template <int R, int kStagesT, int M>
__global__ void __launch_bounds__(Threads<R, M>(), MinBlocks<R, M>())
    Q8GemmTcKernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx,
                   const __grid_constant__ CUtensorMap tu, TcArgs g) {
  using L = Tc<R, kStagesT, M>;
  constexpr int S = L::kStages;
  constexpr int kConvWarps = ConvWarps<R, M>();
  constexpr int kThreads = Threads<R, M>();
  constexpr int kN = kDigits * R;                 // MMA N over all digit planes
  constexpr int kMmas = kN <= 256 ? 1 : 2;        // R = 128: two MMAs of N = 256
  constexpr int kNMma = kN / kMmas;
  constexpr uint32_t kCols = kN <= 64 ? 64 : (kN <= 128 ? 128 : (kN <= 256 ? 256 : 512));
  constexpr uint32_t kIdesc = InstrDescS8(kNMma);
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_w[S], full_x[S], empty[S], xready, accf;
  __shared__ uint32_t tmem_s;
  __shared__ int32_t exp_s[R];
  __shared__ uint32_t amax_s[M == kAPlanes ? 1 : 2 * R];
  __shared__ double inv_s[M == kAPlanes ? 1 : R];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t raw_addr = SmemAddr(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023) & ~1023u) - raw_addr);
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * kBn;
  const int64_t row0 = static_cast<int64_t>(blockIdx.z) * R;
  const int kb_begin = blockIdx.y * g.kb_per_split;
  const int nkb = max(0, min(g.kb_total, kb_begin + g.kb_per_split) - kb_begin);

  // The next kernel may launch at once, or (TRIGGER_AFTER_WAIT) only once a
  // thread of this CTA has waited for the previous kernel: then every kernel
  // before this one has completed when the next one starts.
  const bool late = (g.ep.flags & ACCEL_B200_EP_TRIGGER_AFTER_WAIT) != 0;
  if (!late) PdlTrigger();
  const auto wait_prev = [late] {
    PdlWait();
    if (late) PdlTrigger();
  };
  if (warp == 1) TmemAlloc(&tmem_s, kCols);
  // The epilogue's column scales, lane l's four columns 4l .. 4l + 3 of the
  // tile in every warp. The latency-bound in-kernel modes load them here
  // (immutable, so before the wait); planes mode, whose long weight streams
  // want the registers, loads them at the epilogue.
  constexpr bool kEarly = M != kAPlanes;
  const int64_t cols = Min64(kBn, g.n - n0);
  const int c4 = lane * 4;
  float sc[4];
  const auto load_scales = [&] {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      sc[j] = (c4 + j < cols) ? (g.scalar_scale ? __ldg(g.scale) : __ldg(g.scale + n0 + c4 + j)) : 0.f;
    }
  };
  if constexpr (kEarly) load_scales();
  // Split K (a cluster along grid y): rank `rank` sums rows [rank * rpr, +rpr)
  // of the tile over the cluster. A thread owns one group of four columns
  // (lane) in rows ew, ew + kEpiWarps, ... of that range, where ew is its
  // epilogue warp: the converter warps in the in-kernel modes (which load
  // their residual rows right after the wait, long before the epilogue reads
  // them), every warp in planes mode.
  const auto split_rows = [&](int* r_begin, int* r_end) {
    const int splits = static_cast<int>(gridDim.y);
    const int rows = static_cast<int>(Min64(R, g.m - row0));
    const int rank = static_cast<int>(blockIdx.y);  // cluster (1, splits, 1): rank = y
    const int rpr = (rows + splits - 1) / splits;
    const int ew = kEarly ? warp - 2 : warp;
    // A warp that takes no epilogue rows (producer, MMA issuer) gets an
    // empty range: r_begin >= r_end for every row it would step through.
    *r_begin = ew < 0 ? 0 : rank * rpr + ew;
    *r_end = ew < 0 ? 0 : min(rows, (rank + 1) * rpr);
  };
  constexpr int kEpiWarps = kEarly ? kConvWarps : kThreads / 32;
  constexpr int kMaxJ = (R / 2 + kEpiWarps - 1) / kEpiWarps;  // rows per thread (splits >= 2)
  float4 res[kEarly ? kMaxJ : 1];
  const bool res_pre = kEarly && gridDim.y > 1 && g.res_vec && !g.silu_pairs && c4 + 4 <= cols;
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      MbarInit(&full_w[s], 1);
      MbarInit(&full_x[s], 1);
      MbarInit(&empty[s], 1);
    }
    MbarInit(&xready, kConvWarps);
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
        MbarArriveExpectTx(&full_w[i], kWBytes);
        TmaLoad2D(smem + i * L::kStage + L::kXBytes, &tw, static_cast<int32_t>(n0), (kb_begin + i) * kBk, &full_w[i]);
      }
      if constexpr (M == kAPlanes) {
        wait_prev();
        for (int i = 0; i < nkb; ++i) {
          const int s = i % S;
          uint8_t* stage = smem + s * L::kStage;
          const int32_t k0 = (kb_begin + i) * kBk;
          if (i >= S) {
            ok &= MbarWait(&empty[s], ((i / S) & 1) ^ 1);
            MbarArriveExpectTx(&full_w[s], kWBytes);
            TmaLoad2D(stage + L::kXBytes, &tw, static_cast<int32_t>(n0), k0, &full_w[s]);
          }
          MbarArriveExpectTx(&full_x[s], L::kXBytes);
          TmaLoad3D(stage, &tx, k0, static_cast<int32_t>(row0), 0, &full_x[s]);
        }
      } else {
        // The fp32 tiles of every k block of the CTA, one barrier per block
        // (64-row tiles; smaller ones are loaded by the converter warps).
        wait_prev();
        float* ytiles = reinterpret_cast<float*>(smem + S * L::kStage);
        const int tiles = g.amode == kASilu ? 2 : 1;
        for (int i = 0; i < (R <= 32 ? 0 : nkb); ++i) {  // R <= 32: the converter warps load the rows
          const int32_t k0 = (kb_begin + i) * kBk;
          float* dst = ytiles + i * tiles * R * kBk;
          MbarArriveExpectTx(&full_x[i], static_cast<uint32_t>(tiles * L::kYTile));
          TmaLoad2D(dst, &tx, k0, static_cast<int32_t>(row0), &full_x[i]);
          if (tiles == 2) TmaLoad2D(dst + R * kBk, &tu, k0, static_cast<int32_t>(row0), &full_x[i]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // Nothing for the MMA arrives before the previous kernel completes: wait
      // in griddepcontrol.wait (no issue slots) rather than polling barriers
      // while that kernel still runs on this SM.
      wait_prev();
      // Suspended, not polling: a polling warp would compete for the shared
      // memory pipe with the converter warps that form the operand meanwhile.
      if constexpr (M != kAPlanes) ok &= MbarWaitSleep(&xready, 0);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S;
        ok &= MbarWait(&full_w[s], (i / S) & 1);
        if constexpr (M == kAPlanes) ok &= MbarWait(&full_x[s], (i / S) & 1);
        TcFenceAfterSync();
        const uint32_t b_addr = SmemAddr(smem + s * L::kStage);
        const uint32_t a_addr = b_addr + L::kXBytes;
#pragma unroll
        for (int ks = 0; ks < kBk / kMmaK; ++ks) {
          // A (weights, n-contiguous; the 128 features are one 128-byte atom,
          // so there is no second atom for LBO to locate): 32 k rows = 4096
          // bytes per step, 8-row k groups 1024 apart (SBO).
          // B (digit rows, k-contiguous): 32 bytes of k per step inside the
          // swizzled row; 8-row groups 1024 apart (SBO).
          const uint64_t adesc = SmemDescSw128(a_addr + ks * (kMmaK * kBn), 0, 1024);
#pragma unroll
          for (int mm = 0; mm < kMmas; ++mm) {
            const uint64_t bdesc = SmemDescSw128(b_addr + mm * kNMma * kBk + ks * kMmaK, 16, 1024);
            MmaS8(tmem + mm * kNMma, adesc, bdesc, kIdesc, (i | ks) != 0);
          }
        }
        MmaCommit(&empty[s]);
      }
      if (nkb > 0) MmaCommit(&accf);
    }
  } else {
    const int ct = tid - 64;
    const int valid = static_cast<int>(Min64(R, g.m - row0));
    wait_prev();
    if constexpr (kEarly) {
      if (res_pre) {
        int r_begin, r_end;
        split_rows(&r_begin, &r_end);
#pragma unroll
        for (int j = 0; j < kMaxJ; ++j) {
          const int r = r_begin + j * kEpiWarps;
          res[j] = r < r_end
                       ? __ldg(reinterpret_cast<const float4*>(g.ep.residual + (row0 + r) * g.ep.residual_ld + n0 + c4))
                       : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    }
    if constexpr (M == kAPlanes) {
      if (ct < R) exp_s[ct] = ct < valid ? g.row_exp[blockIdx.y * g.m + row0 + ct] : 0;
      if (nkb > 0) ok &= MbarWaitSleep(&accf, 0);
    } else {
      if (g.amode == kANorm) {
        // Row RMS of the valid rows: from the producer's sums of squares when
        // given, else from the whole rows of A.
        if (g.sq_in != nullptr) {
          if (ct < valid) {
            const double* p = g.sq_in + (row0 + ct) * g.sq_ld;
            double sum = 0.0;
            for (int t = 0; t < g.sq_n; ++t) sum += p[t];
            inv_s[ct] = 1.0 / sqrt(sum / static_cast<double>(g.k) + static_cast<double>(g.eps));
          }
        } else {
          TileInverseRms<R, kConvWarps>(g.a, g.lda, row0, valid, g.k, g.eps, ct, inv_s);
        }
        if (ct >= valid && ct < R) inv_s[ct] = 0.0;  // rows past the matrix (their tiles read as zero)
        asm volatile("bar.sync 1, %0;" ::"n"(kConvWarps * 32) : "memory");  // converter warps only
      }
      if constexpr (R > 32) {
        for (int i = 0; i < nkb; ++i) ok &= MbarWaitSleep(&full_x[i], 0);
      }
      BuildDigits<R, kConvWarps>(g, nkb, static_cast<int64_t>(kb_begin) * kBk, inv_s,
                        reinterpret_cast<float*>(smem + S * L::kStage), amax_s, exp_s, smem, L::kStage, ct, row0);
      FenceProxyAsyncSmem();
      __syncwarp();
      if (lane == 0) MbarArrive(&xready);
      if (nkb > 0) ok &= MbarWaitSleep(&accf, 0);
    }
  }
  // Every thread past this point may read the residual or write the output.
  wait_prev();
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
  int r_begin, r_end;
  split_rows(&r_begin, &r_end);
  float* tile = reinterpret_cast<float*>(smem);  // [R][kBn], over the stages
  if (warp >= 2) {
    // Thread (quarter, lane) holds feature 32 * quarter + lane: its TMEM lane.
    // Column p * R + r holds digit plane p of row r. With eight converter
    // warps, the two warps of a quarter take alternate 16-row chunks.
    const int quarter = warp & 3;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    constexpr int kChunk = 16;
    constexpr int kWarpsPerQuarter = kConvWarps / 4;
#pragma unroll 1
    for (int c0 = ((warp - 2) >> 2) * kChunk; c0 < R; c0 += kChunk * kWarpsPerQuarter) {
      float v[kChunk];
      if (nkb > 0 && cta_ok) {
        uint32_t d[kDigits][kChunk];
#pragma unroll
        for (int p = 0; p < kDigits; ++p) TmemLoad16Raw(lane_base + p * R + c0, d[p]);
        TmemWaitLoads();
#pragma unroll
        for (int j = 0; j < kChunk; ++j) {
          v[j] = PlanesToFloat(static_cast<int32_t>(d[0][j]), static_cast<int32_t>(d[1][j]),
                               static_cast<int32_t>(d[2][j]), static_cast<int32_t>(d[3][j]), exp_s[c0 + j]);
        }
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
  if constexpr (!kEarly) load_scales();
  if (splits == 1) {
    if (warp == 1) TmemDealloc(tmem, kCols);
    if (cta_ok) {
      if constexpr (kEarly) {
        StoreUnsplitCold<kThreads / 32>(g, tile, rows, warp, lane, c4, make_float4(sc[0], sc[1], sc[2], sc[3]), cols,
                                        row0, n0);
      } else {
        StoreUnsplitBody<kThreads / 32>(g, tile, rows, warp, lane, c4, sc, cols, row0, n0);
      }
    }
    return;
  }
  ClusterSync();  // every partial tile of the cluster is complete
  float4 sum[kMaxJ];
  if (c4 < cols) {
#pragma unroll
    for (int j = 0; j < kMaxJ; ++j) {
      const int r = r_begin + j * kEpiWarps;
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
    const int r = r_begin + j * kEpiWarps;  // the same for the 32 lanes of a warp
    if (r < r_end && g.silu_pairs) {
      StoreSiluPairs(g.c, g.ldc, g.vec_store, row0 + r, n0, lane, sum[j], sc);
    } else if (r < r_end) {
      double sq = 0.0;
      if (c4 < cols) {
        const int64_t row = row0 + r;
        const float v[4] = {sum[j].x, sum[j].y, sum[j].z, sum[j].w};
        float o[4];
        if (res_pre) {
          // The residual comes last in the epilogue (ApplyEpilogue's order).
          Epilogue head = g.ep;
          head.residual = nullptr;
          const float4 rj = res[kEarly ? j : 0];  // loaded after the wait (converter branch)
          const float rv[4] = {rj.x, rj.y, rj.z, rj.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            o[q] = __fadd_rn(ApplyEpilogue(head, __fmul_rn(v[q], sc[q]), row, n0 + c4 + q), rv[q]);
          }
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q) o[q] = ApplyEpilogue(g.ep, __fmul_rn(v[q], sc[q]), row, n0 + c4 + q);
        }
        if (g.ep.row_sq != nullptr) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if (c4 + q < cols) {
              const double dv = static_cast<double>(o[q]);
              sq = fma(dv, dv, sq);  // one fused multiply-add, as every kernel that writes row sums does
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
  if (warp == 1) TmemDealloc(tmem, kCols);  // off the reduction's path: the read-out finished above
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");  // peers are done with this tile
}

// Planes mode operand. Segment s of row r (k in [s * seg, min(k, (s + 1) *
// seg)): the range CTA s of a split-K cluster walks) is formed as the mode does
// (M: kAF32, kASilu or kANorm), its exponent found over the segment, and its
// four digit planes written (plane p of row r at p * m * kp + r * kp) with the
// exponent at row_exp[s * m + r]. A group of 2^group_log2 threads (32 .. 256)
// takes one (row, segment) item and keeps up to kDigitQuads quads per thread in
// registers; a longer segment is formed twice.
constexpr int kDigitQuads = 8;
constexpr int kDigitThreads = 256;

template <int M>
__global__ void __launch_bounds__(kDigitThreads)
    DigitPlanesKernel(const float* __restrict__ a, const float* __restrict__ up, int64_t lda,
                      const float* __restrict__ gamma, float eps, int64_t m, int64_t k, int64_t kp, int64_t seg,
                      int64_t nseg, uint8_t* __restrict__ planes, int32_t* __restrict__ row_exp, int group_log2) {
  __shared__ uint32_t part[kDigitThreads / 32];
  __shared__ double inv_sh[kDigitThreads / 32];
  PdlTrigger();
  PdlWait();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int group_threads = 1 << group_log2, groups = kDigitThreads >> group_log2;
  const int gi = tid >> group_log2, t = tid & (group_threads - 1);
  const int64_t items = m * nseg, plane = m * kp;
  // The loop bound is the same for every thread of the CTA (barriers inside).
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * groups; base < items;
       base += static_cast<int64_t>(gridDim.x) * groups) {
    const int64_t item = base + gi;
    const bool live = item < items;
    const int64_t r = live ? item / nseg : 0, sg = live ? item % nseg : 0;
    const int64_t k0 = sg * seg;
    const int64_t quads = live ? Min64(seg, k - k0) / 4 : 0;
    const float* in = a + r * lda;
    const float* uin = M == kASilu ? up + r * lda + k0 : nullptr;
    const float* gam = M == kANorm ? gamma + k0 : nullptr;
    double inv = 0.0;
    if constexpr (M == kANorm) {
      if (t < 32 && live) {
        const double iv = RowInverseRms(in, k, eps, lane);  // the whole row, as RmsNormKernel sums it
        if (lane == 0) inv_sh[gi] = iv;
      }
      __syncthreads();
      inv = inv_sh[gi];
    }
    float4 y[kDigitQuads];
    uint32_t amax = 0;
#pragma unroll
    for (int j = 0; j < kDigitQuads; ++j) {
      const int64_t q = t + static_cast<int64_t>(j) * group_threads;
      y[j] = q < quads ? FormQuad<M>(in + k0, uin, gam, inv, q) : make_float4(0.f, 0.f, 0.f, 0.f);
      amax = max(amax, AbsMaxBits(y[j]));
    }
    for (int64_t q = t + static_cast<int64_t>(kDigitQuads) * group_threads; q < quads; q += group_threads) {
      amax = max(amax, AbsMaxBits(FormQuad<M>(in + k0, uin, gam, inv, q)));
    }
    amax = __reduce_max_sync(kFull, amax);
    if (lane == 0) part[warp] = amax;
    __syncthreads();
    uint32_t gmax = 0;
    for (int w = gi * (group_threads >> 5); w < (gi + 1) * (group_threads >> 5); ++w) gmax = max(gmax, part[w]);
    const int32_t e = RowExponent(gmax);
    __syncthreads();  // `part` is rewritten by the next item
    uint8_t* dst = planes + r * kp + k0;
#pragma unroll
    for (int j = 0; j < kDigitQuads; ++j) {
      const int64_t q = t + static_cast<int64_t>(j) * group_threads;
      if (q < quads) {
        uint32_t w[kDigits] = {0u, 0u, 0u, 0u};
        if (e != kBadRow) FourDigits(y[j], FixScale(e), w);
#pragma unroll
        for (int p = 0; p < kDigits; ++p) *reinterpret_cast<uint32_t*>(dst + p * plane + 4 * q) = w[p];
      }
    }
    for (int64_t q = t + static_cast<int64_t>(kDigitQuads) * group_threads; q < quads; q += group_threads) {
      uint32_t w[kDigits] = {0u, 0u, 0u, 0u};
      if (e != kBadRow) FourDigits(FormQuad<M>(in + k0, uin, gam, inv, q), FixScale(e), w);
#pragma unroll
      for (int p = 0; p < kDigits; ++p) *reinterpret_cast<uint32_t*>(dst + p * plane + 4 * q) = w[p];
    }
    if (live && t == 0) row_exp[sg * m + r] = e;
  }
}

struct TcPlan {
  int r;
  int mode;  // AMode
  int64_t feature_tiles, row_tiles;
  int32_t kb_total, kb_per_split, splits;
  int64_t kp;           // digit plane row stride (bytes)
  size_t digits_bytes;  // planes mode: the digit planes in the workspace (1024-aligned)
  size_t planes_bytes;  // planes mode: digit planes and segment exponents
};

// Activation rows per tile (the MMA's N is four times this). Above 32 rows,
// 64-row tiles: two CTAs (two stages each) share an SM, so that one CTA's
// prologue and epilogue overlap the other's MMAs.
int64_t TileRows(int64_t m) { return m <= 16 ? 16 : (m <= 32 ? 32 : 64); }

TcPlan MakeTcPlan(int64_t m, int64_t k, int64_t n, bool silu, bool norm) {
  TcPlan p{};
  p.r = static_cast<int>(TileRows(m));
  p.feature_tiles = CeilDiv(n, kBn);
  p.row_tiles = CeilDiv(m, p.r);
  p.kb_total = static_cast<int32_t>(CeilDiv(k, kBk));
  // When the tile grid is smaller than the GPU, split K across a cluster of up
  // to 8 CTAs: the largest split whose grid still fits in one wave of the CTAs
  // an SM holds (three at R = 16, two above).
  const int64_t base = p.feature_tiles * p.row_tiles;
  int64_t splits = 1;
  if (base < kSms && p.kb_total > 1) {
    const int64_t per_sm = p.r == 16 ? 3 : 2;
    splits = Min64(p.kb_total, Max64(1, per_sm * kSms / base));
    if (splits > 8) splits = 8;
  }
  splits = Max64(splits, CeilDiv(p.kb_total, kMaxBlocksPerCta));  // TcEligible keeps this <= 8
  p.kb_per_split = static_cast<int32_t>(CeilDiv(p.kb_total, splits));
  p.splits = static_cast<int32_t>(CeilDiv(p.kb_total, p.kb_per_split));
  // A CTA that forms its own operand saves the planes pass (one launch) but
  // holds its whole k range in shared memory: worth it for CTAs that walk few
  // blocks (latency-bound decode products), not for long weight streams.
  const bool planes = m > 64 || p.kb_per_split > kInKernelBlocks;
  p.mode = planes ? kAPlanes : (silu ? kASilu : (norm ? kANorm : kAF32));
  p.kp = (k + 15) / 16 * 16;
  p.digits_bytes = planes ? (static_cast<size_t>(kDigits) * m * p.kp + 1023) / 1024 * 1024 : 0;
  p.planes_bytes = planes ? p.digits_bytes + (static_cast<size_t>(p.splits) * m * 4 + 1023) / 1024 * 1024 : 0;
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
  return CheckLaunchEx(LaunchK(Q8GemmTcKernel<R, ST, M>, grid, dim3(Threads<R, M>()), L::kSmem, s, 1u,
                               static_cast<unsigned>(p.splits), tw, tx, tu, g),
                       "matmul_q8_tc");
}

// In-kernel operand modes (m <= 64): one instantiation per tile height, the
// mode in TcArgs::amode.
int LaunchTcRows(const CUtensorMap& tw, const CUtensorMap& tx, const CUtensorMap& tu, const TcArgs& g,
                 const TcPlan& p, cudaStream_t s) {
  switch (p.r) {
    case 16: return LaunchTc<16, kInKernelBlocks, kAIn>(tw, tx, tu, g, p, s);
    case 32: return LaunchTc<32, kInKernelBlocks, kAIn>(tw, tx, tu, g, p, s);
    default: return LaunchTc<64, kInKernelBlocks, kAIn>(tw, tx, tu, g, p, s);
  }
}

// Planes mode, stages by tile rows: as many CTAs per SM as fit (three at R =
// 16, two at R = 32 and 64) with the stages that leaves room for.
int LaunchTcPlanes(const CUtensorMap& tw, const CUtensorMap& tx, const TcArgs& g, const TcPlan& p, cudaStream_t s) {
  switch (p.r) {
    case 16: return LaunchTc<16, 3, kAPlanes>(tw, tx, tx, g, p, s);
    case 32: return LaunchTc<32, 3, kAPlanes>(tw, tx, tx, g, p, s);
    default: return LaunchTc<64, 2, kAPlanes>(tw, tx, tx, g, p, s);
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
// scale without zero points; weight rows a multiple of 16 bytes (TMA stride)
// and activation rows a multiple of 8 elements; 16-byte aligned; at most 8 x
// 1023 * 128 k (the int32 sums of a CTA hold 1023 * 128 k).
bool TcEligible(const float* a, int64_t lda, const int8_t* w, int32_t axis, const int8_t* zero, int64_t m, int64_t k,
                int64_t n) {
  if (zero != nullptr || (axis != 1 && axis != -1)) return false;
  if (m <= 0 || k <= 0 || n <= 0 || n % 16 != 0 || k % 8 != 0 || lda % 4 != 0) return false;
  if (reinterpret_cast<uintptr_t>(a) % 16 != 0 || reinterpret_cast<uintptr_t>(w) % 16 != 0) return false;
  if (k > int64_t{8} * kMaxBlocksPerCta * kBk || n > (int64_t{1} << 31) - 1 || m > (int64_t{1} << 31) - 1) {
    return false;
  }
  return CeilDiv(m, TileRows(m)) <= 65535 && EncodeFn() != nullptr;
}

size_t TcWorkspace(int64_t m, int64_t k, int64_t n) {
  const TcPlan p = MakeTcPlan(m, k, n, false, false);
  return kCounterRegion + p.planes_bytes;
}

// a: fp32 rows (lda); with `up` set, the product's A is SiluMul(a, up) (same
// row stride); with `gamma` set, A is RmsNorm(a) with weights gamma [k] and
// eps (a's rows are whole rows of length k). With silu_pairs, n % 128 == 0,
// the weight columns are gate|up 64-column pairs and C receives SiluMul(gate,
// up) (n / 2 columns; the epilogue is the plain product, no peers). The caller
// checked TcEligible for a (and up).
int RunTc(const float* a, const float* up, int64_t lda, const float* gamma, float eps, const int8_t* w,
          const float* scale, bool scalar_scale, float* c, int64_t ldc, int64_t m, int64_t k, int64_t n,
          const Epilogue& ep, void* workspace, size_t workspace_bytes, int32_t* status, cudaStream_t stream,
          const PeerOut* peers, const double* sq_in, int64_t sq_ld, int32_t sq_n, bool silu_pairs) {
  const TcPlan p = MakeTcPlan(m, k, n, up != nullptr, gamma != nullptr);
  if (p.planes_bytes > 0 && (workspace == nullptr || workspace_bytes < kCounterRegion + p.planes_bytes)) {
    return SetError(ACCEL_B200_EINVAL, "matmul_q8: workspace too small");
  }
  CUtensorMap tw{}, tx{}, tu{};
  // Weight blocks [128 k][128 n] with 128-byte swizzle: the MMA's MN-major layout.
  if (!Encode2D(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, n, k, n, kBn, kBk, CU_TENSOR_MAP_SWIZZLE_128B)) {
    return SetError(ACCEL_B200_EINVAL, "matmul_q8: weight tensor map rejected");
  }
  const int32_t* row_exp = nullptr;
  if (p.mode == kAPlanes) {
    auto* planes = static_cast<uint8_t*>(workspace) + kCounterRegion;
    auto* exps = reinterpret_cast<int32_t*>(planes + p.digits_bytes);
    row_exp = exps;
    // Threads per (row, segment): enough for kDigitQuads quads each.
    const int64_t seg = static_cast<int64_t>(p.kb_per_split) * kBk;
    const int64_t quads = Min64(seg, k) / 4;
    int group_log2 = 5;
    while (group_log2 < 8 && (int64_t{1} << group_log2) * kDigitQuads < quads) ++group_log2;
    const int64_t items = m * p.splits;
    const int64_t groups = kDigitThreads >> group_log2;
    const dim3 grid(static_cast<unsigned>(Min64(CeilDiv(items, groups), kSms * 16)));
    const int64_t nseg = p.splits;
    const float* none = nullptr;
    int rc;
    if (gamma != nullptr) {
      rc = CheckLaunchEx(LaunchK(DigitPlanesKernel<kANorm>, grid, dim3(kDigitThreads), 0, stream, 1u, 1u, a, none, lda,
                                 gamma, eps, m, k, p.kp, seg, nseg, planes, exps, group_log2),
                         "matmul_q8_digits_norm");
    } else if (up != nullptr) {
      rc = CheckLaunchEx(LaunchK(DigitPlanesKernel<kASilu>, grid, dim3(kDigitThreads), 0, stream, 1u, 1u, a, up, lda,
                                 none, 0.f, m, k, p.kp, seg, nseg, planes, exps, group_log2),
                         "matmul_q8_digits_silu");
    } else {
      rc = CheckLaunchEx(LaunchK(DigitPlanesKernel<kAF32>, grid, dim3(kDigitThreads), 0, stream, 1u, 1u, a, none, lda,
                                 none, 0.f, m, k, p.kp, seg, nseg, planes, exps, group_log2),
                         "matmul_q8_digits");
    }
    if (rc != ACCEL_B200_OK) return rc;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(m), kDigits};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(p.kp), static_cast<cuuint64_t>(m) * p.kp};
    const cuuint32_t box[3] = {kBk, static_cast<cuuint32_t>(p.r), kDigits};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (EncodeFn()(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, planes, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      return SetError(ACCEL_B200_EINVAL, "matmul_q8: activation tensor map rejected");
    }
  } else {
    // fp32 tiles [R rows x 128 k]; rows and k beyond the matrix read as zero.
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
  g.up = up;
  g.lda = lda;
  g.gamma = gamma;
  g.eps = eps;
  g.sq_in = sq_in;
  g.sq_ld = sq_ld;
  g.sq_n = sq_n;
  g.row_exp = row_exp;
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
  g.silu_pairs = silu_pairs ? 1 : 0;
  g.ep = ep;
  g.res_vec = (ep.residual != nullptr && reinterpret_cast<uintptr_t>(ep.residual) % 16 == 0 && ep.residual_ld % 4 == 0)
                  ? 1 : 0;
  g.peers = peers != nullptr ? *peers : PeerOut{};
  for (int i = 0; i < g.peers.n; ++i) {
    if (reinterpret_cast<uintptr_t>(g.peers.c[i]) % 16 != 0) g.vec_store = 0;
  }
  switch (p.mode) {
    case kAPlanes: return LaunchTcPlanes(tw, tx, g, p, stream);
    default:
      g.amode = p.mode;
      return LaunchTcRows(tw, tx, tu, g, p, stream);
  }
}

}  // namespace accel_b200
