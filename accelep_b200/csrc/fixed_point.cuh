// The 30-bit fixed point of the int8 tensor-core products (gemm_tc.cu): the
// operand formed inside the product kernel and the one the digit pass writes
// use the same helpers, so both form the same integers from the same fp32
// values.
//
// A row segment is scaled by a power of two against its largest magnitude:
// with e the smallest exponent such that every |y| < 2^e, X = rint(y * 2^(30 -
// e)); X is split into four balanced base-256 digits (int8, X = d0 2^24 + d1
// 2^16 + d2 2^8 + d3), the MMA's digit planes. After the integer products,
// the planes recombine exactly in int64, round once to fp32 and scale back by
// 2^(e - 30).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace accel_b200 {

constexpr int kDigits = 4;           // int8 digits per fixed-point activation
constexpr int kExpMin = -96;         // smallest row exponent: keeps 2^(30 - e) a normal float
constexpr int32_t kBadRow = 0x7fff;  // exponent of a row holding Inf or NaN

// Largest |y| of four values as float bits: unsigned order is magnitude order
// for non-negative floats, and Inf and NaN order above every finite value.
__device__ __forceinline__ uint32_t AbsMaxBits(float4 y) {
  const uint32_t a = __float_as_uint(y.x) & 0x7fffffffu, b = __float_as_uint(y.y) & 0x7fffffffu;
  const uint32_t c = __float_as_uint(y.z) & 0x7fffffffu, d = __float_as_uint(y.w) & 0x7fffffffu;
  return max(max(a, b), max(c, d));
}

// The exponent e of a row whose largest |y| has float bits `amax`: every |y|
// < 2^e (e >= kExpMin), or kBadRow when the row holds Inf or NaN.
__device__ __forceinline__ int32_t RowExponent(uint32_t amax) {
  if (amax >= 0x7f800000u) return kBadRow;
  const int32_t e = static_cast<int32_t>(amax >> 23) - 126;
  return e < kExpMin ? kExpMin : e;
}

// 2^(30 - e) as a float (exact: 30 - e lies in [-98, 126]).
__device__ __forceinline__ float FixScale(int32_t e) { return __int_as_float((127 + 30 - e) << 23); }

// The digit planes of four consecutive elements: word p holds digit p of the
// four fixed-point values, byte i for element i. For one value, (X + 0x808080)
// carries the balanced form's carries into bytes 1 .. 3, so XOR 0x808080 of it
// holds the digits [d3, d2, d1, d0] in bytes 0 .. 3 (d3 = X mod 256 read as a
// signed byte); a 4 x 4 byte transpose then gathers each digit's bytes.
__device__ __forceinline__ void FourDigits(float4 y, float s, uint32_t (&w)[kDigits]) {
  const auto word = [s](float v) {
    return (static_cast<uint32_t>(__float2int_rn(__fmul_rn(v, s))) + 0x808080u) ^ 0x808080u;
  };
  const uint32_t v0 = word(y.x), v1 = word(y.y), v2 = word(y.z), v3 = word(y.w);
  const uint32_t t0 = __byte_perm(v0, v1, 0x5140), t1 = __byte_perm(v0, v1, 0x7362);  // bytes 0,1 | 2,3 of v0, v1
  const uint32_t t2 = __byte_perm(v2, v3, 0x5140), t3 = __byte_perm(v2, v3, 0x7362);
  w[3] = __byte_perm(t0, t2, 0x5410);
  w[2] = __byte_perm(t0, t2, 0x7632);
  w[1] = __byte_perm(t1, t3, 0x5410);
  w[0] = __byte_perm(t1, t3, 0x7632);
}

// The product of a row segment with exponent e from its four digit-plane sums
// (int32 each, exact): recombined in int64, rounded once to fp32, scaled by
// 2^(e - 30) (exact: a normal float for every exponent a row takes); NaN for
// a segment that held Inf or NaN.
__device__ __forceinline__ float PlanesToFloat(int32_t d0, int32_t d1, int32_t d2, int32_t d3, int32_t e) {
  long long sum = static_cast<long long>(d3);
  sum += static_cast<long long>(d2) * 256;
  sum += static_cast<long long>(d1) * 65536;
  sum += static_cast<long long>(d0) * 16777216;
  const float t = __ll2float_rn(sum);
  return e == kBadRow ? __int_as_float(0x7fc00000) : __fmul_rn(t, __int_as_float((127 - 30 + e) << 23));
}

}  // namespace accel_b200
