// Next-token choice (src/sim_sample.cc:25-115) on the device.
//
// Greedy rows: one CTA per row, a (value, id) reduction in which NaN never
// wins and the earlier id wins a tie, which is what the reference's
// sequential `logits[i] > best_v` scan computes (a NaN at id 0 pins the
// answer to 0, as it does there).
//
// Sampled rows: one CTA per row. The top-k table is the top min(top_k, 64)
// logits ordered by (logit descending, id ascending), which is the set the
// reference's evict-the-worst scan keeps; it is then walked in id order with
// the same double arithmetic in one thread. The full-vocabulary draw sums in
// double in parallel and finds the crossing in the prefix sums.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "accel_b200.h"
#include "common.cuh"

namespace accel_b200 {
namespace {

constexpr int kSampleThreads = 1024;

struct Best {
  float v;
  int32_t i;  // -1: no candidate
};

__device__ __forceinline__ Best Better(Best a, Best b) {
  if (a.i < 0) return b;
  if (b.i < 0) return a;
  if (b.v > a.v) return b;
  if (a.v > b.v) return a;
  return b.i < a.i ? b : a;
}

__device__ __forceinline__ Best WarpBest(Best x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Best y;
    y.v = __shfl_xor_sync(kFull, x.v, o);
    y.i = __shfl_xor_sync(kFull, x.i, o);
    x = Better(x, y);
  }
  return x;
}

// Block-wide best over per-thread candidates. All threads get the result.
__device__ Best BlockBest(Best x, Best* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
  x = WarpBest(x);
  __syncthreads();
  if (lane == 0) scratch[warp] = x;
  __syncthreads();
  if (warp == 0) {
    Best y = lane < warps ? scratch[lane] : Best{0.f, -1};
    y = WarpBest(y);
    if (lane == 0) scratch[32] = y;
  }
  __syncthreads();
  return scratch[32];
}

// `after` excludes every id ranked at or above (after_v, after_i) in the
// (logit desc, id asc) order; after_i < 0 excludes nothing.
__device__ Best RowBest(const float* row, int64_t vocab, float after_v, int32_t after_i, Best* scratch) {
  Best mine{0.f, -1};
  for (int64_t i = threadIdx.x; i < vocab; i += blockDim.x) {
    const float v = row[i];
    if (isnan(v)) continue;
    if (after_i >= 0 && !(v < after_v || (v == after_v && i > after_i))) continue;
    if (mine.i < 0 || v > mine.v) mine = Best{v, static_cast<int32_t>(i)};
  }
  return BlockBest(mine, scratch);
}

__global__ void ArgmaxRowsKernel(const float* __restrict__ logits, int64_t vocab, int64_t ld, int32_t* chosen,
                                 int64_t chosen_stride, int64_t chosen_offset) {
  __shared__ Best scratch[33];
  const float* row = logits + static_cast<int64_t>(blockIdx.x) * ld;
  Best b = RowBest(row, vocab, 0.f, -1, scratch);
  if (threadIdx.x == 0) {
    int32_t id = b.i < 0 ? 0 : b.i;
    if (isnan(row[0])) id = 0;
    chosen[static_cast<int64_t>(blockIdx.x) * chosen_stride + chosen_offset] = id;
  }
}

__device__ __forceinline__ uint32_t NextRand(uint32_t x) {
  x ^= x << 13;
  x ^= x >> 17;
  x ^= x << 5;
  return x;
}

__global__ void SampleRowsKernel(const float* __restrict__ logits, int64_t vocab, int64_t ld, int32_t* chosen,
                                 int64_t chosen_stride, int64_t chosen_offset, float temperature, uint32_t* rng,
                                 int32_t top_k) {
  __shared__ Best scratch[33];
  __shared__ Best table[64];
  __shared__ double part[kSampleThreads];
  __shared__ int32_t found;
  const int64_t r = blockIdx.x;
  const float* row = logits + r * ld;
  int32_t* out = chosen + r * chosen_stride + chosen_offset;
  uint32_t* state = rng + r;
  const int tid = threadIdx.x;

  if (!(temperature > 0.f)) {
    Best b = RowBest(row, vocab, 0.f, -1, scratch);
    if (tid == 0) *out = (b.i < 0 || isnan(row[0])) ? 0 : b.i;
    return;
  }
  const bool full = top_k <= 0 || static_cast<int64_t>(top_k) >= vocab;
  const double inv_t = 1.0 / static_cast<double>(temperature);
  if (!full) {
    const int capped = top_k > 64 ? 64 : top_k;
    // A NaN among the first `capped` ids stays in the reference's table and
    // makes its sum NaN: the answer is id 0 and the state is not advanced.
    bool nan_head = false;
    for (int i = tid; i < capped; i += blockDim.x) nan_head |= isnan(row[i]) != 0;
    nan_head = __syncthreads_or(nan_head);
    if (nan_head) {
      if (tid == 0) *out = 0;
      return;
    }
    float after_v = 0.f;
    int32_t after_i = -1;
    for (int s = 0; s < capped; ++s) {
      const Best b = RowBest(row, vocab, after_v, after_i, scratch);
      if (tid == 0) table[s] = b;
      after_v = b.v;
      after_i = b.i;
    }
    __syncthreads();
    if (tid == 0) {
      // Id order, then the reference's max / sum / walk (sim_sample.cc:68-114).
      for (int i = 1; i < capped; ++i) {
        const Best key = table[i];
        int j = i;
        while (j > 0 && table[j - 1].i > key.i) {
          table[j] = table[j - 1];
          --j;
        }
        table[j] = key;
      }
      float max_v = table[0].v;
      for (int s = 1; s < capped; ++s)
        if (table[s].v > max_v) max_v = table[s].v;
      double sum = 0.0;
      for (int s = 0; s < capped; ++s) sum += exp((static_cast<double>(table[s].v) - static_cast<double>(max_v)) * inv_t);
      if (!(sum > 0.0)) {
        *out = 0;
        return;
      }
      const uint32_t x = NextRand(*state);
      *state = x;
      const double draw = (static_cast<double>(x) + 0.5) / 4294967296.0 * sum;
      double acc = 0.0;
      for (int s = 0; s < capped; ++s) {
        acc += exp((static_cast<double>(table[s].v) - static_cast<double>(max_v)) * inv_t);
        if (acc >= draw) {
          *out = table[s].i;
          return;
        }
      }
      *out = table[capped - 1].i;
    }
    return;
  }
  // Whole vocabulary. max_v follows the reference scan: logits[0] first,
  // NaN never replaces it (a NaN at id 0 makes every term NaN).
  Best b = RowBest(row, vocab, 0.f, -1, scratch);
  const float max_v = isnan(row[0]) ? row[0] : b.v;
  // Contiguous chunk per thread so the prefix order follows id order.
  const int64_t chunk = (vocab + blockDim.x - 1) / blockDim.x;
  const int64_t lo = tid * chunk;
  const int64_t hi = lo + chunk < vocab ? lo + chunk : vocab;
  double mine = 0.0;
  for (int64_t i = lo; i < hi; ++i) mine += exp((static_cast<double>(row[i]) - static_cast<double>(max_v)) * inv_t);
  part[tid] = mine;
  __syncthreads();
  // Inclusive scan of the chunk sums (Hillis-Steele over kSampleThreads).
  for (int off = 1; off < kSampleThreads; off <<= 1) {
    const double add = tid >= off ? part[tid - off] : 0.0;
    __syncthreads();
    part[tid] += add;
    __syncthreads();
  }
  const double sum = part[blockDim.x - 1];
  if (!(sum > 0.0)) {
    if (tid == 0) *out = 0;
    return;
  }
  __shared__ double draw_s;
  if (tid == 0) {
    const uint32_t x = NextRand(*state);
    *state = x;
    draw_s = (static_cast<double>(x) + 0.5) / 4294967296.0 * sum;
    found = -1;
  }
  __syncthreads();
  const double draw = draw_s;
  const double before = tid == 0 ? 0.0 : part[tid - 1];
  if (before < draw && part[tid] >= draw) {
    double acc = before;
    int32_t pick = static_cast<int32_t>(hi - 1);
    for (int64_t i = lo; i < hi; ++i) {
      acc += exp((static_cast<double>(row[i]) - static_cast<double>(max_v)) * inv_t);
      if (acc >= draw) {
        pick = static_cast<int32_t>(i);
        break;
      }
    }
    found = pick;  // the prefix sums are monotone: exactly one thread crosses
  }
  __syncthreads();
  if (tid == 0) *out = found >= 0 ? found : static_cast<int32_t>(vocab - 1);
}

}  // namespace
}  // namespace accel_b200

using namespace accel_b200;

extern "C" {

ACCEL_B200_API int accel_b200_argmax_rows(const float* logits, int64_t rows, int64_t vocab, int64_t ld, int32_t* chosen,
                                          int64_t chosen_stride, int64_t chosen_offset, void* stream) {
  if (rows < 0 || vocab <= 0 || ld < vocab || chosen_offset < 0) return SetError(ACCEL_B200_EINVAL, "argmax: bad size");
  if (rows == 0) return ClearError();
  if (rows > 2147483647LL) return SetError(ACCEL_B200_EINVAL, "argmax: too many rows");
  if (logits == nullptr || chosen == nullptr) return SetError(ACCEL_B200_EINVAL, "argmax: null pointer");
  ArgmaxRowsKernel<<<static_cast<unsigned>(rows), 1024, 0, AsStream(stream)>>>(logits, vocab, ld, chosen, chosen_stride,
                                                                              chosen_offset);
  return CheckLaunch("argmax_rows");
}

ACCEL_B200_API int accel_b200_sample(const float* logits, int32_t* chosen, int64_t chosen_index, int64_t vocab,
                                     float temperature, uint32_t* rng_state, int32_t top_k, void* stream) {
  if (vocab <= 0 || chosen_index < 0 || vocab > 2147483647LL) return SetError(ACCEL_B200_EINVAL, "SampleToken is out of range");
  if (logits == nullptr || chosen == nullptr) return SetError(ACCEL_B200_EINVAL, "SampleToken is out of range");
  if (rng_state == nullptr) return SetError(ACCEL_B200_EINVAL, "SampleToken rng is out of range");
  SampleRowsKernel<<<1, kSampleThreads, 0, AsStream(stream)>>>(logits, vocab, vocab, chosen, 0, chosen_index,
                                                               temperature, rng_state, top_k);
  return CheckLaunch("sample");
}

ACCEL_B200_API int accel_b200_sample_rows(const float* logits, int64_t rows, int64_t vocab, int64_t ld, int32_t* chosen,
                                          int64_t chosen_stride, int64_t chosen_offset, float temperature,
                                          uint32_t* rng_states, int32_t top_k, void* stream) {
  if (rows < 0 || vocab <= 0 || ld < vocab || vocab > 2147483647LL || rows > 2147483647LL)
    return SetError(ACCEL_B200_EINVAL, "sample_rows: bad size");
  if (rows == 0) return ClearError();
  if (logits == nullptr || chosen == nullptr || rng_states == nullptr) return SetError(ACCEL_B200_EINVAL, "sample_rows: null pointer");
  SampleRowsKernel<<<static_cast<unsigned>(rows), kSampleThreads, 0, AsStream(stream)>>>(
      logits, vocab, ld, chosen, chosen_stride, chosen_offset, temperature, rng_states, top_k);
  return CheckLaunch("sample_rows");
}

}  // extern "C"
