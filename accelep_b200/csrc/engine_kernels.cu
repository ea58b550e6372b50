// Kernels of the batched Llama decode loop that fuse several reference calls:
//
//  * RopeAppendKernel: Rope on the query heads, Rope on the key heads, and
//    AppendCache of the key and value rows (src/llama_model.cc:229-232) in one
//    pass over the fused q|k|v projection rows. Each row carries its own
//    sequence slot and absolute position, so prefill rows of many sequences
//    and one decode row per sequence use the same kernel. A row with position
//    < 0 belongs to a finished sequence and writes nothing.
//  * SiluMulRowsKernel: SiluMul (src/sim_silu.cc:8-13) over the fused
//    gate|up projection rows into a separate activation buffer.
//  * GreedyStepKernel: the per-step bookkeeping of Generate
//    (src/llama_model.cc:113-128) for every sequence at once: argmax of the
//    logit row (or an id already drawn by the sampling kernel), record the
//    id, stop on eos or a full context, and otherwise set the next row's
//    token and position.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "accel_b200.h"
#include "common.cuh"

namespace accel_b200 {
namespace {

// One CTA per row. Query pairs are rotated in place; key pairs are rotated
// into the cache; value rows are copied into the cache.
__global__ void RopeAppendKernel(float* __restrict__ qkv, int64_t ld, const int32_t* __restrict__ row_seq,
                                 const int32_t* __restrict__ row_pos, int32_t heads, int32_t kv_heads,
                                 int32_t head_dim, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                 float* __restrict__ k_cache, float* __restrict__ v_cache, int64_t seq_stride,
                                 int64_t head_stride, int64_t row_stride) {
  const int64_t r = blockIdx.x;
  const int64_t pos = row_pos[r];
  if (pos < 0) return;
  const int64_t seq = row_seq != nullptr ? row_seq[r] : 0;
  const int half = head_dim / 2;
  const float* c = cos_t + pos * head_dim;
  const float* s = sin_t + pos * head_dim;
  float* row = qkv + r * ld;
  const int64_t kvd = static_cast<int64_t>(kv_heads) * head_dim;
  float* kslot = k_cache + seq * seq_stride + pos * row_stride;
  float* vslot = v_cache + seq * seq_stride + pos * row_stride;
  const int q_pairs = heads * half, k_pairs = kv_heads * half;
  for (int p = threadIdx.x; p < q_pairs; p += blockDim.x) {
    const int h = p / half, i = p % half;
    float* x = row + h * head_dim;
    float lo, hi;
    RopePair(x[i], x[half + i], c, s, i, half, &lo, &hi);
    x[i] = lo;
    x[half + i] = hi;
  }
  const float* kin = row + static_cast<int64_t>(heads) * head_dim;
  for (int p = threadIdx.x; p < k_pairs; p += blockDim.x) {
    const int h = p / half, i = p % half;
    const float* x = kin + h * head_dim;
    float lo, hi;
    RopePair(x[i], x[half + i], c, s, i, half, &lo, &hi);
    kslot[h * head_stride + i] = lo;
    kslot[h * head_stride + half + i] = hi;
  }
  const float* vin = kin + kvd;
  for (int64_t i = threadIdx.x; i < kvd; i += blockDim.x) vslot[(i / head_dim) * head_stride + i % head_dim] = vin[i];
}

__global__ void SiluMulRowsKernel(const float* __restrict__ gu, int64_t ld, float* __restrict__ out, int64_t ldo,
                                  int64_t rows, int64_t inter) {
  PdlTrigger();
  PdlWait();
  const int64_t total = rows * inter;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = idx / inter, i = idx - r * inter;
    const float g = gu[r * ld + i];
    const float u = gu[r * ld + inter + i];
    out[r * ldo + i] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, expf(-g))), u);
  }
}

// Per sequence b (one CTA each):
//   id = argmax(logits[b]) (first maximum; NaN never wins; NaN at id 0 -> 0)
//   ids[b * ids_stride + step] = id; count[b] = step + 1
//   if id == eos or lens[b] >= context: the sequence is done (row_pos = -1)
//   else: tokens[b] = id; row_pos[b] = lens[b]; lens[b] += 1 (the new row)
// Sequences already done keep row_pos = -1 and record nothing. `step` is a
// device counter advanced by the last CTA to finish, so the same launch can
// be replayed from a CUDA graph.
struct Best {
  float v;
  int32_t i;
};

__device__ __forceinline__ Best BetterOf(Best a, Best b) {
  if (a.i < 0) return b;
  if (b.i < 0) return a;
  if (b.v > a.v) return b;
  if (a.v > b.v) return a;
  return b.i < a.i ? b : a;
}

__global__ void GreedyStepKernel(const float* __restrict__ logits, const int32_t* __restrict__ pre_ids, int64_t vocab,
                                 int64_t ld, int32_t* ids,
                                 int64_t ids_stride, int32_t* count, int32_t* done, int32_t* tokens, int32_t* row_pos,
                                 int32_t* lens, int32_t eos, int32_t context, int32_t* step, int32_t* finished,
                                 int32_t batch) {
  __shared__ Best red[32];
  __shared__ int32_t last;
  PdlTrigger();
  PdlWait();
  const int b = blockIdx.x;
  const int32_t n = *step;
  const bool live = done[b] == 0;
  if (live && pre_ids != nullptr) {
    if (threadIdx.x == 0) {
      const int32_t id = pre_ids[b];
      ids[static_cast<int64_t>(b) * ids_stride + n] = id;
      count[b] = n + 1;
      if (id == eos || lens[b] >= context) {
        done[b] = 1;
        row_pos[b] = -1;
        atomicAdd(finished, 1);
      } else {
        tokens[b] = id;
        row_pos[b] = lens[b];
        lens[b] += 1;
      }
    }
  } else if (live) {
    const float* row = logits + static_cast<int64_t>(b) * ld;
    Best mine{0.f, -1};
    const auto take = [&mine](float v, int64_t i) {
      if (!isnan(v) && (mine.i < 0 || v > mine.v)) mine = Best{v, static_cast<int32_t>(i)};
    };
    int64_t tail = 0;
    if (ld % 4 == 0 && reinterpret_cast<uintptr_t>(logits) % 16 == 0) {
      // 16-byte loads, four per thread in flight; a thread's indices rise, so
      // its first maximum is kept.
      const float4* row4 = reinterpret_cast<const float4*>(row);
      const int64_t n4 = vocab / 4, bd = blockDim.x;
      for (int64_t base = threadIdx.x; base < n4; base += 4 * bd) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          v[u] = base + u * bd < n4 ? __ldg(row4 + base + u * bd) : make_float4(NAN, NAN, NAN, NAN);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int64_t i = 4 * (base + u * bd);
          take(v[u].x, i);
          take(v[u].y, i + 1);
          take(v[u].z, i + 2);
          take(v[u].w, i + 3);
        }
      }
      tail = 4 * n4;
    }
    for (int64_t i = tail + threadIdx.x; i < vocab; i += blockDim.x) take(row[i], i);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      Best y{__shfl_xor_sync(kFull, mine.v, o), __shfl_xor_sync(kFull, mine.i, o)};
      mine = BetterOf(mine, y);
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mine;
    __syncthreads();
    if (threadIdx.x == 0) {
      Best best{0.f, -1};
      for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) best = BetterOf(best, red[w]);
      int32_t id = best.i < 0 ? 0 : best.i;
      if (isnan(row[0])) id = 0;
      ids[static_cast<int64_t>(b) * ids_stride + n] = id;
      count[b] = n + 1;
      if (id == eos || lens[b] >= context) {
        done[b] = 1;
        row_pos[b] = -1;
        atomicAdd(finished, 1);
      } else {
        tokens[b] = id;
        row_pos[b] = lens[b];
        lens[b] += 1;
      }
    }
  } else if (threadIdx.x == 0) {
    row_pos[b] = -1;
  }
  // The last CTA advances the step counter.
  if (threadIdx.x == 0) {
    __threadfence();
    const int32_t arrived = atomicAdd(step + 1, 1);
    last = arrived == batch - 1;
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    step[1] = 0;
    __threadfence();
    step[0] = n + 1;
  }
}

__global__ void GatherRowsKernel(const float* __restrict__ src, int64_t ld, const int32_t* __restrict__ idx,
                                 int64_t cols, float* __restrict__ dst, int64_t ldd) {
  const float* s = src + static_cast<int64_t>(idx[blockIdx.x]) * ld;
  float* d = dst + static_cast<int64_t>(blockIdx.x) * ldd;
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) d[i] = s[i];
}

}  // namespace

int LaunchSiluMulRows(const float* gate_up, int64_t ld, float* out, int64_t ldo, int64_t rows, int64_t inter,
                      cudaStream_t stream) {
  if (rows < 0 || inter < 0 || ld < 2 * inter || ldo < inter) return SetError(ACCEL_B200_EINVAL, "silu_mul_rows: bad arguments");
  if (rows * inter == 0) return ClearError();
  const int64_t blocks = CeilDiv(rows * inter, 256);
  const int grid = static_cast<int>(blocks < kSms * 8 ? blocks : kSms * 8);
  return CheckLaunchEx(LaunchK(SiluMulRowsKernel, dim3(grid), dim3(256), 0, stream, 1u, 1u, gate_up, ld, out, ldo, rows,
                               inter),
                       "silu_mul_rows");
}
}  // namespace accel_b200

using namespace accel_b200;

extern "C" {

ACCEL_B200_API int accel_b200_rope_append(float* qkv, int64_t qkv_ld, const int32_t* row_seq, const int32_t* row_pos,
                                          int64_t rows, int32_t heads, int32_t kv_heads, int32_t head_dim,
                                          const float* cos_table, const float* sin_table, float* k_cache,
                                          float* v_cache, int64_t cache_seq_stride, int64_t cache_head_stride,
                                          int64_t cache_row_stride, void* stream) {
  if (rows < 0 || heads <= 0 || kv_heads <= 0 || head_dim <= 0 || head_dim % 2 != 0 || row_pos == nullptr ||
      qkv_ld < static_cast<int64_t>(heads + 2 * kv_heads) * head_dim) {
    return SetError(ACCEL_B200_EINVAL, "rope_append: bad arguments");
  }
  if (rows == 0) return ClearError();
  if (rows > 2147483647LL) return SetError(ACCEL_B200_EINVAL, "rope_append: too many rows");
  RopeAppendKernel<<<static_cast<unsigned>(rows), 128, 0, AsStream(stream)>>>(
      qkv, qkv_ld, row_seq, row_pos, heads, kv_heads, head_dim, cos_table, sin_table, k_cache, v_cache,
      cache_seq_stride, cache_head_stride, cache_row_stride);
  return CheckLaunch("rope_append");
}

ACCEL_B200_API int accel_b200_silu_mul_rows(const float* gate_up, int64_t ld, float* out, int64_t ldo, int64_t rows,
                                            int64_t inter, void* stream) {
  return LaunchSiluMulRows(gate_up, ld, out, ldo, rows, inter, AsStream(stream));
}

ACCEL_B200_API int accel_b200_greedy_step(const float* logits, const int32_t* pre_ids, int64_t vocab, int64_t ld,
                                          int32_t* ids,
                                          int64_t ids_stride, int32_t* count, int32_t* done, int32_t* tokens,
                                          int32_t* row_pos, int32_t* lens, int32_t eos, int32_t context,
                                          int32_t* step, int32_t* finished, int32_t batch, void* stream) {
  if (batch <= 0 || vocab <= 0 || ld < vocab || step == nullptr) return SetError(ACCEL_B200_EINVAL, "greedy_step: bad arguments");
  return CheckLaunchEx(LaunchK(GreedyStepKernel, dim3(batch), dim3(1024), 0, AsStream(stream), 1u, 1u, logits, pre_ids,
                               vocab, ld, ids, ids_stride, count, done, tokens, row_pos, lens, eos, context, step,
                               finished, batch),
                       "greedy_step");
}

ACCEL_B200_API int accel_b200_gather_rows(const float* src, int64_t ld, const int32_t* idx, int64_t rows, int64_t cols,
                                          float* dst, int64_t ldd, void* stream) {
  if (rows < 0 || cols < 0 || ld < cols || ldd < cols) return SetError(ACCEL_B200_EINVAL, "gather_rows: bad arguments");
  if (rows == 0 || cols == 0) return ClearError();
  if (rows > 2147483647LL) return SetError(ACCEL_B200_EINVAL, "gather_rows: too many rows");
  GatherRowsKernel<<<static_cast<unsigned>(rows), 256, 0, AsStream(stream)>>>(src, ld, idx, cols, dst, ldd);
  return CheckLaunch("gather_rows");
}

}  // extern "C"
