// One decode step of a layer's attention for a batch of sequences, fused:
// RoPE of the new query and key rows (src/sim_rope.cc:16-17), the append of
// the new key and value rows to the cache (src/sim_cache.cc) and causal
// grouped-query attention over the whole context (src/sim_attend.cc:9-46),
// as Generate runs them per token (src/llama_model.cc:229-233).
//
// Layout. The cache is head-major: slot b, kv head g, position t at
// k_cache + b * seq_stride + g * head_stride + t * 64 (floats), so the rows of
// one (sequence, kv head) are one contiguous block. head_dim is 64.
//
// Work split. One thread-block cluster of S CTAs per (sequence, kv head); the
// context's 64-row chunks are dealt to the S ranks in contiguous ranges. A
// CTA streams its chunks through two shared-memory buffers with bulk copies
// (the next chunk is in flight while the current one is scored), keeps an
// online softmax (reference maximum, sum and weighted values) for the G query heads
// of its kv head, and publishes that state in shared memory. The cluster then
// merges the S states in rank order through distributed shared memory
// (log-sum-exp rule), so the result does not depend on scheduling and no
// workspace or counters are needed. The rank whose range holds the new row
// computes it (RoPE on the key), writes it to the cache and places it in its
// buffer instead of copying it.
//
// Rows with position < 0 (finished sequences) do nothing. Every mbarrier wait
// is bounded; a wait that runs out sets ACCEL_B200_STATUS_COPY_TIMEOUT and the
// CTA still reaches the cluster barriers.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <mutex>
#include <string>

#include "accel_b200.h"
#include "cluster.cuh"
#include "common.cuh"
#include "tma.cuh"

namespace accel_b200 {
namespace {

constexpr int kD = 64;          // head_dim
constexpr int kRows = 64;       // context rows per chunk
constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxG = 8;        // query heads per kv head
constexpr int kMaxSplit = 8;    // CTAs per cluster
constexpr float kSlack = 8.f;   // how far a score may pass a warp's softmax reference before it moves
constexpr int kChunkFloats = kRows * kD;
constexpr int kSmemBytes = 2 * 2 * kChunkFloats * 4;  // two buffers of K and V

struct FusedArgs {
  const float* qkv;  // row r: heads * 64 query | kv_heads * 64 key | kv_heads * 64 value (before RoPE)
  int64_t qkv_ld;
  const int32_t* row_seq;  // cache slot of row r; null: slot r
  const int32_t* row_pos;  // position of row r's token; < 0: finished, skipped
  const float* cos_t;      // [context][64]
  const float* sin_t;
  float* k_cache;
  float* v_cache;
  int64_t seq_stride;
  int64_t head_stride;
  int32_t heads;
  int32_t kv_heads;
  int32_t context;
  float scale;
  float* out;  // row r: heads * 64 at out + r * out_ld
  int64_t out_ld;
  int32_t* status;
  accel_b200_l2_prefetch prefetch;  // ranges brought into L2 before the wait (count 0: none)
};

constexpr int64_t kPrefetchChunk = 32 * 1024;  // bytes per L2 prefetch instruction

// This CTA's share of the prefetch ranges: chunk c of the ranges' 32 KiB
// chunks goes to CTA c mod (CTAs).
__device__ __forceinline__ void PrefetchShare(const accel_b200_l2_prefetch& pf) {
  const int64_t cta = blockIdx.x + static_cast<int64_t>(gridDim.x) * (blockIdx.y + static_cast<int64_t>(gridDim.y) *
                                                                                       blockIdx.z);
  const int64_t ctas = static_cast<int64_t>(gridDim.x) * gridDim.y * gridDim.z;
  for (int i = 0; i < pf.count && i < 4; ++i) {
    const char* base = static_cast<const char*>(pf.ptr[i]);
    for (int64_t off = cta * kPrefetchChunk; off < pf.bytes[i]; off += ctas * kPrefetchChunk) {
      const uint32_t n = static_cast<uint32_t>(Min64(kPrefetchChunk, pf.bytes[i] - off)) & ~15u;
      if (n > 0) PrefetchL2(base + off, n);
    }
  }
}

template <int G>
__global__ void __launch_bounds__(kThreads, 3) AttnDecodeFusedKernel(FusedArgs a) {
  extern __shared__ __align__(128) float buf[];  // [2][K | V][64 rows][64]
  __shared__ __align__(8) uint64_t full[2], full_v[2], empty[2];  // keys landed, values landed, buffer free
  __shared__ __align__(16) float qs[G * kD];        // roped query heads
  __shared__ __align__(16) float wo[kWarps][G * kD];  // per-warp weighted values
  __shared__ __align__(16) float ps[kWarps][G][kRows / kWarps];  // per-warp weights of the chunk's rows
  __shared__ float wm[kWarps][G], wl[kWarps][G];    // per-warp running max and sum
  __shared__ __align__(16) float mo[G * kD];        // published weighted values
  __shared__ float m_run[G], l_run[G];
  PdlTrigger();
  // Ranges for later kernels (immutable weights) go to L2 while this kernel
  // waits for its inputs.
  if (threadIdx.x == 0 && a.prefetch.count > 0) PrefetchShare(a.prefetch);
  // The q|k|v rows come from the previous kernel. The row positions, slots
  // and cache rows come from kernels before it: with CACHE_BEFORE_WAIT those
  // have completed when this kernel starts (the previous kernel let it launch
  // only after its own wait), so they are read, and the first chunks' copies
  // issued, before the wait.
  const bool early = (a.prefetch.flags & ACCEL_B200_ATTN_CACHE_BEFORE_WAIT) != 0;
  if (!early) PdlWait();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rank = static_cast<int>(blockIdx.x), S = static_cast<int>(gridDim.x);
  const int g = static_cast<int>(blockIdx.y);
  const int64_t r = blockIdx.z;
  const int64_t pos = a.row_pos[r];
  const int h0 = g * G;

  // The chunk range of this rank.
  const int64_t len = pos + 1;
  const int used = pos >= 0 ? static_cast<int>((len + kRows - 1) / kRows) : 0;
  const int per = (used + S - 1) / S;
  const int c_begin = min(used, rank * per), c_end = min(used, c_begin + per);
  const int nloc = c_end - c_begin;
  const int64_t slot = a.row_seq != nullptr ? a.row_seq[r] : r;
  float* kbase = a.k_cache + slot * a.seq_stride + g * a.head_stride;
  float* vbase = a.v_cache + slot * a.seq_stride + g * a.head_stride;
  const float* row = a.qkv + r * a.qkv_ld;

  if (tid == 0) {
    for (int b = 0; b < 2; ++b) {
      MbarInit(&full[b], 1);
      MbarInit(&full_v[b], 1);
      MbarInit(&empty[b], kWarps);
    }
    FenceBarrierInit();
  }
  __syncthreads();

  // Issues the copies of local chunk i into buffer i & 1, keys and values on
  // their own barriers (the scores need only the keys). The new row (the last
  // of the context) is not copied: the owner writes it.
  auto issue = [&](int i) {
    const int64_t t0 = static_cast<int64_t>(c_begin + i) * kRows;
    const int64_t cnt = Min64(kRows, len - t0);
    const int64_t copy = t0 + cnt == len ? cnt - 1 : cnt;
    float* kb = buf + (i & 1) * 2 * kChunkFloats;
    uint64_t* bar_k = &full[i & 1];
    uint64_t* bar_v = &full_v[i & 1];
    if (copy > 0) {
      // Read once per step: evict first, ahead of the weights the layer's
      // products read next.
      const uint32_t bytes = static_cast<uint32_t>(copy) * kD * 4;
      const uint64_t policy = EvictFirstPolicy();
      MbarArriveExpectTx(bar_k, bytes);
      BulkCopyG2SHint(kb, kbase + t0 * kD, bytes, bar_k, policy);
      MbarArriveExpectTx(bar_v, bytes);
      BulkCopyG2SHint(kb + kChunkFloats, vbase + t0 * kD, bytes, bar_v, policy);
    } else {
      MbarArrive(bar_k);
      MbarArrive(bar_v);
    }
  };
  if (tid == 0) {
    if (nloc > 0) issue(0);
    if (nloc > 1) issue(1);
  }
  if (early) PdlWait();

  // RoPE of the G query heads into shared memory (all ranks need them).
  if (pos >= 0) {
    const float* c = a.cos_t + pos * kD;
    const float* s = a.sin_t + pos * kD;
    for (int p = tid; p < G * (kD / 2); p += kThreads) {
      const int hh = p / (kD / 2), i = p % (kD / 2);
      const float* x = row + static_cast<int64_t>(h0 + hh) * kD;
      float lo, hi;
      RopePair(x[i], x[kD / 2 + i], c, s, i, kD / 2, &lo, &hi);
      qs[hh * kD + i] = lo;
      qs[hh * kD + kD / 2 + i] = hi;
    }
  }
  __syncthreads();

  // Warp w owns rows 16w .. 16w + 15 of every chunk and keeps its own online
  // softmax: lane pair (2j, 2j + 1) scores row 16w + j (each lane over half of
  // the dimensions); the pair's even lane puts the row's weights in shared
  // memory, from which every lane reads four rows' weights per head at once,
  // and lane l accumulates dimensions 2l and 2l + 1 of the weighted values for
  // all G heads. No CTA barrier per chunk: a warp frees a buffer through
  // `empty`, and the producer (thread 0) refills it once all four warps are
  // done with it.
  constexpr int kWarpRows = kRows / kWarps;
  const int wr0 = warp * kWarpRows;
  float m_w[G], l_w[G], o[G][2];
#pragma unroll
  for (int hh = 0; hh < G; ++hh) {
    m_w[hh] = -INFINITY;
    l_w[hh] = 0.f;
    o[hh][0] = 0.f;
    o[hh][1] = 0.f;
  }
  bool ok = true;

  for (int i = 0; i < nloc; ++i) {
    float* kb = buf + (i & 1) * 2 * kChunkFloats;
    float* vb = kb + kChunkFloats;
    const int64_t t0 = static_cast<int64_t>(c_begin + i) * kRows;
    const int cnt = static_cast<int>(Min64(kRows, len - t0));
    ok &= MbarWait(&full[i & 1], (i >> 1) & 1);
    if (t0 + cnt == len && (cnt - 1) / kWarpRows == warp) {
      // The new row lies in this warp's rows: RoPE on its key, append key and
      // value to the cache, and place both in the buffer as row cnt - 1.
      const float* c = a.cos_t + pos * kD;
      const float* s = a.sin_t + pos * kD;
      const float* kin = row + static_cast<int64_t>(a.heads + g) * kD;
      const float* vin = row + static_cast<int64_t>(a.heads + a.kv_heads + g) * kD;
      float lo, hi;
      RopePair(kin[lane], kin[kD / 2 + lane], c, s, lane, kD / 2, &lo, &hi);
      kb[(cnt - 1) * kD + lane] = lo;
      kb[(cnt - 1) * kD + kD / 2 + lane] = hi;
      kbase[pos * kD + lane] = lo;
      kbase[pos * kD + kD / 2 + lane] = hi;
      const float v0 = vin[lane], v1 = vin[lane + 32];
      vb[(cnt - 1) * kD + lane] = v0;
      vb[(cnt - 1) * kD + lane + 32] = v1;
      vbase[pos * kD + lane] = v0;
      vbase[pos * kD + lane + 32] = v1;
      __syncwarp();
    }
    if (wr0 < cnt) {
      // Scores of row j: the float4 index rotates with the row so a
      // quarter-warp hits 32 banks.
      const int j = wr0 + (lane >> 1), half = lane & 1;
      const bool valid = j < cnt;
      float sc[G];
#pragma unroll
      for (int hh = 0; hh < G; ++hh) sc[hh] = 0.f;
      if (valid) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int d4 = half * 8 + ((q + j + 4 * half) & 7);
          const float4 kv = *reinterpret_cast<const float4*>(kb + j * kD + d4 * 4);
#pragma unroll
          for (int hh = 0; hh < G; ++hh) {
            const float4 qv = *reinterpret_cast<const float4*>(qs + hh * kD + d4 * 4);
            sc[hh] = fmaf(qv.x, kv.x, sc[hh]);
            sc[hh] = fmaf(qv.y, kv.y, sc[hh]);
            sc[hh] = fmaf(qv.z, kv.z, sc[hh]);
            sc[hh] = fmaf(qv.w, kv.w, sc[hh]);
          }
        }
      }
      float p[G];
#pragma unroll
      for (int hh = 0; hh < G; ++hh) {
        const float full_dot = sc[hh] + __shfl_xor_sync(kFull, sc[hh], 1);
        const float x = valid ? full_dot * a.scale : -INFINITY;
        // The weights are taken against the warp's reference m_w, which moves
        // to the running maximum only when a score passes it by more than
        // kSlack (always on the warp's first rows, where m_w is -inf): a
        // vote instead of a warp maximum per chunk, and no weight above
        // e^kSlack.
        if (__any_sync(kFull, x > m_w[hh] + kSlack)) {
          const float mx = fmaxf(WarpMax(x), m_w[hh]);  // finite: row wr0 < cnt is valid
          const float corr = expf(m_w[hh] - mx);         // 0 on this warp's first rows
          l_w[hh] *= corr;
          o[hh][0] *= corr;
          o[hh][1] *= corr;
          m_w[hh] = mx;
        }
        p[hh] = valid ? expf(x - m_w[hh]) : 0.f;
        if (half == 0) l_w[hh] += p[hh];  // this lane's rows; summed over the warp after the loop
      }
      const int rows = min(kWarpRows, cnt - wr0);
      ok &= MbarWait(&full_v[i & 1], (i >> 1) & 1);
      if (half == 0) {
#pragma unroll
        for (int hh = 0; hh < G; ++hh) ps[warp][hh][lane >> 1] = p[hh];
      }
      __syncwarp();
      if (rows == kWarpRows) {
        // A full chunk: every row's value load can be issued up front.
#pragma unroll
        for (int r4 = 0; r4 < kWarpRows; r4 += 4) {
          float4 pw[G];
#pragma unroll
          for (int hh = 0; hh < G; ++hh) pw[hh] = *reinterpret_cast<const float4*>(&ps[warp][hh][r4]);
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const float2 v = *reinterpret_cast<const float2*>(vb + (wr0 + r4 + t) * kD + 2 * lane);
#pragma unroll
            for (int hh = 0; hh < G; ++hh) {
              const float pr = t == 0 ? pw[hh].x : t == 1 ? pw[hh].y : t == 2 ? pw[hh].z : pw[hh].w;
              o[hh][0] = fmaf(pr, v.x, o[hh][0]);
              o[hh][1] = fmaf(pr, v.y, o[hh][1]);
            }
          }
        }
      } else {
        for (int r4 = 0; r4 < rows; r4 += 4) {
          float4 pw[G];
#pragma unroll
          for (int hh = 0; hh < G; ++hh) pw[hh] = *reinterpret_cast<const float4*>(&ps[warp][hh][r4]);
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            if (r4 + t < rows) {
              const float2 v = *reinterpret_cast<const float2*>(vb + (wr0 + r4 + t) * kD + 2 * lane);
#pragma unroll
              for (int hh = 0; hh < G; ++hh) {
                const float pr = t == 0 ? pw[hh].x : t == 1 ? pw[hh].y : t == 2 ? pw[hh].z : pw[hh].w;
                o[hh][0] = fmaf(pr, v.x, o[hh][0]);
                o[hh][1] = fmaf(pr, v.y, o[hh][1]);
              }
            }
          }
        }
      }
      __syncwarp();  // the weights are read before the next chunk rewrites them
    } else {
      // No rows of this (last) chunk: still see its values land, so that no
      // copy is in flight into a buffer this warp has released.
      ok &= MbarWait(&full_v[i & 1], (i >> 1) & 1);
    }
    __syncwarp();
    if (lane == 0) MbarArrive(&empty[i & 1]);
    if (tid == 0 && i + 2 < nloc) {
      ok &= MbarWait(&empty[i & 1], (i >> 1) & 1);  // all warps are done with this buffer
      issue(i + 2);
    }
  }
  ok = __syncthreads_and(ok);
  if (!ok) {
    if (tid == 0 && a.status != nullptr) atomicOr(a.status, ACCEL_B200_STATUS_COPY_TIMEOUT);
    // Copies still in flight land before the CTA leaves (bounded waits).
    for (int i = 0; i < nloc && i < 2; ++i) {
      MbarWait(&full[i & 1], ((nloc - 1 - i) >> 1) & 1);
      MbarWait(&full_v[i & 1], ((nloc - 1 - i) >> 1) & 1);
    }
  }
  // The four warp states -> one CTA state (log-sum-exp, warps in order).
#pragma unroll
  for (int hh = 0; hh < G; ++hh) l_w[hh] = WarpSum(l_w[hh]);
#pragma unroll
  for (int hh = 0; hh < G; ++hh) {
    wo[warp][hh * kD + 2 * lane] = o[hh][0];
    wo[warp][hh * kD + 2 * lane + 1] = o[hh][1];
    if (lane == 0) {
      wm[warp][hh] = m_w[hh];
      wl[warp][hh] = l_w[hh];
    }
  }
  __syncthreads();
  for (int e = tid; e < G * kD; e += kThreads) {
    const int hh = e / kD;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, wm[w][hh]);
    float l = 0.f, acc = 0.f;
    if (mx != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float f = expf(wm[w][hh] - mx);
        l = fmaf(wl[w][hh], f, l);
        acc = fmaf(wo[w][e], f, acc);
      }
    }
    mo[e] = acc;
    if ((e & (kD - 1)) == 0) {
      m_run[hh] = mx;
      l_run[hh] = ok ? l : __int_as_float(0x7fc00000);
    }
  }
  ClusterSync();  // every rank's state is published
  if (pos >= 0) {
    // Rank `rank` merges outputs rank, rank + S, ... of the G * 64: every
    // peer's state is loaded first (one round trip), then combined in rank
    // order. A rank whose wait ran out published a NaN sum, so its tile's
    // outputs are NaN (and the status word carries the timeout bit).
    for (int e = rank * kThreads + tid; e < G * kD; e += S * kThreads) {
      const int hh = e / kD;
      float pm[kMaxSplit], pl[kMaxSplit], po[kMaxSplit];
#pragma unroll
      for (int p = 0; p < kMaxSplit; ++p) {
        if (p < S) {
          pm[p] = LoadPeer(&m_run[hh], static_cast<uint32_t>(p));
          pl[p] = LoadPeer(&l_run[hh], static_cast<uint32_t>(p));
          po[p] = LoadPeer(&mo[e], static_cast<uint32_t>(p));
        }
      }
      float mx = -INFINITY;
#pragma unroll
      for (int p = 0; p < kMaxSplit; ++p)
        if (p < S) mx = fmaxf(mx, pm[p]);
      float l = 0.f, o = 0.f;
#pragma unroll
      for (int p = 0; p < kMaxSplit; ++p) {
        if (p < S) {
          const float w = expf(pm[p] - mx);
          l = fmaf(pl[p], w, l);
          o = fmaf(po[p], w, o);
        }
      }
      a.out[r * a.out_ld + static_cast<int64_t>(h0) * kD + e] = o / l;
    }
  }
  ClusterSync();  // no CTA leaves while a peer may still read its state
}

// CTAs per cluster: about 2.5 CTAs per SM over the whole grid, at most one
// per chunk of the longest context and at most 8.
int SplitFor(int64_t rows, int32_t kv_heads, int32_t context) {
  const int64_t pairs = rows * kv_heads;
  int64_t s = CeilDiv(5 * kSms / 2, pairs);
  s = Min64(s, CeilDiv(context, kRows));
  return static_cast<int>(Max64(1, Min64(s, kMaxSplit)));
}

template <int G>
int LaunchFused(const FusedArgs& a, int64_t rows, cudaStream_t stream) {
  static std::once_flag once[16];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 15], [] {
    cudaFuncSetAttribute(AttnDecodeFusedKernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  });
  const int S = SplitFor(rows, a.kv_heads, a.context);
  const dim3 grid(static_cast<unsigned>(S), static_cast<unsigned>(a.kv_heads), static_cast<unsigned>(rows));
  return CheckLaunchEx(LaunchK(AttnDecodeFusedKernel<G>, grid, dim3(kThreads), kSmemBytes, stream,
                               static_cast<unsigned>(S), 1u, a),
                       "decode_attention");
}

}  // namespace
}  // namespace accel_b200

using namespace accel_b200;

extern "C" {

ACCEL_B200_API int accel_b200_decode_attention_prefetch(
    const float* qkv, int64_t qkv_ld, const int32_t* row_seq, const int32_t* row_pos, int64_t rows, int32_t heads,
    int32_t kv_heads, int32_t head_dim, const float* cos_table, const float* sin_table, int32_t context,
    float* k_cache, float* v_cache, int64_t seq_stride, int64_t head_stride, float* out, int64_t out_ld,
    int32_t* status, const accel_b200_l2_prefetch* prefetch, void* stream) {
  if (rows < 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads != 0 || head_dim != kD || context <= 0 ||
      qkv == nullptr || row_pos == nullptr || cos_table == nullptr || sin_table == nullptr || k_cache == nullptr ||
      v_cache == nullptr || out == nullptr) {
    return SetError(ACCEL_B200_EINVAL, "decode_attention: bad arguments (head_dim must be 64)");
  }
  if (rows == 0) return ClearError();
  if (rows > 65535) return SetError(ACCEL_B200_EINVAL, "decode_attention: more than 65535 rows");
  if (qkv_ld < static_cast<int64_t>(heads + 2 * kv_heads) * kD || out_ld < static_cast<int64_t>(heads) * kD) {
    return SetError(ACCEL_B200_EINVAL, "decode_attention: row strides too small");
  }
  if (head_stride < static_cast<int64_t>(context) * kD || seq_stride < head_stride * kv_heads) {
    return SetError(ACCEL_B200_EINVAL, "decode_attention: cache strides do not hold the context");
  }
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) % 16 != 0 || seq_stride % 4 != 0 ||
      head_stride % 4 != 0) {
    return SetError(ACCEL_B200_EINVAL, "decode_attention: cache rows must be 16-byte aligned");
  }
  const int group = heads / kv_heads;
  if (group > kMaxG) return SetError(ACCEL_B200_EINVAL, "decode_attention: more than 8 query heads per kv head");
  accel_b200_l2_prefetch pf{};
  if (prefetch != nullptr) {
    if (prefetch->count < 0 || prefetch->count > 4 || (prefetch->flags & ~ACCEL_B200_ATTN_CACHE_BEFORE_WAIT) != 0) {
      return SetError(ACCEL_B200_EINVAL, "decode_attention: bad prefetch");
    }
    for (int i = 0; i < prefetch->count; ++i) {
      if (prefetch->bytes[i] < 0 || (prefetch->bytes[i] > 0 && prefetch->ptr[i] == nullptr) ||
          reinterpret_cast<uintptr_t>(prefetch->ptr[i]) % 16 != 0) {
        return SetError(ACCEL_B200_EINVAL, "decode_attention: prefetch ranges must be 16-byte aligned");
      }
    }
    pf = *prefetch;
  }
  FusedArgs a{qkv,     qkv_ld,  row_seq,    row_pos,     cos_table, sin_table, k_cache,
              v_cache, seq_stride, head_stride, heads, kv_heads,  context,   1.f / sqrtf(static_cast<float>(kD)),
              out,     out_ld,  status, pf};
  cudaStream_t s = AsStream(stream);
  switch (group) {
    case 1: return LaunchFused<1>(a, rows, s);
    case 2: return LaunchFused<2>(a, rows, s);
    case 3: return LaunchFused<3>(a, rows, s);
    case 4: return LaunchFused<4>(a, rows, s);
    case 5: return LaunchFused<5>(a, rows, s);
    case 6: return LaunchFused<6>(a, rows, s);
    case 7: return LaunchFused<7>(a, rows, s);
    default: return LaunchFused<8>(a, rows, s);
  }
}

ACCEL_B200_API int accel_b200_decode_attention(const float* qkv, int64_t qkv_ld, const int32_t* row_seq,
                                               const int32_t* row_pos, int64_t rows, int32_t heads, int32_t kv_heads,
                                               int32_t head_dim, const float* cos_table, const float* sin_table,
                                               int32_t context, float* k_cache, float* v_cache, int64_t seq_stride,
                                               int64_t head_stride, float* out, int64_t out_ld, int32_t* status,
                                               void* stream) {
  return accel_b200_decode_attention_prefetch(qkv, qkv_ld, row_seq, row_pos, rows, heads, kv_heads, head_dim,
                                              cos_table, sin_table, context, k_cache, v_cache, seq_stride,
                                              head_stride, out, out_ld, status, nullptr, stream);
}

}  // extern "C"
