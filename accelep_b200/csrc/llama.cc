// The Llama engine behind accel_llama_* (include/accel/sim_api.h:39-116 of the
// reference; src/llama_model.cc is the CPU model).
//
// The reference runs a forward as 17 device calls per layer on one
// sequence. Here a forward runs over a set of rows that may belong to many
// sequences (a prefill of several prompts, or one new token per sequence in
// decode). With int8 weights a decode layer is 5 launches:
//
//   q|k|v product (RmsNorm fused into its operand) -> fused RoPE + cache
//   append + attention -> o product (residual add fused) -> gate|up product
//   (RmsNorm fused into its operand, SiluMul into its epilogue) -> down
//   product (residual add fused)
//
// and a prefill layer adds the separate RoPE + append and the tiled prefill
// attention in place of the fused decode attention.
//
// Linear weights live in HBM in the reference's device layout [in, out]
// (src/llama_model.cc:75-84 transposes Hugging Face [out, in]); q, k and v of
// a layer share one [hidden, q + 2 kv] matrix and gate and up one
// [hidden, 2 intermediate] matrix, so each is one product. A weight is fp32
// or int8 with a per-output scale. The KV cache is fp32 and head-major,
// [slot][kv head][context][head_dim] per layer, so one (sequence, kv head)
// run of rows is contiguous for the decode kernel's bulk copies;
// accel_llama_cache_rows returns rows in the reference's [context][kv
// heads][head_dim] layout.
//
// Decode: the step (choose the next id of every live sequence, then one
// forward of one row per sequence) is captured once as a CUDA graph and
// replayed; ids, positions and lengths stay on the device, so the loop needs
// no host round trip per token.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <exception>
#include <map>
#include <memory>
#include <mutex>
#include <new>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

#include "accel_b200.h"
#include "accel_b200_llama.h"
#include "stats.h"
#include "status.h"

namespace accel_b200 {
namespace {

thread_local std::string g_llama_error;

void Fail(const std::string& message) { g_llama_error = message; }
void Clear() { g_llama_error.clear(); }

void Cuda(cudaError_t err, const char* what) {
  if (err == cudaSuccess) return;
  cudaGetLastError();
  if (err == cudaErrorMemoryAllocation) throw std::bad_alloc();
  throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(err));
}

void Abi(int rc) {
  if (rc == ACCEL_B200_OK) return;
  const std::string msg = accel_b200_last_error();
  if (rc == ACCEL_B200_EINVAL || rc == ACCEL_B200_EDEVICE) throw std::invalid_argument(msg);
  if (rc == ACCEL_B200_ENOMEM) throw std::bad_alloc();
  throw std::runtime_error(msg);
}

class DeviceScope {
 public:
  explicit DeviceScope(int ordinal) {
    cudaGetDevice(&prev_);
    if (prev_ != ordinal) cudaSetDevice(ordinal);
    restore_ = prev_ != ordinal;
  }
  ~DeviceScope() {
    if (restore_) cudaSetDevice(prev_);
  }

 private:
  int prev_ = 0;
  bool restore_ = false;
};

// Zero-filled device memory (SimDevice zero-fills too, sim_device.cc:139).
struct DevBuf {
  void* p = nullptr;
  size_t bytes = 0;
  DevBuf() = default;
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  DevBuf(DevBuf&& o) noexcept : p(o.p), bytes(o.bytes) {
    o.p = nullptr;
    o.bytes = 0;
  }
  ~DevBuf() { Reset(); }
  void Reset() {
    if (p != nullptr) cudaFree(p);
    p = nullptr;
    bytes = 0;
  }
  void Alloc(size_t b) {
    Reset();
    Cuda(cudaMalloc(&p, b == 0 ? 1 : b), "device allocation");
    bytes = b;
    Cuda(cudaMemset(p, 0, b == 0 ? 1 : b), "zero fill");
    // The engine's stream does not wait for the legacy stream the fill ran on.
    Cuda(cudaDeviceSynchronize(), "zero fill");
  }
  // Grows to at least b bytes; returns true when the address changed.
  bool Ensure(size_t b) {
    if (p != nullptr && bytes >= b) return false;
    Alloc(b);
    return true;
  }
  template <typename T>
  T* as() const {
    return static_cast<T*>(p);
  }
};

struct PinnedBuf {
  void* p = nullptr;
  size_t bytes = 0;
  ~PinnedBuf() {
    if (p != nullptr) cudaFreeHost(p);
  }
  void Ensure(size_t b) {
    if (p != nullptr && bytes >= b) return;
    if (p != nullptr) cudaFreeHost(p);
    p = nullptr;
    Cuda(cudaMallocHost(&p, b == 0 ? 1 : b), "pinned allocation");
    bytes = b;
  }
  template <typename T>
  T* as() const {
    return static_cast<T*>(p);
  }
};

enum class WKind { Unset, F32, Q8 };

// A product weight [k, n] assembled from members that occupy column ranges.
struct Group {
  WKind kind = WKind::Unset;
  int64_t k = 0;
  int64_t n = 0;
  std::vector<int64_t> col0;
  std::vector<int64_t> width;
  DevBuf w;
  DevBuf scale;
  uint32_t loaded = 0;
  // int8 gate|up stored in 64-column pairs (gate block t, then up block t):
  // the product's epilogue then writes SiluMul(gate, up) directly.
  bool paired = false;

  void Define(int64_t k_in, std::vector<int64_t> widths) {
    k = k_in;
    width = std::move(widths);
    col0.clear();
    n = 0;
    for (int64_t w_ : width) {
      col0.push_back(n);
      n += w_;
    }
  }
  bool Full() const { return loaded == (1u << width.size()) - 1u; }
};

struct Layer {
  DevBuf attn_norm;
  DevBuf post_norm;
  Group qkv;   // members q, k, v
  Group o;     // member o
  Group gu;    // members gate, up
  Group down;  // member down
};

class Engine {
 public:
  explicit Engine(const AccelLlamaConfig& c) : cfg(c) {
    Cuda(cudaGetDevice(&device), "current device");
    head_dim = cfg.hidden / cfg.heads;
    q_out = cfg.heads * head_dim;
    kv_out = cfg.kv_heads * head_dim;
    Cuda(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "stream");
    layers.resize(static_cast<size_t>(cfg.layers));
    for (Layer& l : layers) {
      l.qkv.Define(cfg.hidden, {q_out, kv_out, kv_out});
      l.o.Define(q_out, {cfg.hidden});
      l.gu.Define(cfg.hidden, {cfg.intermediate, cfg.intermediate});
      l.down.Define(cfg.intermediate, {cfg.hidden});
    }
    lm_head.Define(cfg.hidden, {cfg.vocab});
    // RoPE tables exactly as src/llama_model.cc:333-349 builds them.
    const int64_t ctx = cfg.context, dim = head_dim, half = dim / 2;
    std::vector<float> cos_t(static_cast<size_t>(ctx * dim)), sin_t(static_cast<size_t>(ctx * dim));
    for (int64_t pos = 0; pos < ctx; ++pos) {
      for (int64_t i = 0; i < half; ++i) {
        const double inv = 1.0 / std::pow(static_cast<double>(cfg.rope_theta), (2.0 * i) / static_cast<double>(dim));
        const double angle = static_cast<double>(pos) * inv;
        const float cv = static_cast<float>(std::cos(angle));
        const float sv = static_cast<float>(std::sin(angle));
        cos_t[pos * dim + i] = cos_t[pos * dim + half + i] = cv;
        sin_t[pos * dim + i] = sin_t[pos * dim + half + i] = sv;
      }
    }
    UploadRaw(&rope_cos, cos_t.data(), cos_t.size() * sizeof(float));
    UploadRaw(&rope_sin, sin_t.data(), sin_t.size() * sizeof(float));
    EnsureSlots(1);
  }

  ~Engine() {
    DropGraphs();
    if (stream != nullptr) {
      cudaStreamSynchronize(stream);
      cudaStreamDestroy(stream);
    }
  }

  // ----------------------------------------------------------------- weights

  bool Ready() const {
    if (embed.p == nullptr || final_norm.p == nullptr || !lm_head.Full()) return false;
    for (const Layer& l : layers) {
      if (l.attn_norm.p == nullptr || l.post_norm.p == nullptr || !l.qkv.Full() || !l.o.Full() || !l.gu.Full() ||
          !l.down.Full()) {
        return false;
      }
    }
    return true;
  }

  // src/llama_model.cc:288-314 (ShapeOk).
  bool ShapeOk(int32_t kind, int64_t rows, int64_t cols) const {
    const int64_t hidden = cfg.hidden;
    switch (kind) {
      case ACCEL_W_EMBED:
      case ACCEL_W_LM_HEAD:
        return rows == cfg.vocab && cols == hidden;
      case ACCEL_W_FINAL_NORM:
      case ACCEL_W_ATTN_NORM:
      case ACCEL_W_POST_NORM:
        return rows == hidden && cols == 1;
      case ACCEL_W_Q:
        return rows == q_out && cols == hidden;
      case ACCEL_W_K:
      case ACCEL_W_V:
        return rows == kv_out && cols == hidden;
      case ACCEL_W_O:
        return rows == hidden && cols == q_out;
      case ACCEL_W_DOWN:
        return rows == hidden && cols == cfg.intermediate;
      case ACCEL_W_GATE:
      case ACCEL_W_UP:
        return rows == cfg.intermediate && cols == hidden;
      default:
        return false;
    }
  }

  void WeightF32(int32_t kind, int32_t layer, const float* data, int64_t rows, int64_t cols) {
    if (kind == ACCEL_W_EMBED || kind == ACCEL_W_FINAL_NORM || kind == ACCEL_W_ATTN_NORM || kind == ACCEL_W_POST_NORM) {
      DevBuf* slot = PlainSlot(kind, layer);
      UploadRaw(slot, data, static_cast<size_t>(rows * cols) * sizeof(float));
      return;
    }
    Group* g;
    int member;
    GroupSlot(kind, layer, &g, &member);
    if (g->kind == WKind::Q8) throw std::invalid_argument("fp32 and int8 weights cannot share a fused product");
    if (g->kind == WKind::Unset) {
      g->w.Alloc(static_cast<size_t>(g->k * g->n) * sizeof(float));
      g->kind = WKind::F32;
    }
    // Hugging Face [out, in] -> [in, out] columns of the fused matrix.
    std::vector<float> t(static_cast<size_t>(rows * cols));
    for (int64_t o = 0; o < rows; ++o)
      for (int64_t i = 0; i < cols; ++i) t[static_cast<size_t>(i * rows + o)] = data[o * cols + i];
    Cuda(cudaMemcpy2D(g->w.as<float>() + g->col0[member], g->n * sizeof(float), t.data(), rows * sizeof(float),
                      rows * sizeof(float), cols, cudaMemcpyHostToDevice),
         "weight upload");
    NoteBytesToDevice(t.size() * sizeof(float));
    g->loaded |= 1u << member;
    DropGraphs();
  }

  void WeightQ8(int32_t kind, int32_t layer, const int8_t* q, const float* scale, int64_t rows, int64_t cols) {
    Group* g;
    int member;
    GroupSlot(kind, layer, &g, &member);
    if (g->kind == WKind::F32) throw std::invalid_argument("fp32 and int8 weights cannot share a fused product");
    if (g->kind == WKind::Unset) {
      g->w.Alloc(static_cast<size_t>(g->k * g->n));
      g->scale.Alloc(static_cast<size_t>(g->n) * sizeof(float));
      g->kind = WKind::Q8;
      g->paired = (kind == ACCEL_W_GATE || kind == ACCEL_W_UP) && cfg.intermediate % 64 == 0 && cfg.hidden % 8 == 0;
    }
    std::vector<int8_t> t(static_cast<size_t>(rows * cols));
    for (int64_t o = 0; o < rows; ++o)
      for (int64_t i = 0; i < cols; ++i) t[static_cast<size_t>(i * rows + o)] = q[o * cols + i];
    if (g->paired) {
      // Block b of this member (gate: 0, up: 1) to columns 128 b + 64 member.
      for (int64_t b = 0; b < rows / 64; ++b) {
        Cuda(cudaMemcpy2D(g->w.as<int8_t>() + 128 * b + 64 * member, g->n, t.data() + 64 * b, rows, 64, cols,
                          cudaMemcpyHostToDevice),
             "weight upload");
        Cuda(cudaMemcpy(g->scale.as<float>() + 128 * b + 64 * member, scale + 64 * b, 64 * sizeof(float),
                        cudaMemcpyHostToDevice),
             "scale upload");
      }
    } else {
      Cuda(cudaMemcpy2D(g->w.as<int8_t>() + g->col0[member], g->n, t.data(), rows, rows, cols,
                        cudaMemcpyHostToDevice),
           "weight upload");
      Cuda(cudaMemcpy(g->scale.as<float>() + g->col0[member], scale, rows * sizeof(float), cudaMemcpyHostToDevice),
           "scale upload");
    }
    NoteBytesToDevice(t.size() + rows * sizeof(float));
    g->loaded |= 1u << member;
    DropGraphs();
  }

  // ------------------------------------------------------------- generation

  // src/llama_model.cc:150-166.
  void ForwardIds(const int32_t* ids, int32_t count, bool reset) {
    if (!Ready()) throw std::invalid_argument("llama weights are incomplete");
    if (ids == nullptr || count <= 0) throw std::invalid_argument("invalid forward");
    if (reset) filled = 0;
    if (filled < 0 || count > cfg.context - filled) throw std::invalid_argument("forward exceeds context");
    CheckIds(ids, count);
    EnsureRows(count, 1);
    PinnedBuf& st = staging;
    st.Ensure(static_cast<size_t>(count) * 12 + 32);
    int32_t* h = st.as<int32_t>();
    for (int32_t r = 0; r < count; ++r) {
      h[r] = ids[r];
      h[count + r] = 0;
      h[2 * count + r] = filled + r;
    }
    h[3 * count] = count - 1;
    h[3 * count + 1] = 0;       // first row of sequence 0
    h[3 * count + 2] = count;   // its rows
    h[3 * count + 3] = filled;  // its first position
    Cuda(cudaMemcpyAsync(seq_first.p, h + 3 * count + 1, 4, cudaMemcpyHostToDevice, stream), "rows");
    Cuda(cudaMemcpyAsync(seq_count.p, h + 3 * count + 2, 4, cudaMemcpyHostToDevice, stream), "rows");
    Cuda(cudaMemcpyAsync(seq_pos0.p, h + 3 * count + 3, 4, cudaMemcpyHostToDevice, stream), "rows");
    prefill_max_rows = count;
    Cuda(cudaMemcpyAsync(tokens.p, h, count * 4, cudaMemcpyHostToDevice, stream), "ids");
    NoteBytesToDevice(static_cast<size_t>(count) * 4);
    Cuda(cudaMemcpyAsync(row_seq.p, h + count, count * 4, cudaMemcpyHostToDevice, stream), "rows");
    Cuda(cudaMemcpyAsync(row_pos.p, h + 2 * count, count * 4, cudaMemcpyHostToDevice, stream), "rows");
    Cuda(cudaMemcpyAsync(last_rows.p, h + 3 * count, 4, cudaMemcpyHostToDevice, stream), "rows");
    Forward(count, 1, false);
    Cuda(cudaStreamSynchronize(stream), "forward");
    filled += count;
    logit_rows = 1;
  }

  // src/llama_model.cc:101-131, for `batch` sequences at once.
  void Generate(const int32_t* prompts, const int32_t* counts, int32_t batch, int32_t max_new, int32_t eos,
                float temperature, uint32_t seed, const uint32_t* seeds, int32_t top_k, int32_t* out_ids,
                int32_t* out_counts, bool single) {
    filled = 0;
    if (batch <= 0) throw std::invalid_argument("invalid generate");
    int64_t rows = 0;
    int32_t min_count = cfg.context;
    for (int32_t b = 0; b < batch; ++b) {
      if (counts[b] <= 0 || counts[b] > cfg.context) throw std::invalid_argument("forward exceeds context");
      rows += counts[b];
      min_count = std::min(min_count, counts[b]);
    }
    CheckIds(prompts, rows);
    // A sequence produces at most context - prompt + 1 ids (the loop stops
    // once the cache is full), so this bounds every sequence's count.
    const int32_t steps = std::max(0, std::min<int32_t>(max_new, cfg.context - min_count + 1));
    EnsureSlots(batch);
    EnsureRows(std::max<int64_t>(rows, batch), batch);
    EnsureIds(batch, std::max(steps, 1));
    const bool sampled = temperature > 0.f;

    PinnedBuf& st = staging;
    st.Ensure(static_cast<size_t>(rows) * 12 + static_cast<size_t>(batch) * 28 + 64);
    int32_t* h = st.as<int32_t>();
    int32_t* h_tok = h;
    int32_t* h_seq = h + rows;
    int32_t* h_pos = h + 2 * rows;
    int32_t* h_last = h + 3 * rows;
    int32_t* h_lens = h_last + batch;
    uint32_t* h_rng = reinterpret_cast<uint32_t*>(h_lens + batch);
    int32_t* h_ident = reinterpret_cast<int32_t*>(h_rng + batch);
    int32_t* h_first = h_ident + batch;
    int32_t* h_count = h_first + batch;
    int32_t* h_pos0 = h_count + batch;
    int64_t r = 0;
    prefill_max_rows = 0;
    for (int32_t b = 0; b < batch; ++b) {
      h_first[b] = static_cast<int32_t>(r);
      h_count[b] = counts[b];
      h_pos0[b] = 0;
      prefill_max_rows = std::max(prefill_max_rows, counts[b]);
      for (int32_t s = 0; s < counts[b]; ++s, ++r) {
        h_tok[r] = prompts[r];
        h_seq[r] = b;
        h_pos[r] = s;
      }
      h_last[b] = static_cast<int32_t>(r - 1);
      h_lens[b] = counts[b];
      const uint32_t sd = seeds != nullptr ? seeds[b] : seed;
      h_rng[b] = sd == 0 ? 0x6d2b79f5u : sd;  // src/llama_model.cc:111
      h_ident[b] = b;
    }
    Cuda(cudaMemcpyAsync(tokens.p, h_tok, rows * 4, cudaMemcpyHostToDevice, stream), "prompt ids");
    NoteBytesToDevice(static_cast<size_t>(rows) * 4);
    Cuda(cudaMemcpyAsync(row_seq.p, h_seq, rows * 4, cudaMemcpyHostToDevice, stream), "rows");
    Cuda(cudaMemcpyAsync(row_pos.p, h_pos, rows * 4, cudaMemcpyHostToDevice, stream), "rows");
    Cuda(cudaMemcpyAsync(last_rows.p, h_last, batch * 4, cudaMemcpyHostToDevice, stream), "rows");
    Cuda(cudaMemcpyAsync(lens.p, h_lens, batch * 4, cudaMemcpyHostToDevice, stream), "lens");
    Cuda(cudaMemcpyAsync(rng.p, h_rng, batch * 4, cudaMemcpyHostToDevice, stream), "rng");
    Cuda(cudaMemcpyAsync(dec_seq.p, h_ident, batch * 4, cudaMemcpyHostToDevice, stream), "rows");
    Cuda(cudaMemcpyAsync(seq_first.p, h_first, batch * 4, cudaMemcpyHostToDevice, stream), "rows");
    Cuda(cudaMemcpyAsync(seq_count.p, h_count, batch * 4, cudaMemcpyHostToDevice, stream), "rows");
    Cuda(cudaMemcpyAsync(seq_pos0.p, h_pos0, batch * 4, cudaMemcpyHostToDevice, stream), "rows");
    Cuda(cudaMemsetAsync(done.p, 0, batch * 4, stream), "state");
    Cuda(cudaMemsetAsync(count.p, 0, batch * 4, stream), "state");
    Cuda(cudaMemsetAsync(step.p, 0, 16, stream), "state");
    Forward(rows, batch, false);
    logit_rows = batch;

    cudaGraphExec_t exec = steps > 0 ? StepGraph(batch, sampled, temperature, top_k, eos) : nullptr;
    PinnedBuf& fin = finished_host;
    fin.Ensure(static_cast<size_t>(batch) * 4 + 16);
    for (int32_t n = 0; n < steps; ++n) {
      Cuda(cudaGraphLaunch(exec, stream), "decode step");
      NoteLaunches(graph_nodes);
      NoteKernelMatmuls(static_cast<int64_t>(7) * cfg.layers + 1);
      if ((n + 1) % 32 == 0 && n + 1 < steps) {
        Cuda(cudaMemcpyAsync(fin.p, finished.p, 4, cudaMemcpyDeviceToHost, stream), "progress");
        Cuda(cudaStreamSynchronize(stream), "decode");
        if (*fin.as<int32_t>() >= batch) break;
      }
    }
    // Counts, then the ids (src/llama_model.cc:129-130).
    std::vector<int32_t> cnt(static_cast<size_t>(batch));
    fin.Ensure(static_cast<size_t>(batch) * 4 + 16);
    Cuda(cudaMemcpyAsync(fin.p, count.p, batch * 4, cudaMemcpyDeviceToHost, stream), "counts");
    Cuda(cudaMemcpyAsync(fin.as<int32_t>() + batch, status.p, 4, cudaMemcpyDeviceToHost, stream), "status");
    Cuda(cudaStreamSynchronize(stream), "counts");
    std::memcpy(cnt.data(), fin.p, cnt.size() * 4);
    if (fin.as<int32_t>()[batch] != 0) {
      Cuda(cudaMemsetAsync(status.p, 0, 4, stream), "status");
      throw std::runtime_error("a decode attention copy did not complete within its wait bound");
    }
    if (single) {
      Cuda(cudaMemcpy(out_ids, ids.p, static_cast<size_t>(cnt[0]) * 4, cudaMemcpyDeviceToHost), "ids");
      NoteBytesToHost(static_cast<size_t>(cnt[0]) * 4);
      int32_t len0 = 0;
      Cuda(cudaMemcpy(&len0, lens.p, 4, cudaMemcpyDeviceToHost), "lens");
      filled = len0;
    } else {
      const int64_t width = std::max(1, max_new);
      if (steps > 0) {
        Cuda(cudaMemcpy2D(out_ids, width * 4, ids.p, ids_stride * 4, static_cast<size_t>(steps) * 4, batch,
                          cudaMemcpyDeviceToHost),
             "ids");
      }
      NoteBytesToHost(static_cast<size_t>(batch) * std::max(steps, 0) * 4);
      filled = 0;
    }
    for (int32_t b = 0; b < batch; ++b) out_counts[b] = cnt[static_cast<size_t>(b)];
  }

  float LogitMaxAbs(const float* reference, int32_t n) {
    if (reference == nullptr || n != cfg.vocab) throw std::invalid_argument("invalid logit reference");
    DevBuf ref;
    ref.Alloc(static_cast<size_t>(n) * 4 + 4);
    Cuda(cudaMemcpyAsync(ref.p, reference, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice, stream), "reference row");
    float* out = ref.as<float>() + n;
    Abi(accel_b200_max_abs_diff(logits.as<float>(), ref.as<float>(), n, out, stream));
    float host = 0.f;
    Cuda(cudaMemcpyAsync(&host, out, 4, cudaMemcpyDeviceToHost, stream), "max abs");
    Cuda(cudaStreamSynchronize(stream), "max abs");
    return host;
  }

  // One row per sequence of the last forward (n = rows * vocab); after a
  // batched generate, row b is sequence b's last forward.
  void Logits(float* out, int32_t n) {
    if (out == nullptr || n <= 0 || n % cfg.vocab != 0 || n / cfg.vocab > logit_rows) {
      throw std::invalid_argument("invalid logit buffer");
    }
    Cuda(cudaMemcpyAsync(out, logits.p, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToHost, stream), "logits");
    Cuda(cudaStreamSynchronize(stream), "logits");
  }

  void CacheRows(int32_t slot, int32_t layer, int32_t which, int32_t nrows, float* out) {
    if (slot < 0 || slot >= slots || layer < 0 || layer >= cfg.layers || (which != 0 && which != 1) || nrows < 0 ||
        nrows > cfg.context || out == nullptr) {
      throw std::invalid_argument("invalid cache read");
    }
    // Head-major in HBM; the reference layout [rows, kv_heads, head_dim] on the host.
    const DevBuf& c = which == 0 ? k_cache[static_cast<size_t>(layer)] : v_cache[static_cast<size_t>(layer)];
    const int64_t head_stride = static_cast<int64_t>(cfg.context) * head_dim;
    const float* src = c.as<float>() + static_cast<int64_t>(slot) * head_stride * cfg.kv_heads;
    for (int32_t g = 0; g < cfg.kv_heads && nrows > 0; ++g) {
      Cuda(cudaMemcpy2DAsync(out + g * head_dim, kv_out * 4, src + g * head_stride, head_dim * 4, head_dim * 4, nrows,
                             cudaMemcpyDeviceToHost, stream),
           "cache");
    }
    Cuda(cudaStreamSynchronize(stream), "cache");
  }

  AccelLlamaConfig cfg;
  int device = 0;
  int32_t head_dim = 0, q_out = 0, kv_out = 0;
  int32_t filled = 0;
  int32_t logit_rows = 0;  // logit rows the last forward wrote
  cudaStream_t stream = nullptr;
  std::mutex mu;

 private:
  DevBuf* PlainSlot(int32_t kind, int32_t layer) {
    if (kind == ACCEL_W_EMBED) return &embed;
    if (kind == ACCEL_W_FINAL_NORM) return &final_norm;
    if (layer < 0 || layer >= cfg.layers) throw std::invalid_argument("unknown weight");
    return kind == ACCEL_W_ATTN_NORM ? &layers[static_cast<size_t>(layer)].attn_norm
                                     : &layers[static_cast<size_t>(layer)].post_norm;
  }

  void GroupSlot(int32_t kind, int32_t layer, Group** g, int* member) {
    if (kind == ACCEL_W_LM_HEAD) {
      *g = &lm_head;
      *member = 0;
      return;
    }
    if (layer < 0 || layer >= cfg.layers) throw std::invalid_argument("unknown weight");
    Layer& l = layers[static_cast<size_t>(layer)];
    switch (kind) {
      case ACCEL_W_Q: *g = &l.qkv; *member = 0; return;
      case ACCEL_W_K: *g = &l.qkv; *member = 1; return;
      case ACCEL_W_V: *g = &l.qkv; *member = 2; return;
      case ACCEL_W_O: *g = &l.o; *member = 0; return;
      case ACCEL_W_GATE: *g = &l.gu; *member = 0; return;
      case ACCEL_W_UP: *g = &l.gu; *member = 1; return;
      case ACCEL_W_DOWN: *g = &l.down; *member = 0; return;
      default: throw std::invalid_argument("unknown weight");
    }
  }

  void UploadRaw(DevBuf* slot, const void* data, size_t bytes) {
    slot->Alloc(bytes);
    if (bytes > 0) {
      Cuda(cudaMemcpy(slot->p, data, bytes, cudaMemcpyHostToDevice), "upload");
      NoteBytesToDevice(bytes);
    }
    DropGraphs();
  }

  // src/sim_embed.cc:13-15 rejects ids outside the vocabulary.
  void CheckIds(const int32_t* ids, int64_t n) const {
    for (int64_t i = 0; i < n; ++i) {
      if (ids[i] < 0 || ids[i] >= cfg.vocab) throw std::invalid_argument("token id is outside the vocabulary");
    }
  }

  void EnsureSlots(int32_t n) {
    if (n <= slots) return;
    cudaStreamSynchronize(stream);
    const size_t per = static_cast<size_t>(n) * cfg.context * kv_out * sizeof(float);
    k_cache.clear();
    v_cache.clear();
    k_cache.resize(static_cast<size_t>(cfg.layers));
    v_cache.resize(static_cast<size_t>(cfg.layers));
    for (int32_t l = 0; l < cfg.layers; ++l) {
      k_cache[static_cast<size_t>(l)].Alloc(per);
      v_cache[static_cast<size_t>(l)].Alloc(per);
    }
    slots = n;
    DropGraphs();
  }

  void EnsureRows(int64_t rows, int32_t seqs) {
    bool moved = false;
    const int64_t H = cfg.hidden, I = cfg.intermediate;
    const size_t R = static_cast<size_t>(rows);
    moved |= hidden.Ensure(R * H * 4);
    moved |= normed.Ensure(R * H * 4);
    moved |= qkv.Ensure(R * (q_out + 2 * kv_out) * 4);
    moved |= mixed.Ensure(R * q_out * 4);
    moved |= gu.Ensure(R * 2 * I * 4);
    moved |= act.Ensure(R * I * 4);
    moved |= tokens.Ensure(R * 4);
    moved |= row_seq.Ensure(R * 4);
    moved |= row_pos.Ensure(R * 4);
    const size_t S = static_cast<size_t>(seqs);
    moved |= gathered.Ensure(S * H * 4);
    moved |= normed_last.Ensure(S * H * 4);
    moved |= logits.Ensure(S * cfg.vocab * 4);
    moved |= last_rows.Ensure(S * 4);
    moved |= seq_first.Ensure(S * 4);
    moved |= row_sq.Ensure(static_cast<size_t>(S) * SqBlocks() * sizeof(double));
    moved |= seq_count.Ensure(S * 4);
    moved |= seq_pos0.Ensure(S * 4);
    moved |= lens.Ensure(S * 4);
    moved |= dec_seq.Ensure(S * 4);
    moved |= dec_pos.Ensure(S * 4);
    moved |= done.Ensure(S * 4);
    moved |= count.Ensure(S * 4);
    moved |= pre_ids.Ensure(S * 4);
    moved |= rng.Ensure(S * 4);
    moved |= step.Ensure(16);
    moved |= finished.Ensure(16);
    size_t ws = 0;
    for (int64_t m : {rows, static_cast<int64_t>(seqs)}) {
      for (const Layer& l : layers) {
        for (const Group* g : {&l.qkv, &l.o, &l.gu, &l.down}) ws = std::max(ws, GemmWorkspace(*g, m));
        if (l.down.kind == WKind::Q8) ws = std::max(ws, accel_b200_matmul_q8_silu_workspace(m, l.down.k, l.down.n));
        for (const Group* g : {&l.qkv, &l.gu}) {
          if (g->kind == WKind::Q8) ws = std::max(ws, accel_b200_matmul_q8_rmsnorm_workspace(m, g->k, g->n));
        }
      }
      ws = std::max(ws, GemmWorkspace(lm_head, std::min<int64_t>(m, seqs)));
      if (lm_head.kind == WKind::Q8) {
        ws = std::max(ws, accel_b200_matmul_q8_rmsnorm_workspace(std::min<int64_t>(m, seqs), lm_head.k, lm_head.n));
      }
    }
    moved |= gemm_ws.Ensure(ws);
    moved |= status.Ensure(16);
    if (moved) DropGraphs();
  }

  void EnsureIds(int32_t seqs, int32_t width) {
    if (ids.p != nullptr && ids_rows >= seqs && ids_stride >= width) return;
    ids_rows = std::max(ids_rows, seqs);
    ids_stride = std::max(ids_stride, static_cast<int64_t>(width));
    ids.Alloc(static_cast<size_t>(ids_rows) * ids_stride * 4);
    DropGraphs();
  }

  static size_t GemmWorkspace(const Group& g, int64_t m) {
    if (g.kind == WKind::Q8) return accel_b200_matmul_q8_workspace(m, g.k, g.n);
    return accel_b200_matmul_f32_workspace(m, g.k, g.n);
  }

  void Gemm(const float* a, int64_t lda, const Group& g, int64_t m, float* c, int64_t ldc,
            const accel_b200_epilogue* ep) {
    if (g.kind == WKind::Q8) {
      accel_b200_q8_plane plane{g.w.as<int8_t>(), g.scale.as<float>(), nullptr, 0, 1};
      Abi(accel_b200_matmul_q8(a, lda, &plane, c, ldc, m, g.k, g.n, ep, gemm_ws.p, gemm_ws.bytes, stream));
    } else {
      Abi(accel_b200_matmul_f32(a, lda, g.w.as<float>(), c, ldc, m, g.k, g.n, ep, gemm_ws.p, gemm_ws.bytes, stream));
    }
  }

  // RmsNorm(x) then the product (src/llama_model.cc:228-229, :237-238, :245-246):
  // one kernel for int8 weights; through `normed` for fp32 weights.
  // With `sq` (decode, int8 weights) the rows' sums of squares come from the
  // product that wrote x, so the norm reads 5 values per row, not the row.
  void NormGemm(const float* x, const DevBuf& gamma, const Group& g, int64_t m, float* c, int64_t ldc,
                const accel_b200_epilogue* ep, DevBuf& normed_buf, const double* sq = nullptr) {
    const int64_t H = cfg.hidden;
    if (g.kind == WKind::Q8 && sq != nullptr) {
      accel_b200_q8_plane plane{g.w.as<int8_t>(), g.scale.as<float>(), nullptr, 0, 1};
      Abi(accel_b200_matmul_q8_rmsnorm_stats(x, H, sq, SqBlocks(), static_cast<int32_t>(SqBlocks()),
                                             gamma.as<float>(), cfg.eps, &plane, c, ldc, m, g.k, g.n, ep, gemm_ws.p,
                                             gemm_ws.bytes, stream));
    } else if (g.kind == WKind::Q8) {
      accel_b200_q8_plane plane{g.w.as<int8_t>(), g.scale.as<float>(), nullptr, 0, 1};
      Abi(accel_b200_matmul_q8_rmsnorm(x, H, gamma.as<float>(), cfg.eps, &plane, c, ldc, m, g.k, g.n, ep, gemm_ws.p,
                                       gemm_ws.bytes, stream));
    } else {
      Abi(accel_b200_rmsnorm(x, gamma.as<float>(), normed_buf.as<float>(), m, H, cfg.eps, 0, stream));
      Gemm(normed_buf.as<float>(), H, g, m, c, ldc, ep);
    }
  }

  // 128-column blocks of a hidden row (one sum of squares each).
  int64_t SqBlocks() const { return (cfg.hidden + 127) / 128; }

  // Whether every product that writes or normalizes the hidden rows runs on
  // int8 weights (the GEMV and tensor-core kernels write row sums of squares).
  bool AllQ8() const {
    for (const Layer& l : layers) {
      if (l.qkv.kind != WKind::Q8 || l.o.kind != WKind::Q8 || l.gu.kind != WKind::Q8 || l.down.kind != WKind::Q8) {
        return false;
      }
    }
    return true;
  }

  // src/llama_model.cc:209-247 over `rows` rows of `seqs` sequences. The
  // last row of each sequence gives its logit row. decode: rows == seqs,
  // row b is sequence b's new token at dec_pos[b].
  void Forward(int64_t rows, int32_t seqs, bool decode) {
    const int64_t H = cfg.hidden, I = cfg.intermediate;
    const int64_t qkv_ld = q_out + 2 * kv_out;
    // Head-major cache: slot -> kv head -> row -> dim, so one (sequence, kv
    // head) chunk of rows is one contiguous block for the decode kernel.
    const int64_t row_stride = head_dim;
    const int64_t head_stride = static_cast<int64_t>(cfg.context) * head_dim;
    const int64_t slot_stride = head_stride * cfg.kv_heads;
    const int32_t* tok = decode ? pre_tokens() : tokens.as<int32_t>();
    const int32_t* rseq = decode ? dec_seq.as<int32_t>() : row_seq.as<int32_t>();
    const int32_t* rpos = decode ? dec_pos.as<int32_t>() : row_pos.as<int32_t>();
    float* hid = hidden.as<float>();
    accel_b200_epilogue residual{};
    residual.alpha = 1.f;
    residual.residual = hid;
    residual.residual_ld = H;
    // Decode on int8 weights: the o and down products also write each hidden
    // row's sums of squares, which the next RmsNorm-fed product reads.
    const double* sq = nullptr;
    if (decode && AllQ8()) {
      residual.row_sq = row_sq.as<double>();
      residual.row_sq_ld = SqBlocks();
      sq = row_sq.as<double>();
    }
    Abi(accel_b200_embed(tok, 0, embed.as<float>(), hid, rows, H, cfg.vocab, nullptr, stream));
    for (int32_t li = 0; li < cfg.layers; ++li) {
      Layer& l = layers[static_cast<size_t>(li)];
      float* kc = k_cache[static_cast<size_t>(li)].as<float>();
      float* vc = v_cache[static_cast<size_t>(li)].as<float>();
      // Decode: the q|k|v product lets the attention launch only after its
      // own wait, so the attention reads the cache (written by earlier
      // kernels, all completed by then) and starts its first copies before
      // it waits for the q|k|v rows.
      const bool fused = decode && head_dim == 64;
      accel_b200_epilogue qkv_ep{};
      qkv_ep.alpha = 1.f;
      qkv_ep.flags = ACCEL_B200_EP_TRIGGER_AFTER_WAIT;
      const bool early = fused && l.qkv.kind == WKind::Q8;
      NormGemm(hid, l.attn_norm, l.qkv, rows, qkv.as<float>(), qkv_ld, early ? &qkv_ep : nullptr, normed,
               li > 0 ? sq : nullptr);
      if (fused) {
        // Rope, AppendCache and attention of the new rows in one kernel.
        // While it runs, the int8 weights of the products that follow (this
        // layer's o, gate|up and down, then the next layer's q|k|v or, after
        // the last layer, the LM head) go to L2.
        accel_b200_l2_prefetch pf{};
        const Group* next[4] = {&l.o, &l.gu, &l.down,
                                li + 1 < cfg.layers ? &layers[static_cast<size_t>(li) + 1].qkv : &lm_head};
        for (const Group* g : next) {
          if (g == nullptr || g->kind != WKind::Q8) continue;
          pf.ptr[pf.count] = g->w.p;
          pf.bytes[pf.count] = g->k * g->n;
          ++pf.count;
        }
        if (early) pf.flags = ACCEL_B200_ATTN_CACHE_BEFORE_WAIT;
        Abi(accel_b200_decode_attention_prefetch(qkv.as<float>(), qkv_ld, rseq, rpos, rows, cfg.heads, cfg.kv_heads,
                                                 head_dim, rope_cos.as<float>(), rope_sin.as<float>(), cfg.context,
                                                 kc, vc, slot_stride, head_stride, mixed.as<float>(), q_out,
                                                 status.as<int32_t>(), &pf, stream));
      } else {
        Abi(accel_b200_rope_append(qkv.as<float>(), qkv_ld, rseq, rpos, rows, cfg.heads, cfg.kv_heads, head_dim,
                                   rope_cos.as<float>(), rope_sin.as<float>(), kc, vc, slot_stride, head_stride,
                                   row_stride, stream));
        if (!decode && head_dim == 64 && cfg.heads / cfg.kv_heads <= 4) {
          Abi(accel_b200_attention_prefill(qkv.as<float>(), qkv_ld, kc, vc, slot_stride, head_stride,
                                           mixed.as<float>(), q_out, seq_first.as<int32_t>(), seq_count.as<int32_t>(),
                                           seq_pos0.as<int32_t>(), seqs, prefill_max_rows, cfg.heads, cfg.kv_heads,
                                           head_dim, stream));
        } else {
          Abi(accel_b200_attention_rows(qkv.as<float>(), qkv_ld, kc, vc, row_stride, head_stride, slot_stride,
                                        mixed.as<float>(), q_out, rseq, decode ? dec_len_pos() : rpos, rows,
                                        cfg.heads, cfg.kv_heads, head_dim, stream));
        }
      }
      Gemm(mixed.as<float>(), q_out, l.o, rows, hid, H, &residual);
      if (l.gu.kind == WKind::Q8 && l.gu.paired) {
        // RmsNorm -> gate|up -> SiluMul in one product, then the down product.
        accel_b200_q8_plane plane{l.gu.w.as<int8_t>(), l.gu.scale.as<float>(), nullptr, 0, 1};
        Abi(accel_b200_matmul_q8_rmsnorm_silu_pairs(hid, H, sq, SqBlocks(), static_cast<int32_t>(SqBlocks()),
                                                    l.post_norm.as<float>(), cfg.eps, &plane, act.as<float>(), I,
                                                    rows, H, 2 * I, gemm_ws.p, gemm_ws.bytes, stream));
        Gemm(act.as<float>(), I, l.down, rows, hid, H, &residual);
        continue;
      }
      NormGemm(hid, l.post_norm, l.gu, rows, gu.as<float>(), 2 * I, nullptr, normed, sq);
      if (l.down.kind == WKind::Q8) {
        // SiluMul feeds the down projection's operand directly.
        accel_b200_q8_plane plane{l.down.w.as<int8_t>(), l.down.scale.as<float>(), nullptr, 0, 1};
        Abi(accel_b200_matmul_q8_silu(gu.as<float>(), 2 * I, I, &plane, hid, H, rows, H, &residual, gemm_ws.p,
                                      gemm_ws.bytes, stream));
      } else {
        Abi(accel_b200_silu_mul_rows(gu.as<float>(), 2 * I, act.as<float>(), I, rows, I, stream));
        Gemm(act.as<float>(), I, l.down, rows, hid, H, &residual);
      }
    }
    const float* last = hid;
    if (!decode) {
      Abi(accel_b200_gather_rows(hid, H, last_rows.as<int32_t>(), seqs, H, gathered.as<float>(), H, stream));
      last = gathered.as<float>();
    }
    NormGemm(last, final_norm, lm_head, seqs, logits.as<float>(), cfg.vocab, nullptr, normed_last);
    // A captured decode forward is counted once per replay instead.
    if (!decode) NoteKernelMatmuls(static_cast<int64_t>(7) * cfg.layers + 1);
  }

  // Decode reads the tokens the step kernel chose.
  const int32_t* pre_tokens() const { return tokens.as<int32_t>(); }
  // The generic attention path of a decode row attends through its own
  // position (dec_pos); finished rows carry -1 and are skipped upstream.
  const int32_t* dec_len_pos() const { return dec_pos.as<int32_t>(); }

  cudaGraphExec_t StepGraph(int32_t batch, bool sampled, float temperature, int32_t top_k, int32_t eos) {
    const auto key = std::make_tuple(batch, sampled, sampled ? temperature : 0.f, sampled ? top_k : 0, eos);
    if (graph_exec != nullptr && key == graph_key) return graph_exec;
    DropGraphs();
    Cuda(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal), "capture");
    try {
      if (sampled) {
        Abi(accel_b200_sample_rows(logits.as<float>(), batch, cfg.vocab, cfg.vocab, pre_ids.as<int32_t>(), 1, 0,
                                   temperature, rng.as<uint32_t>(), top_k, stream));
      }
      Abi(accel_b200_greedy_step(logits.as<float>(), sampled ? pre_ids.as<int32_t>() : nullptr, cfg.vocab, cfg.vocab,
                                 ids.as<int32_t>(), ids_stride, count.as<int32_t>(), done.as<int32_t>(),
                                 tokens.as<int32_t>(), dec_pos.as<int32_t>(), lens.as<int32_t>(), eos, cfg.context,
                                 step.as<int32_t>(), finished.as<int32_t>(), batch, stream));
      Forward(batch, batch, true);
    } catch (...) {
      cudaGraph_t g = nullptr;
      cudaStreamEndCapture(stream, &g);
      if (g != nullptr) cudaGraphDestroy(g);
      throw;
    }
    cudaGraph_t g = nullptr;
    Cuda(cudaStreamEndCapture(stream, &g), "capture");
    size_t nodes = 0;
    cudaGraphGetNodes(g, nullptr, &nodes);
    const cudaError_t err = cudaGraphInstantiate(&graph_exec, g, 0);
    cudaGraphDestroy(g);
    Cuda(err, "graph instantiate");
    graph_key = key;
    graph_nodes = static_cast<int64_t>(nodes);
    return graph_exec;
  }

  void DropGraphs() {
    if (graph_exec != nullptr) {
      cudaGraphExecDestroy(graph_exec);
      graph_exec = nullptr;
    }
  }

  DevBuf embed, final_norm, rope_cos, rope_sin;
  std::vector<Layer> layers;
  Group lm_head;
  std::vector<DevBuf> k_cache, v_cache;
  int32_t slots = 0;
  DevBuf hidden, normed, qkv, mixed, gu, act, gathered, normed_last, logits;
  DevBuf tokens, row_seq, row_pos, last_rows, lens, dec_seq, dec_pos, done, count, pre_ids, rng, step, finished;
  // Prefill rows by sequence: first row, row count and first position.
  DevBuf seq_first, seq_count, seq_pos0;
  DevBuf row_sq;  // decode: per hidden row, sums of squares of its 128-column blocks
  int32_t prefill_max_rows = 0;
  DevBuf ids;
  int32_t ids_rows = 0;
  int64_t ids_stride = 0;
  DevBuf gemm_ws, status;
  PinnedBuf staging, finished_host;
  cudaGraphExec_t graph_exec = nullptr;
  std::tuple<int32_t, bool, float, int32_t, int32_t> graph_key;
  int64_t graph_nodes = 0;
};

Engine* Cast(AccelLlama* h) { return reinterpret_cast<Engine*>(h); }

template <typename F>
int Guarded(Engine* e, F&& body) {
  try {
    std::lock_guard<std::mutex> lock(e->mu);
    DeviceScope scope(e->device);
    body();
    Clear();
    return 0;
  } catch (const std::exception& ex) {
    Fail(ex.what());
    return 1;
  }
}

}  // namespace
}  // namespace accel_b200

using namespace accel_b200;

extern "C" {

ACCEL_B200_API AccelLlama* accel_llama_create(const AccelLlamaConfig* config) {
  // src/llama_model.cc:318-324.
  if (config == nullptr || config->vocab <= 0 || config->hidden <= 0 || config->layers <= 0 || config->heads <= 0 ||
      config->kv_heads <= 0 || config->intermediate <= 0 || config->context <= 0 || config->hidden % config->heads != 0 ||
      config->heads % config->kv_heads != 0) {
    Fail("invalid llama config");
    return nullptr;
  }
  try {
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
      cudaGetLastError();
      throw std::runtime_error("no CUDA device is available for the B200 backend");
    }
    auto e = std::unique_ptr<Engine>(new Engine(*config));
    Clear();
    return reinterpret_cast<AccelLlama*>(e.release());
  } catch (const std::exception& ex) {
    Fail(ex.what());
    return nullptr;
  }
}

ACCEL_B200_API void accel_llama_destroy(AccelLlama* model) {
  Engine* e = Cast(model);
  if (e == nullptr) return;
  DeviceScope scope(e->device);
  delete e;
}

ACCEL_B200_API int accel_llama_weight(AccelLlama* handle, int32_t kind, int32_t layer, const float* data, int64_t rows,
                                      int64_t cols) {
  Engine* e = Cast(handle);
  if (e == nullptr || data == nullptr || rows <= 0 || cols <= 0 || !e->ShapeOk(kind, rows, cols)) {
    Fail("invalid weight");
    return 1;
  }
  return Guarded(e, [&] { e->WeightF32(kind, layer, data, rows, cols); });
}

ACCEL_B200_API int accel_llama_weight_q8(AccelLlama* handle, int32_t kind, int32_t layer, const int8_t* q,
                                         const float* scale, int64_t rows, int64_t cols) {
  Engine* e = Cast(handle);
  const bool linear = kind == ACCEL_W_LM_HEAD || (kind >= ACCEL_W_Q && kind <= ACCEL_W_DOWN);
  if (e == nullptr || q == nullptr || scale == nullptr || rows <= 0 || cols <= 0 || !linear ||
      !e->ShapeOk(kind, rows, cols)) {
    Fail("invalid weight");
    return 1;
  }
  return Guarded(e, [&] { e->WeightQ8(kind, layer, q, scale, rows, cols); });
}

ACCEL_B200_API int accel_llama_tokenizer(AccelLlama* handle, const char* path) {
  (void)handle;
  (void)path;
  Fail("the B200 backend does not load tokenizers; pass token ids");
  return 1;
}

ACCEL_B200_API int accel_llama_generate(AccelLlama* handle, const int32_t* prompt, int32_t prompt_count,
                                        int32_t max_new, int32_t eos_id, float temperature, uint32_t seed,
                                        int32_t top_k, int32_t* out_ids, int32_t* out_count) {
  Engine* e = Cast(handle);
  if (e == nullptr || prompt == nullptr || out_ids == nullptr || out_count == nullptr || prompt_count <= 0 ||
      max_new < 0) {
    Fail("invalid generate");
    return 1;
  }
  return Guarded(e, [&] {
    if (!e->Ready()) throw std::invalid_argument("llama weights are incomplete");
    e->Generate(prompt, &prompt_count, 1, max_new, eos_id, temperature, seed, nullptr, top_k, out_ids, out_count, true);
  });
}

ACCEL_B200_API int accel_llama_generate_batch(AccelLlama* handle, const int32_t* prompts, const int32_t* prompt_counts,
                                              int32_t batch, int32_t max_new, int32_t eos_id, float temperature,
                                              uint32_t seed, const uint32_t* seeds, int32_t top_k, int32_t* out_ids,
                                              int32_t* out_counts) {
  Engine* e = Cast(handle);
  if (e == nullptr || prompts == nullptr || prompt_counts == nullptr || out_ids == nullptr || out_counts == nullptr ||
      batch <= 0 || max_new < 0) {
    Fail("invalid generate");
    return 1;
  }
  return Guarded(e, [&] {
    if (!e->Ready()) throw std::invalid_argument("llama weights are incomplete");
    e->Generate(prompts, prompt_counts, batch, max_new, eos_id, temperature, seed, seeds, top_k, out_ids, out_counts,
                false);
  });
}

ACCEL_B200_API int accel_llama_encode(AccelLlama* model, const char* text, int32_t text_len, int32_t* out_ids,
                                      int32_t out_cap, int32_t* out_count) {
  (void)model, (void)text, (void)text_len, (void)out_ids, (void)out_cap, (void)out_count;
  Fail("the B200 backend does not load tokenizers; pass token ids");
  return 1;
}

ACCEL_B200_API int accel_llama_decode(AccelLlama* model, const int32_t* ids, int32_t count, int32_t skip_special,
                                      char* out_text, int32_t out_cap, int32_t* out_len) {
  (void)model, (void)ids, (void)count, (void)skip_special, (void)out_text, (void)out_cap, (void)out_len;
  Fail("the B200 backend does not load tokenizers; pass token ids");
  return 1;
}

ACCEL_B200_API int accel_llama_complete_stream(AccelLlama* model, const char* prompt, int32_t prompt_len,
                                               int32_t max_new, int32_t eos_id, float temperature, uint32_t seed,
                                               int32_t top_k, char* out_text, int32_t out_text_cap,
                                               int32_t* out_text_len, int32_t* out_ids, int32_t out_ids_cap,
                                               int32_t* out_count, int32_t* prompt_tokens, AccelLlamaTokenFn on_token,
                                               void* user) {
  (void)model, (void)prompt, (void)prompt_len, (void)max_new, (void)eos_id, (void)temperature, (void)seed;
  (void)top_k, (void)out_text, (void)out_text_cap, (void)out_text_len, (void)out_ids, (void)out_ids_cap;
  (void)out_count, (void)prompt_tokens, (void)on_token, (void)user;
  Fail("the B200 backend does not load tokenizers; pass token ids");
  return 1;
}

ACCEL_B200_API int accel_llama_complete(AccelLlama* model, const char* prompt, int32_t prompt_len, int32_t max_new,
                                        int32_t eos_id, float temperature, uint32_t seed, int32_t top_k,
                                        char* out_text, int32_t out_text_cap, int32_t* out_text_len, int32_t* out_ids,
                                        int32_t out_ids_cap, int32_t* out_count, int32_t* prompt_tokens) {
  return accel_llama_complete_stream(model, prompt, prompt_len, max_new, eos_id, temperature, seed, top_k, out_text,
                                     out_text_cap, out_text_len, out_ids, out_ids_cap, out_count, prompt_tokens,
                                     nullptr, nullptr);
}

ACCEL_B200_API int accel_llama_forward_ids(AccelLlama* handle, const int32_t* ids, int32_t count, int32_t reset) {
  Engine* e = Cast(handle);
  if (e == nullptr) {
    Fail("invalid forward");
    return 1;
  }
  return Guarded(e, [&] { e->ForwardIds(ids, count, reset != 0); });
}

ACCEL_B200_API int accel_llama_logit_max_abs(AccelLlama* handle, const float* reference, int32_t count,
                                             float* out_max_abs) {
  Engine* e = Cast(handle);
  if (e == nullptr || out_max_abs == nullptr) {
    Fail("invalid logit reference");
    return 1;
  }
  return Guarded(e, [&] { *out_max_abs = e->LogitMaxAbs(reference, count); });
}

ACCEL_B200_API int accel_llama_logits(AccelLlama* handle, float* out, int32_t count) {
  Engine* e = Cast(handle);
  if (e == nullptr) {
    Fail("invalid logit buffer");
    return 1;
  }
  return Guarded(e, [&] { e->Logits(out, count); });
}

ACCEL_B200_API int accel_llama_cache_rows(AccelLlama* handle, int32_t slot, int32_t layer, int32_t which, int32_t rows,
                                          float* out) {
  Engine* e = Cast(handle);
  if (e == nullptr) {
    Fail("invalid cache read");
    return 1;
  }
  return Guarded(e, [&] { e->CacheRows(slot, layer, which, rows, out); });
}

ACCEL_B200_API void accel_llama_reset(AccelLlama* handle) {
  Engine* e = Cast(handle);
  if (e == nullptr) return;
  std::lock_guard<std::mutex> lock(e->mu);
  e->filled = 0;
}

ACCEL_B200_API const char* accel_llama_last_error(void) { return g_llama_error.c_str(); }

ACCEL_B200_API void* accel_llama_stream(AccelLlama* handle) {
  Engine* e = Cast(handle);
  return e == nullptr ? nullptr : static_cast<void*>(e->stream);
}

}  // extern "C"
