// B200Device: AccelEP's accel::Device on one B200 (include/accel/device.h:69-125
// of the reference; SimDevice in src/sim_device.cc:126-373 is the CPU model).
//
// Allocations are zero-filled HBM from the stream-ordered pool; every call
// is a launch on the device's one stream, checked on the host with the same
// range rules and exception types SimDevice uses (sim_device.cc:44-102):
// std::invalid_argument, std::overflow_error, std::logic_error for an
// unknown free, std::bad_alloc. CopyDeviceToHost synchronizes the stream.
#include <cuda_runtime.h>

#include <atomic>
#include <cstring>
#include <mutex>
#include <new>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "accel_b200.h"
#include "accel_b200_device.h"
#include "stats.h"

namespace accel {
#ifndef ACCEL_B200_USE_HOST_CONTRACT
// src/device_buffer.cc:5-12 of the reference, for the mirrored contract.
void OwnedBuffer::Reset() noexcept {
  if (device != nullptr && buffer.data != nullptr) device->Free(buffer);
  device = nullptr;
  buffer = {};
  shape.clear();
}
#endif
}  // namespace accel

namespace accel_b200 {
namespace {

std::atomic<uint64_t> g_next_id{1};
std::atomic<int64_t> g_live{0};

size_t CheckedBytes(int64_t rows, int64_t cols) {
  if (rows < 0 || cols < 0) throw std::invalid_argument("negative matrix dimension");
  if (rows != 0 && static_cast<uint64_t>(cols) > (UINT64_MAX / sizeof(float)) / static_cast<uint64_t>(rows)) {
    throw std::overflow_error("matrix is too large");
  }
  return static_cast<size_t>(rows) * static_cast<size_t>(cols) * sizeof(float);
}

int64_t CheckedSpan(int64_t offset, int64_t count) {
  if (offset < 0 || count < 0) throw std::invalid_argument("negative matrix dimension");
  if (offset > INT64_MAX - count) throw std::overflow_error("matrix is too large");
  return offset + count;
}

size_t CheckedFloats(int64_t depth, int64_t rows, int64_t cols) {
  if (depth < 0 || rows < 0 || cols < 0) throw std::invalid_argument("negative matrix dimension");
  if (depth == 0 || rows == 0 || cols == 0) return 0;
  if (static_cast<uint64_t>(rows) > UINT64_MAX / static_cast<uint64_t>(depth)) throw std::overflow_error("matrix is too large");
  const uint64_t plane = static_cast<uint64_t>(depth) * static_cast<uint64_t>(rows);
  if (static_cast<uint64_t>(cols) > UINT64_MAX / plane) throw std::overflow_error("matrix is too large");
  const uint64_t count = plane * static_cast<uint64_t>(cols);
  if (count > UINT64_MAX / sizeof(float)) throw std::overflow_error("matrix is too large");
  return static_cast<size_t>(count * sizeof(float));
}

size_t CheckedIntBytes(int64_t count) {
  if (count < 0) throw std::invalid_argument("negative matrix dimension");
  if (count != 0 && static_cast<uint64_t>(count) > UINT64_MAX / sizeof(int32_t)) throw std::overflow_error("matrix is too large");
  return static_cast<size_t>(count) * sizeof(int32_t);
}

void RequireBytes(const accel::DeviceBuffer& buffer, size_t need, const char* what) {
  if (need == 0) return;
  if (buffer.data == nullptr || buffer.bytes < need) throw std::invalid_argument(what);
}

// Turns a kernel-ABI status into the reference's exception types.
void Check(int rc) {
  if (rc == ACCEL_B200_OK) return;
  const std::string msg = accel_b200_last_error();
  if (rc == ACCEL_B200_EINVAL || rc == ACCEL_B200_EDEVICE) throw std::invalid_argument(msg);
  if (rc == ACCEL_B200_EOVERFLOW) throw std::overflow_error(msg);
  if (rc == ACCEL_B200_ENOMEM) throw std::bad_alloc();
  throw std::runtime_error(msg);
}

void CheckCuda(cudaError_t err, const char* what) {
  if (err == cudaErrorMemoryAllocation) throw std::bad_alloc();
  if (err != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(err));
}

// The counters SimDevice keeps (src/sim_device.cc:171-208): the host
// project's own (src/runtime.cc:450-458) when this file is built inside it,
// this library's otherwise.
#ifdef ACCEL_B200_USE_HOST_CONTRACT
void CountKernelMatmul() { accel::NoteKernelMatmul(); }
void CountTranspose() { accel::NoteDeviceTranspose(); }
void CountToDevice(size_t bytes) { accel::NoteBytesToDevice(bytes); }
void CountToHost(size_t bytes) { accel::NoteBytesToHost(bytes); }
#else
void CountKernelMatmul() { NoteKernelMatmuls(1); }
void CountTranspose() {}
void CountToDevice(size_t bytes) { NoteBytesToDevice(bytes); }
void CountToHost(size_t bytes) { NoteBytesToHost(bytes); }
#endif

int32_t ActCode(accel::Activation act) {
  return act == accel::Activation::Relu ? ACCEL_B200_ACT_RELU
         : act == accel::Activation::Gelu ? ACCEL_B200_ACT_GELU
                                          : ACCEL_B200_ACT_NONE;
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

class B200Device final : public accel::Device {
 public:
  explicit B200Device(int ordinal) : ordinal_(ordinal) {
    DeviceScope scope(ordinal_);
    CheckCuda(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "stream");
    CheckCuda(cudaMalloc(&status_, 16), "status word");
    CheckCuda(cudaMemset(status_, 0, 16), "status word");
    CheckCuda(cudaMallocHost(&pinned_, 16), "pinned word");
  }

  ~B200Device() override {
    DeviceScope scope(ordinal_);
    cudaStreamSynchronize(stream_);
    if (workspace_ != nullptr) cudaFree(workspace_);
    cudaFree(status_);
    cudaFreeHost(pinned_);
    cudaStreamDestroy(stream_);
  }

  const char* Name() const override { return "b200"; }

  accel::DeviceBuffer Allocate(size_t bytes) override {
    DeviceScope scope(ordinal_);
    const size_t store = bytes == 0 ? 1 : bytes;
    void* ptr = nullptr;
    if (cudaMallocAsync(&ptr, store, stream_) != cudaSuccess || ptr == nullptr) {
      cudaGetLastError();
      throw std::bad_alloc();
    }
    CheckCuda(cudaMemsetAsync(ptr, 0, store, stream_), "zero fill");
    const uint64_t id = g_next_id.fetch_add(1, std::memory_order_relaxed);
    {
      std::lock_guard<std::mutex> lock(mu_);
      live_.emplace(ptr, Live{bytes, id});
    }
    g_live.fetch_add(1, std::memory_order_relaxed);
    return accel::DeviceBuffer{ptr, bytes, id};
  }

  void Free(accel::DeviceBuffer buffer) override {
    if (buffer.data == nullptr) return;
    DeviceScope scope(ordinal_);
    {
      std::lock_guard<std::mutex> lock(mu_);
      auto it = live_.find(buffer.data);
      if (it == live_.end() || it->second.bytes != buffer.bytes || it->second.id != buffer.id) {
        throw std::logic_error("free of unknown device buffer");
      }
      live_.erase(it);
    }
    g_live.fetch_sub(1, std::memory_order_relaxed);
    cudaFreeAsync(buffer.data, stream_);
  }

  void CopyHostToDevice(accel::DeviceBuffer dst, const void* src, size_t bytes) override {
    if (bytes == 0) return;
    if (src == nullptr || dst.data == nullptr || bytes > dst.bytes) throw std::invalid_argument("invalid host-to-device copy");
    DeviceScope scope(ordinal_);
    CheckCuda(cudaMemcpyAsync(dst.data, src, bytes, cudaMemcpyHostToDevice, stream_), "host-to-device copy");
    CountToDevice(bytes);
  }

  void CopyDeviceToHost(void* dst, accel::DeviceBuffer src, size_t bytes) override {
    if (bytes == 0) return;
    if (dst == nullptr || src.data == nullptr || bytes > src.bytes) throw std::invalid_argument("invalid device-to-host copy");
    DeviceScope scope(ordinal_);
    CheckCuda(cudaMemcpyAsync(dst, src.data, bytes, cudaMemcpyDeviceToHost, stream_), "device-to-host copy");
    CheckCuda(cudaStreamSynchronize(stream_), "device-to-host copy");
    CountToHost(bytes);
  }

  void MatMul(accel::DeviceBuffer a, accel::DeviceBuffer b, accel::DeviceBuffer c, int64_t m, int64_t k,
              int64_t n) override {
    RequireBytes(a, CheckedBytes(m, k), "MatMul A is out of range");
    RequireBytes(b, CheckedBytes(k, n), "MatMul B is out of range");
    RequireBytes(c, CheckedBytes(m, n), "MatMul C is out of range");
    DeviceScope scope(ordinal_);
    Check(accel_b200_matmul(static_cast<const float*>(a.data), static_cast<const float*>(b.data),
                            static_cast<float*>(c.data), m, k, n, stream_));
    CountKernelMatmul();
  }

  void Transpose(accel::DeviceBuffer src, accel::DeviceBuffer dst, int64_t rows, int64_t cols) override {
    RequireBytes(src, CheckedBytes(rows, cols), "Transpose source is out of range");
    RequireBytes(dst, CheckedBytes(cols, rows), "Transpose destination is out of range");
    DeviceScope scope(ordinal_);
    Check(accel_b200_transpose(static_cast<const float*>(src.data), static_cast<float*>(dst.data), rows, cols, stream_));
    CountTranspose();
  }

  void GemmEpilogue(accel::DeviceBuffer c, int64_t m, int64_t n, float alpha, const accel::DeviceBuffer* bias,
                    const std::vector<int64_t>& bias_shape, float beta, accel::Activation activation) override {
    RequireBytes(c, CheckedBytes(m, n), "Gemm epilogue destination is out of range");
    if (bias != nullptr) {
      int64_t elems = 1;
      for (int64_t dim : bias_shape) {
        if (dim < 0) throw std::invalid_argument("negative bias shape");
        elems *= dim;
      }
      RequireBytes(*bias, static_cast<size_t>(elems) * sizeof(float), "Gemm bias is out of range");
    }
    DeviceScope scope(ordinal_);
    Check(accel_b200_gemm_epilogue(static_cast<float*>(c.data), m, n, alpha,
                                   bias != nullptr ? static_cast<const float*>(bias->data) : nullptr,
                                   bias_shape.empty() ? nullptr : bias_shape.data(),
                                   static_cast<int32_t>(bias_shape.size()), beta, ActCode(activation), stream_));
  }

  void Embedding(accel::DeviceBuffer ids, int64_t id_offset, accel::DeviceBuffer table, accel::DeviceBuffer out,
                 int64_t seq, int64_t hidden, int64_t vocab) override {
    const int64_t id_count = CheckedSpan(id_offset, seq);
    RequireBytes(ids, CheckedIntBytes(id_count), "Embedding ids are out of range");
    RequireBytes(table, CheckedBytes(vocab, hidden), "Embedding table is out of range");
    RequireBytes(out, CheckedBytes(seq, hidden), "Embedding output is out of range");
    DeviceScope scope(ordinal_);
    CheckCuda(cudaMemsetAsync(status_, 0, sizeof(int32_t), stream_), "status word");
    Check(accel_b200_embed(static_cast<const int32_t*>(ids.data), id_offset, static_cast<const float*>(table.data),
                           static_cast<float*>(out.data), seq, hidden, vocab, static_cast<int32_t*>(status_), stream_));
    // The reference throws from inside the call (src/sim_embed.cc:13-15), so
    // the id check is read back here rather than at the next copy.
    CheckCuda(cudaMemcpyAsync(pinned_, status_, sizeof(int32_t), cudaMemcpyDeviceToHost, stream_), "status word");
    CheckCuda(cudaStreamSynchronize(stream_), "embedding");
    if (*static_cast<int32_t*>(pinned_) & ACCEL_B200_STATUS_BAD_TOKEN) {
      throw std::invalid_argument("token id is outside the vocabulary");
    }
  }

  void RmsNorm(accel::DeviceBuffer x, accel::DeviceBuffer weight, accel::DeviceBuffer y, int64_t rows, int64_t dim,
               float eps, int64_t row_offset) override {
    const int64_t x_rows = CheckedSpan(row_offset, rows);
    RequireBytes(x, CheckedBytes(x_rows, dim), "RmsNorm input is out of range");
    RequireBytes(weight, CheckedBytes(dim, 1), "RmsNorm weight is out of range");
    RequireBytes(y, CheckedBytes(rows, dim), "RmsNorm output is out of range");
    DeviceScope scope(ordinal_);
    Check(accel_b200_rmsnorm(static_cast<const float*>(x.data), static_cast<const float*>(weight.data),
                             static_cast<float*>(y.data), rows, dim, eps, row_offset, stream_));
  }

  void Rope(accel::DeviceBuffer states, accel::DeviceBuffer cos_table, accel::DeviceBuffer sin_table, int64_t seq,
            int64_t n_heads, int64_t head_dim, int64_t position) override {
    const int64_t positions = CheckedSpan(position, seq);
    RequireBytes(states, CheckedFloats(seq, n_heads, head_dim), "Rope states are out of range");
    RequireBytes(cos_table, CheckedBytes(positions, head_dim), "Rope cos table is out of range");
    RequireBytes(sin_table, CheckedBytes(positions, head_dim), "Rope sin table is out of range");
    DeviceScope scope(ordinal_);
    Check(accel_b200_rope(static_cast<float*>(states.data), static_cast<const float*>(cos_table.data),
                          static_cast<const float*>(sin_table.data), seq, n_heads, head_dim, position, stream_));
  }

  void AppendCache(accel::DeviceBuffer src, accel::DeviceBuffer cache, int64_t seq, int64_t position, int64_t n_heads,
                   int64_t head_dim) override {
    const int64_t rows = CheckedSpan(position, seq);
    RequireBytes(src, CheckedFloats(seq, n_heads, head_dim), "AppendCache source is out of range");
    RequireBytes(cache, CheckedFloats(rows, n_heads, head_dim), "AppendCache cache is out of range");
    DeviceScope scope(ordinal_);
    Check(accel_b200_append_cache(static_cast<const float*>(src.data), static_cast<float*>(cache.data), seq, position,
                                  n_heads, head_dim, stream_));
  }

  void Attention(accel::DeviceBuffer q, accel::DeviceBuffer k, accel::DeviceBuffer v, accel::DeviceBuffer scores,
                 accel::DeviceBuffer out, int64_t seq, int64_t position, int64_t heads, int64_t kv_heads,
                 int64_t head_dim) override {
    if (kv_heads <= 0 || (heads > 0 && heads % kv_heads != 0)) {
      throw std::invalid_argument("Attention kv heads are out of range");
    }
    const int64_t seen = CheckedSpan(position, seq);
    RequireBytes(q, CheckedFloats(seq, heads, head_dim), "Attention query is out of range");
    RequireBytes(k, CheckedFloats(seen, kv_heads, head_dim), "Attention key is out of range");
    RequireBytes(v, CheckedFloats(seen, kv_heads, head_dim), "Attention value is out of range");
    RequireBytes(scores, CheckedBytes(seen, 1), "Attention scores are out of range");
    RequireBytes(out, CheckedFloats(seq, heads, head_dim), "Attention output is out of range");
    DeviceScope scope(ordinal_);
    Check(accel_b200_attention(static_cast<const float*>(q.data), static_cast<const float*>(k.data),
                               static_cast<const float*>(v.data), static_cast<float*>(out.data), seq, position, heads,
                               kv_heads, head_dim, stream_));
  }

  void SiluMul(accel::DeviceBuffer gate, accel::DeviceBuffer up, int64_t count) override {
    const size_t bytes = CheckedBytes(count, 1);
    RequireBytes(gate, bytes, "SiluMul gate is out of range");
    RequireBytes(up, bytes, "SiluMul up is out of range");
    DeviceScope scope(ordinal_);
    Check(accel_b200_silu_mul(static_cast<float*>(gate.data), static_cast<const float*>(up.data), count, stream_));
  }

  void ResidualAdd(accel::DeviceBuffer dest, accel::DeviceBuffer extra, int64_t count) override {
    const size_t bytes = CheckedBytes(count, 1);
    RequireBytes(dest, bytes, "ResidualAdd destination is out of range");
    RequireBytes(extra, bytes, "ResidualAdd extra is out of range");
    DeviceScope scope(ordinal_);
    Check(accel_b200_residual_add(static_cast<float*>(dest.data), static_cast<const float*>(extra.data), count, stream_));
  }

  void SampleToken(accel::DeviceBuffer logits, accel::DeviceBuffer chosen_ids, int64_t chosen_index, int64_t vocab,
                   float temperature, uint32_t* rng_state, int top_k) override {
    if (vocab <= 0 || chosen_index < 0) throw std::invalid_argument("SampleToken is out of range");
    if (rng_state == nullptr) throw std::invalid_argument("SampleToken rng is out of range");
    RequireBytes(logits, CheckedBytes(vocab, 1), "SampleToken logits are out of range");
    RequireBytes(chosen_ids, CheckedIntBytes(CheckedSpan(chosen_index, 1)), "SampleToken ids are out of range");
    DeviceScope scope(ordinal_);
    // The reference keeps the xorshift state in host memory; it travels to
    // the device for the draw and comes back advanced.
    uint32_t* dev_rng = reinterpret_cast<uint32_t*>(static_cast<char*>(status_) + 8);
    uint32_t* host_word = reinterpret_cast<uint32_t*>(static_cast<char*>(pinned_) + 8);
    *host_word = *rng_state;
    CheckCuda(cudaMemcpyAsync(dev_rng, host_word, 4, cudaMemcpyHostToDevice, stream_), "rng state");
    Check(accel_b200_sample(static_cast<const float*>(logits.data), static_cast<int32_t*>(chosen_ids.data), chosen_index,
                            vocab, temperature, dev_rng, top_k, stream_));
    CheckCuda(cudaMemcpyAsync(host_word, dev_rng, 4, cudaMemcpyDeviceToHost, stream_), "rng state");
    CheckCuda(cudaStreamSynchronize(stream_), "SampleToken");
    *rng_state = *host_word;
  }

  void MatMulQ8(accel::DeviceBuffer a, const accel::QuantPlane& b, accel::DeviceBuffer c, int64_t m, int64_t k,
                int64_t n) override {
    RequireBytes(a, CheckedBytes(m, k), "quantized MatMul A is out of range");
    RequireBytes(c, CheckedBytes(m, n), "quantized MatMul C is out of range");
    if (m < 0 || k < 0 || n < 0) throw std::invalid_argument("quantized MatMul is out of range");
    if (k * n != 0 && (b.q == nullptr || b.scale == nullptr)) throw std::invalid_argument("quantized MatMul is missing an operand");
    accel_b200_q8_plane plane = MapPlane(b, k, n);
    DeviceScope scope(ordinal_);
    const size_t need = accel_b200_matmul_q8_workspace(m, k, n);
    void* ws = Workspace(need);
    Check(accel_b200_matmul_q8(static_cast<const float*>(a.data), k, &plane, static_cast<float*>(c.data), n, m, k, n,
                               nullptr, ws, need, stream_));
    CountKernelMatmul();
  }

 private:
  struct Live {
    size_t bytes;
    uint64_t id;
  };

  // A QuantPlane addresses its tensor with `offset` plus the [k, n] index;
  // its scale axis may be a leading (batch) axis, a row axis, a column axis
  // or none (DequantAt, src/sim_device.cc:406-424). Map it onto the kernel's
  // 2-D plane.
  static accel_b200_q8_plane MapPlane(const accel::QuantPlane& b, int64_t k, int64_t n) {
    accel_b200_q8_plane p{b.q, b.scale, b.zero, b.offset, -1};
    const int rank = static_cast<int>(b.shape.size());
    if (b.axis < 0) return p;
    if (rank < 2 || b.axis >= rank) throw std::invalid_argument("quantized MatMul plane axis is out of range");
    if (b.shape[rank - 2] != k || b.shape[rank - 1] != n) throw std::invalid_argument("quantized MatMul plane shape");
    if (b.axis == rank - 1) {
      p.axis = 1;
    } else if (b.axis == rank - 2) {
      p.axis = 0;
    } else {
      int64_t stride = 1;
      for (int d = rank - 1; d > b.axis; --d) stride *= b.shape[d];
      const int64_t coord = (b.offset / stride) % b.shape[b.axis];
      p.scale = b.scale + coord;
      p.zero = b.zero != nullptr ? b.zero + coord : nullptr;
      p.axis = -1;
    }
    if (p.axis >= 0 && b.offset % (k * n) != 0) throw std::invalid_argument("quantized MatMul plane offset");
    return p;
  }

  void* Workspace(size_t bytes) {
    if (bytes == 0) return nullptr;
    if (bytes > workspace_bytes_) {
      if (workspace_ != nullptr) {
        cudaStreamSynchronize(stream_);
        cudaFree(workspace_);
        workspace_ = nullptr;
      }
      CheckCuda(cudaMalloc(&workspace_, bytes), "workspace");
      CheckCuda(cudaMemsetAsync(workspace_, 0, bytes, stream_), "workspace");  // arrival counters start at zero
      workspace_bytes_ = bytes;
    }
    return workspace_;
  }

  int ordinal_;
  cudaStream_t stream_ = nullptr;
  void* status_ = nullptr;
  void* pinned_ = nullptr;
  void* workspace_ = nullptr;
  size_t workspace_bytes_ = 0;
  std::mutex mu_;
  std::unordered_map<void*, Live> live_;
};

}  // namespace

std::unique_ptr<accel::Device> CreateB200Device(int ordinal) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    throw std::runtime_error("no CUDA device is available for the B200 backend");
  }
  if (ordinal < 0) CheckCuda(cudaGetDevice(&ordinal), "current device");
  if (ordinal >= count) throw std::invalid_argument("CUDA ordinal is out of range");
  return std::unique_ptr<accel::Device>(new B200Device(ordinal));
}

int64_t LiveB200Allocs() { return g_live.load(std::memory_order_relaxed); }

}  // namespace accel_b200
