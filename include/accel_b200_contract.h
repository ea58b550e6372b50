// accel_b200_contract.h: a mirror of AccelEP's device contract, used when this
// library is built on its own.
//
// The declarations must match the host project's accel/device.h and the
// QuantPlane of accel/runtime.h type for type and virtual for virtual,
// because B200Device overrides them and the host project calls them through
// its own header (include/accel/device.h:11-125 and include/accel/runtime.h:71-78
// of the reference). The one addition is Device::MatMulQ8, the int8 entry
// the host runtime calls in place of the host-side MatMulQuantized.
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <utility>
#include <vector>

namespace accel {

enum class Activation { None, Relu, Gelu };

// Memory owned by a Device. `id` is 0 for a slice of another buffer.
struct DeviceBuffer {
  void* data = nullptr;
  size_t bytes = 0;
  uint64_t id = 0;
};

// Frees `buffer` on `device` when destroyed; movable, not copyable.
struct OwnedBuffer {
  class Device* device = nullptr;
  DeviceBuffer buffer{};
  std::vector<int64_t> shape;

  OwnedBuffer() = default;
  OwnedBuffer(const OwnedBuffer&) = delete;
  OwnedBuffer& operator=(const OwnedBuffer&) = delete;
  OwnedBuffer(OwnedBuffer&& other) noexcept
      : device(other.device), buffer(other.buffer), shape(std::move(other.shape)) {
    other.device = nullptr;
    other.buffer = {};
  }
  OwnedBuffer& operator=(OwnedBuffer&& other) noexcept {
    if (this != &other) {
      Reset();
      device = other.device;
      buffer = other.buffer;
      shape = std::move(other.shape);
      other.device = nullptr;
      other.buffer = {};
    }
    return *this;
  }
  ~OwnedBuffer() { Reset(); }
  void Reset() noexcept;
};

// An int8 constant kept packed; axis < 0 is one scale for the whole tensor.
struct QuantPlane {
  const int8_t* q = nullptr;
  const float* scale = nullptr;
  const int8_t* zero = nullptr;
  std::vector<int64_t> shape;
  int64_t axis = -1;
  int64_t offset = 0;
};

class Device {
 public:
  virtual ~Device() = default;
  virtual const char* Name() const = 0;
  virtual DeviceBuffer Allocate(size_t bytes) = 0;
  virtual void Free(DeviceBuffer buffer) = 0;
  virtual void CopyHostToDevice(DeviceBuffer dst, const void* src, size_t bytes) = 0;
  virtual void CopyDeviceToHost(void* dst, DeviceBuffer src, size_t bytes) = 0;
  virtual void MatMul(DeviceBuffer a, DeviceBuffer b, DeviceBuffer c, int64_t m, int64_t k, int64_t n) = 0;
  virtual void Transpose(DeviceBuffer src, DeviceBuffer dst, int64_t rows, int64_t cols) = 0;
  virtual void GemmEpilogue(DeviceBuffer c, int64_t m, int64_t n, float alpha, const DeviceBuffer* bias,
                            const std::vector<int64_t>& bias_shape, float beta,
                            Activation activation = Activation::None) = 0;
  virtual void Embedding(DeviceBuffer ids, int64_t id_offset, DeviceBuffer table, DeviceBuffer out, int64_t seq,
                         int64_t hidden, int64_t vocab) = 0;
  virtual void RmsNorm(DeviceBuffer x, DeviceBuffer weight, DeviceBuffer y, int64_t rows, int64_t dim, float eps,
                       int64_t row_offset) = 0;
  virtual void Rope(DeviceBuffer states, DeviceBuffer cos_table, DeviceBuffer sin_table, int64_t seq, int64_t n_heads,
                    int64_t head_dim, int64_t position) = 0;
  virtual void AppendCache(DeviceBuffer src, DeviceBuffer cache, int64_t seq, int64_t position, int64_t n_heads,
                           int64_t head_dim) = 0;
  virtual void Attention(DeviceBuffer q, DeviceBuffer k, DeviceBuffer v, DeviceBuffer scores, DeviceBuffer out,
                         int64_t seq, int64_t position, int64_t heads, int64_t kv_heads, int64_t head_dim) = 0;
  virtual void SiluMul(DeviceBuffer gate, DeviceBuffer up, int64_t count) = 0;
  virtual void ResidualAdd(DeviceBuffer dest, DeviceBuffer extra, int64_t count) = 0;
  virtual void SampleToken(DeviceBuffer logits, DeviceBuffer chosen_ids, int64_t chosen_index, int64_t vocab,
                           float temperature, uint32_t* rng_state, int top_k) = 0;
  // Added entry: c[m, n] = a[m, k] @ dequant(b) with `a` and `c` device
  // buffers and `b` a plane of device pointers (replaces the host call
  // MatMulQuantized at src/runtime.cc:326 of the reference).
  virtual void MatMulQ8(DeviceBuffer a, const QuantPlane& b, DeviceBuffer c, int64_t m, int64_t k, int64_t n) = 0;
};

}  // namespace accel
