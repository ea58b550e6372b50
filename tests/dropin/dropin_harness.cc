// C entry points into AccelEP's own runtime (src/runtime.cc, patched by
// reference_on_b200.patch) running on the B200 device.
//
// TEST INFRASTRUCTURE ONLY. tests/dropin/Makefile links this file with the
// reference's runtime, Llama model and one-matmul API compiled from a patched
// copy of the AccelEP sources, and with this repository's B200Device
// (accelep_b200/csrc/device.cc built against the host's accel/device.h).
// tests/test_dropin_gpu.py compares what these calls return with the
// reference on SimDevice (oracle/_ref): outputs within 1e-4, counters equal.
//
// Unlike the SimDevice harness (oracle/ref_harness.cc), the int8 planes here
// are device memory: each call uploads the weights as the plugin's compile
// step does (src/ep.cc:1440-1450 keeps packed planes in device buffers)
// before it resets the counters, so the counters cover the run alone.

#include "accel/device.h"
#include "accel/runtime.h"
#include "accel_b200_device.h"

#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <string>
#include <vector>

#define DROPIN_API extern "C" __attribute__((visibility("default")))

namespace {

thread_local std::string g_error;

template <typename F>
int Guard(F&& body) {
  try {
    body();
    g_error.clear();
    return 0;
  } catch (const std::exception& ex) {
    g_error = ex.what();
    return 1;
  }
}

accel::Device& B200() {
  static std::unique_ptr<accel::Device> dev = accel_b200::CreateB200Device();
  return *dev;
}

accel::OwnedBuffer ToDevice(const void* data, size_t bytes) {
  accel::OwnedBuffer buf;
  buf.device = &B200();
  buf.buffer = B200().Allocate(bytes);
  if (bytes > 0) B200().CopyHostToDevice(buf.buffer, data, bytes);
  return buf;
}

accel::Activation ActOf(int act) {
  return act == 1 ? accel::Activation::Relu : act == 2 ? accel::Activation::Gelu : accel::Activation::None;
}

// A packed int8 operand [rows, cols] whose plane points into device buffers.
accel::Operand Plane(const accel::OwnedBuffer& q, const accel::OwnedBuffer& scale, const accel::OwnedBuffer* zero,
                     int64_t rows, int64_t cols, int64_t axis) {
  accel::Operand op;
  op.quant = true;
  op.shape = {rows, cols};
  op.quant_plane.q = static_cast<const int8_t*>(q.buffer.data);
  op.quant_plane.scale = static_cast<const float*>(scale.buffer.data);
  op.quant_plane.zero = zero != nullptr ? static_cast<const int8_t*>(zero->buffer.data) : nullptr;
  op.quant_plane.shape = {rows, cols};
  op.quant_plane.axis = axis;
  return op;
}

void Stats(int64_t* out9) {
  const accel::AcceleratorStats s = accel::GetAcceleratorStats();
  const int64_t v[9] = {s.matmul_ops,     s.gemm_ops,          s.kernel_matmuls,   s.relu_epilogues, s.gelu_epilogues,
                        s.add_epilogues, s.device_transposes, s.bytes_to_device, s.bytes_to_host};
  std::memcpy(out9, v, sizeof(v));
}

}  // namespace

DROPIN_API const char* dropin_last_error(void) { return g_error.c_str(); }

DROPIN_API const char* dropin_device_name(void) {
  const char* name = nullptr;
  Guard([&] { name = B200().Name(); });
  return name;
}

// accel::ExecuteMatMul (src/runtime.cc:653-670) of host x [m, k] with an int8
// plane [k, n] (scale per `axis`: 1 columns, 0 rows, -1 one value; zero may
// be NULL), the activation, and an optional host residual [m, n]; the result
// comes back to `out`. stats9 receives the counters of the call alone.
DROPIN_API int dropin_execute_matmul_q(const float* x, int64_t m, int64_t k, const int8_t* q, const float* scale,
                                       const int8_t* zero, int64_t axis, int64_t n, int act, const float* residual,
                                       float* out, int64_t* stats9) {
  return Guard([&] {
    const int64_t scales = axis == 1 ? n : axis == 0 ? k : 1;
    accel::OwnedBuffer dq = ToDevice(q, static_cast<size_t>(k * n));
    accel::OwnedBuffer ds = ToDevice(scale, static_cast<size_t>(scales) * sizeof(float));
    accel::OwnedBuffer dz;
    if (zero != nullptr) dz = ToDevice(zero, static_cast<size_t>(scales));
    accel::ResetAcceleratorStats();
    accel::Operand a{x, nullptr, {m, k}};
    accel::Operand res{residual, nullptr, {m, n}};
    accel::ExecuteMatMul(B200(), a, Plane(dq, ds, zero != nullptr ? &dz : nullptr, k, n, axis), out, ActOf(act),
                         residual != nullptr ? &res : nullptr);
    Stats(stats9);
  });
}

// One block of the plugin's int8 MLP chain in RunKernel's order for a prenorm
// step (src/ep.cc:1602-1626): ExecuteMatMul(x, W1, Gelu) retained on the
// device, ExecuteMatMul(h, W2, residual x) retained as the pre-norm sum, then
// Device::RmsNorm; both results are read back. stats9 as above.
DROPIN_API int dropin_mlp_block(const float* x, int64_t m, int64_t hidden, int64_t inter, const int8_t* w1,
                                const float* s1, const int8_t* w2, const float* s2, const float* gamma, float eps,
                                float* pre_norm, float* out, int64_t* stats9) {
  return Guard([&] {
    accel::Device& dev = B200();
    accel::OwnedBuffer q1 = ToDevice(w1, static_cast<size_t>(hidden * inter));
    accel::OwnedBuffer c1 = ToDevice(s1, static_cast<size_t>(inter) * sizeof(float));
    accel::OwnedBuffer q2 = ToDevice(w2, static_cast<size_t>(inter * hidden));
    accel::OwnedBuffer c2 = ToDevice(s2, static_cast<size_t>(hidden) * sizeof(float));
    accel::OwnedBuffer g = ToDevice(gamma, static_cast<size_t>(hidden) * sizeof(float));
    accel::OwnedBuffer normed;
    normed.device = &dev;
    normed.buffer = dev.Allocate(static_cast<size_t>(m * hidden) * sizeof(float));
    accel::ResetAcceleratorStats();
    accel::OwnedBuffer h;
    accel::ExecuteMatMul(dev, accel::Operand{x, nullptr, {m, hidden}}, Plane(q1, c1, nullptr, hidden, inter, 1),
                         nullptr, accel::Activation::Gelu, nullptr, &h);
    accel::Operand h_op;
    h_op.on_device = &h;
    h_op.shape = h.shape;
    accel::Operand res{x, nullptr, {m, hidden}};
    accel::OwnedBuffer skip;
    accel::ExecuteMatMul(dev, h_op, Plane(q2, c2, nullptr, inter, hidden, 1), nullptr, accel::Activation::None, &res,
                         &skip);
    dev.RmsNorm(skip.buffer, g.buffer, normed.buffer, m, hidden, eps, 0);
    Stats(stats9);
    dev.CopyDeviceToHost(pre_norm, skip.buffer, static_cast<size_t>(m * hidden) * sizeof(float));
    dev.CopyDeviceToHost(out, normed.buffer, static_cast<size_t>(m * hidden) * sizeof(float));
  });
}
