// C entry points into the AccelEP reference, compiled from its own sources.
//
// TEST INFRASTRUCTURE ONLY. oracle/Makefile links this file with the
// reference's objects into oracle/_ref/libaccel_ref.so. Tests use it to pin
// the C restatement (oracle/restate.c) and bench.py's reference arm times it.
// The product library never links or calls it.
//
// Each wrapper takes host pointers. SimDevice keeps its "device" heap in host
// memory, so a DeviceBuffer that wraps a host pointer is what SimDevice
// itself would hand out (include/accel/device.h:28-32).

#include "accel/device.h"
#include "accel/runtime.h"
#include "accel/sim_add.h"
#include "accel/sim_attend.h"
#include "accel/sim_cache.h"
#include "accel/sim_embed.h"
#include "accel/sim_rmsnorm.h"
#include "accel/sim_rope.h"
#include "accel/sim_sample.h"
#include "accel/sim_silu.h"

#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <string>
#include <vector>

#define REF_API extern "C" __attribute__((visibility("default")))

namespace {

thread_local std::string g_ref_error;

accel::DeviceBuffer Wrap(const void* ptr, size_t bytes) {
  return accel::DeviceBuffer{const_cast<void*>(ptr), bytes, 0};
}

accel::Activation ActOf(int act) {
  return act == 1 ? accel::Activation::Relu : act == 2 ? accel::Activation::Gelu : accel::Activation::None;
}

template <typename F>
int Guard(F&& body) {
  try {
    body();
    g_ref_error.clear();
    return 0;
  } catch (const std::exception& ex) {
    g_ref_error = ex.what();
    return 1;
  }
}

accel::Device& Sim() {
  static std::unique_ptr<accel::Device> dev = accel::CreateSimDevice();
  return *dev;
}

}  // namespace

REF_API const char* ref_last_error(void) { return g_ref_error.c_str(); }

// src/sim_embed.cc:9-20 through SimDevice::Embedding (sim_device.cc:247-256).
REF_API int ref_embed(const int32_t* ids, int64_t id_offset, const float* table, float* out, int64_t seq,
                      int64_t hidden, int64_t vocab) {
  return Guard([&] {
    Sim().Embedding(Wrap(ids, static_cast<size_t>(id_offset + seq) * 4), id_offset,
                    Wrap(table, static_cast<size_t>(vocab * hidden) * 4), Wrap(out, static_cast<size_t>(seq * hidden) * 4),
                    seq, hidden, vocab);
  });
}

REF_API int ref_rmsnorm(const float* x, const float* w, float* y, int64_t rows, int64_t dim, float eps,
                        int64_t row_offset) {
  return Guard([&] {
    Sim().RmsNorm(Wrap(x, static_cast<size_t>((row_offset + rows) * dim) * 4), Wrap(w, static_cast<size_t>(dim) * 4),
                  Wrap(y, static_cast<size_t>(rows * dim) * 4), rows, dim, eps, row_offset);
  });
}

REF_API int ref_rope(float* states, const float* cos_t, const float* sin_t, int64_t seq, int64_t n_heads,
                     int64_t head_dim, int64_t position) {
  return Guard([&] {
    const size_t table = static_cast<size_t>((position + seq) * head_dim) * 4;
    Sim().Rope(Wrap(states, static_cast<size_t>(seq * n_heads * head_dim) * 4), Wrap(cos_t, table), Wrap(sin_t, table),
               seq, n_heads, head_dim, position);
  });
}

REF_API int ref_append_cache(const float* src, float* cache, int64_t seq, int64_t position, int64_t n_heads,
                             int64_t head_dim) {
  return Guard([&] {
    Sim().AppendCache(Wrap(src, static_cast<size_t>(seq * n_heads * head_dim) * 4),
                      Wrap(cache, static_cast<size_t>((position + seq) * n_heads * head_dim) * 4), seq, position,
                      n_heads, head_dim);
  });
}

REF_API int ref_attention(const float* q, const float* k, const float* v, float* scores, float* out, int64_t seq,
                          int64_t position, int64_t heads, int64_t kv_heads, int64_t head_dim) {
  return Guard([&] {
    const size_t kv = static_cast<size_t>((position + seq) * kv_heads * head_dim) * 4;
    const size_t qo = static_cast<size_t>(seq * heads * head_dim) * 4;
    Sim().Attention(Wrap(q, qo), Wrap(k, kv), Wrap(v, kv), Wrap(scores, static_cast<size_t>(position + seq) * 4),
                    Wrap(out, qo), seq, position, heads, kv_heads, head_dim);
  });
}

REF_API int ref_silu_mul(float* gate, const float* up, int64_t count) {
  return Guard([&] { Sim().SiluMul(Wrap(gate, static_cast<size_t>(count) * 4), Wrap(up, static_cast<size_t>(count) * 4), count); });
}

REF_API int ref_residual_add(float* dest, const float* extra, int64_t count) {
  return Guard(
      [&] { Sim().ResidualAdd(Wrap(dest, static_cast<size_t>(count) * 4), Wrap(extra, static_cast<size_t>(count) * 4), count); });
}

REF_API int ref_sample(const float* logits, int32_t* chosen, int64_t index, int64_t vocab, float temperature,
                       uint32_t* rng, int top_k) {
  return Guard([&] {
    Sim().SampleToken(Wrap(logits, static_cast<size_t>(vocab) * 4), Wrap(chosen, static_cast<size_t>(index + 1) * 4),
                      index, vocab, temperature, rng, top_k);
  });
}

// SimDevice::MatMul -> PackedMatMul (sim_device.cc:185-196, :331-369).
REF_API int ref_matmul(const float* a, const float* b, float* c, int64_t m, int64_t k, int64_t n) {
  return Guard([&] {
    Sim().MatMul(Wrap(a, static_cast<size_t>(m * k) * 4), Wrap(b, static_cast<size_t>(k * n) * 4),
                 Wrap(c, static_cast<size_t>(m * n) * 4), m, k, n);
  });
}

REF_API void ref_reference_matmul(const float* a, const float* b, float* c, int64_t m, int64_t k, int64_t n) {
  accel::ReferenceMatMul(a, b, c, m, k, n);
}

REF_API int ref_transpose(const float* src, float* dst, int64_t rows, int64_t cols) {
  return Guard([&] {
    Sim().Transpose(Wrap(src, static_cast<size_t>(rows * cols) * 4), Wrap(dst, static_cast<size_t>(rows * cols) * 4),
                    rows, cols);
  });
}

// SimDevice::GemmEpilogue (sim_device.cc:211-245). act: 0 none, 1 relu, 2 gelu.
REF_API int ref_gemm_epilogue(float* c, int64_t m, int64_t n, float alpha, const float* bias,
                              const int64_t* bias_shape, int bias_rank, float beta, int act) {
  return Guard([&] {
    std::vector<int64_t> shape(bias_shape, bias_shape + (bias != nullptr ? bias_rank : 0));
    int64_t count = 1;
    for (int64_t d : shape) count *= d;
    const accel::DeviceBuffer bias_buf = Wrap(bias, static_cast<size_t>(count) * 4);
    Sim().GemmEpilogue(Wrap(c, static_cast<size_t>(m * n) * 4), m, n, alpha, bias != nullptr ? &bias_buf : nullptr, shape,
                       beta, ActOf(act));
  });
}

// MatMulQuantized with a right-hand plane (sim_device.cc:541-602).
REF_API int ref_matmul_quantized(const float* a, const int8_t* q, const float* scale, const int8_t* zero,
                                 const int64_t* shape, int rank, int64_t axis, int64_t offset, float* c, int64_t m,
                                 int64_t k, int64_t n) {
  return Guard([&] {
    accel::QuantPlane plane;
    plane.q = q;
    plane.scale = scale;
    plane.zero = zero;
    plane.shape.assign(shape, shape + rank);
    plane.axis = axis;
    plane.offset = offset;
    accel::MatMulQuantized(a, nullptr, nullptr, &plane, c, m, k, n);
  });
}

// ExecuteMatMul with an int8 right-hand operand (runtime.cc:272-350):
// x [m, k] host, q [k, n], per-axis scale, optional zero and residual [m, n].
REF_API int ref_execute_matmul_q(const float* x, int64_t m, int64_t k, const int8_t* q, const float* scale,
                                 const int8_t* zero, int64_t axis, int64_t n, int act, const float* residual,
                                 float* out) {
  return Guard([&] {
    accel::Operand a{x, nullptr, {m, k}};
    accel::Operand b;
    b.quant = true;
    b.shape = {k, n};
    b.quant_plane.q = q;
    b.quant_plane.scale = scale;
    b.quant_plane.zero = zero;
    b.quant_plane.shape = {k, n};
    b.quant_plane.axis = axis;
    accel::Operand res{residual, nullptr, {m, n}};
    accel::ExecuteMatMul(Sim(), a, b, out, ActOf(act), residual != nullptr ? &res : nullptr);
  });
}

// One block of the plugin's int8 MLP chain, in the order RunKernel issues it
// for a prenorm step (ep.cc:1602-1626): ExecuteMatMul(x, W1, Gelu) retained on
// the device, ExecuteMatMul(h, W2, residual x) retained as the pre-norm sum,
// then Device::RmsNorm. Writes the normed rows and the pre-norm sum.
REF_API int ref_mlp_block(const float* x, int64_t m, int64_t hidden, int64_t inter, const int8_t* w1,
                          const float* s1, const int8_t* w2, const float* s2, const float* gamma, float eps,
                          float* pre_norm, float* out) {
  return Guard([&] {
    accel::Device& dev = Sim();
    auto plane = [](const int8_t* q, const float* s, int64_t rows, int64_t cols) {
      accel::Operand op;
      op.quant = true;
      op.shape = {rows, cols};
      op.quant_plane.q = q;
      op.quant_plane.scale = s;
      op.quant_plane.shape = {rows, cols};
      op.quant_plane.axis = 1;
      return op;
    };
    accel::OwnedBuffer h;
    accel::ExecuteMatMul(dev, accel::Operand{x, nullptr, {m, hidden}}, plane(w1, s1, hidden, inter), nullptr,
                         accel::Activation::Gelu, nullptr, &h);
    accel::Operand h_op;
    h_op.on_device = &h;
    h_op.shape = h.shape;
    accel::Operand res{x, nullptr, {m, hidden}};
    accel::OwnedBuffer skip;
    accel::ExecuteMatMul(dev, h_op, plane(w2, s2, inter, hidden), nullptr, accel::Activation::None, &res, &skip);
    std::memcpy(pre_norm, skip.buffer.data, static_cast<size_t>(m * hidden) * 4);
    dev.RmsNorm(skip.buffer, Wrap(gamma, static_cast<size_t>(hidden) * 4), Wrap(out, static_cast<size_t>(m * hidden) * 4),
                m, hidden, eps, 0);
  });
}

REF_API void ref_reset_stats(void) { accel::ResetAcceleratorStats(); }

// {matmul_ops, gemm_ops, kernel_matmuls, relu, gelu, add, transposes, bytes_to_device, bytes_to_host}
REF_API void ref_stats(int64_t* out9) {
  const accel::AcceleratorStats s = accel::GetAcceleratorStats();
  const int64_t v[9] = {s.matmul_ops,     s.gemm_ops,          s.kernel_matmuls,   s.relu_epilogues, s.gelu_epilogues,
                        s.add_epilogues, s.device_transposes, s.bytes_to_device, s.bytes_to_host};
  std::memcpy(out9, v, sizeof(v));
}
