// Test support: a C interface over the accel::Device virtual calls of the
// B200 device, so that tests/test_device_gpu.py can drive the drop-in seam
// (include/accel/device.h:69-125 of the reference, plus MatMulQ8) from Python
// and compare each call with the CPU checker. Built by the test with g++
// against include/ and accelep_b200/lib/libaccelep_b200.so. Buffers are kept
// in a table and named by integer handles; a call that throws returns the
// exception's kind (1 invalid_argument, 2 overflow_error, 3 logic_error,
// 4 bad_alloc, 5 runtime_error, 6 other) and keeps its message.
#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <new>
#include <stdexcept>
#include <string>
#include <vector>

#include "accel_b200_device.h"

namespace {
struct Shim {
  std::unique_ptr<accel::Device> dev;
  std::vector<accel::DeviceBuffer> bufs;
};
thread_local std::string g_msg;

template <typename F>
int Guard(F f) {
  try {
    f();
    g_msg.clear();
    return 0;
  } catch (const std::invalid_argument& e) {
    g_msg = e.what();
    return 1;
  } catch (const std::overflow_error& e) {
    g_msg = e.what();
    return 2;
  } catch (const std::logic_error& e) {
    g_msg = e.what();
    return 3;
  } catch (const std::bad_alloc& e) {
    g_msg = e.what();
    return 4;
  } catch (const std::runtime_error& e) {
    g_msg = e.what();
    return 5;
  } catch (const std::exception& e) {
    g_msg = e.what();
    return 6;
  }
}

accel::DeviceBuffer& B(void* s, int h) { return static_cast<Shim*>(s)->bufs.at(static_cast<size_t>(h)); }
accel::Device& D(void* s) { return *static_cast<Shim*>(s)->dev; }
}  // namespace

extern "C" {

const char* shim_error(void) { return g_msg.c_str(); }

void* shim_create(void) {
  void* out = nullptr;
  Guard([&] {
    auto s = std::make_unique<Shim>();
    s->dev = accel_b200::CreateB200Device(-1);
    out = s.release();
  });
  return out;
}

void shim_destroy(void* s) { delete static_cast<Shim*>(s); }

const char* shim_name(void* s) { return D(s).Name(); }

int64_t shim_live(void) { return accel_b200::LiveB200Allocs(); }

// Allocates `bytes`; the handle goes to *handle.
int shim_alloc(void* s, int64_t bytes, int* handle) {
  return Guard([&] {
    accel::DeviceBuffer b = D(s).Allocate(static_cast<size_t>(bytes));
    static_cast<Shim*>(s)->bufs.push_back(b);
    *handle = static_cast<int>(static_cast<Shim*>(s)->bufs.size() - 1);
  });
}

// A buffer the device does not know: `bytes` at an address it never returned.
int shim_forged(void* s, int64_t bytes, int* handle) {
  accel::DeviceBuffer b;
  b.data = reinterpret_cast<void*>(static_cast<uintptr_t>(0x10000));
  b.bytes = static_cast<size_t>(bytes);
  b.id = 987654321u;
  static_cast<Shim*>(s)->bufs.push_back(b);
  *handle = static_cast<int>(static_cast<Shim*>(s)->bufs.size() - 1);
  return 0;
}

uint64_t shim_id(void* s, int h) { return B(s, h).id; }

int shim_free(void* s, int h) { return Guard([&] { D(s).Free(B(s, h)); }); }

int shim_h2d(void* s, int h, const void* src, int64_t bytes) {
  return Guard([&] { D(s).CopyHostToDevice(B(s, h), src, static_cast<size_t>(bytes)); });
}

int shim_d2h(void* s, void* dst, int h, int64_t bytes) {
  return Guard([&] { D(s).CopyDeviceToHost(dst, B(s, h), static_cast<size_t>(bytes)); });
}

int shim_matmul(void* s, int a, int b, int c, int64_t m, int64_t k, int64_t n) {
  return Guard([&] { D(s).MatMul(B(s, a), B(s, b), B(s, c), m, k, n); });
}

int shim_transpose(void* s, int src, int dst, int64_t rows, int64_t cols) {
  return Guard([&] { D(s).Transpose(B(s, src), B(s, dst), rows, cols); });
}

int shim_gemm_epilogue(void* s, int c, int64_t m, int64_t n, float alpha, int bias, const int64_t* shape, int nshape,
                       float beta, int act) {
  return Guard([&] {
    std::vector<int64_t> bs(shape, shape + nshape);
    const accel::DeviceBuffer* bp = bias >= 0 ? &B(s, bias) : nullptr;
    D(s).GemmEpilogue(B(s, c), m, n, alpha, bp, bs, beta, static_cast<accel::Activation>(act));
  });
}

int shim_embedding(void* s, int ids, int64_t id_offset, int table, int out, int64_t seq, int64_t hidden,
                   int64_t vocab) {
  return Guard([&] { D(s).Embedding(B(s, ids), id_offset, B(s, table), B(s, out), seq, hidden, vocab); });
}

int shim_rmsnorm(void* s, int x, int w, int y, int64_t rows, int64_t dim, float eps, int64_t row_offset) {
  return Guard([&] { D(s).RmsNorm(B(s, x), B(s, w), B(s, y), rows, dim, eps, row_offset); });
}

int shim_rope(void* s, int states, int cos_t, int sin_t, int64_t seq, int64_t n_heads, int64_t head_dim,
              int64_t position) {
  return Guard([&] { D(s).Rope(B(s, states), B(s, cos_t), B(s, sin_t), seq, n_heads, head_dim, position); });
}

int shim_append_cache(void* s, int src, int cache, int64_t seq, int64_t position, int64_t n_heads,
                      int64_t head_dim) {
  return Guard([&] { D(s).AppendCache(B(s, src), B(s, cache), seq, position, n_heads, head_dim); });
}

int shim_attention(void* s, int q, int k, int v, int scores, int out, int64_t seq, int64_t position, int64_t heads,
                   int64_t kv_heads, int64_t head_dim) {
  return Guard([&] {
    D(s).Attention(B(s, q), B(s, k), B(s, v), B(s, scores), B(s, out), seq, position, heads, kv_heads, head_dim);
  });
}

int shim_silu_mul(void* s, int gate, int up, int64_t count) {
  return Guard([&] { D(s).SiluMul(B(s, gate), B(s, up), count); });
}

int shim_residual_add(void* s, int dest, int extra, int64_t count) {
  return Guard([&] { D(s).ResidualAdd(B(s, dest), B(s, extra), count); });
}

int shim_sample_token(void* s, int logits, int chosen, int64_t index, int64_t vocab, float temperature,
                      uint32_t* rng, int top_k) {
  return Guard([&] { D(s).SampleToken(B(s, logits), B(s, chosen), index, vocab, temperature, rng, top_k); });
}

// MatMulQ8 with a plane of device pointers taken from buffers (zero < 0: none).
int shim_matmul_q8(void* s, int a, int q, int scale, int zero, const int64_t* shape, int nshape, int64_t axis,
                   int64_t offset, int c, int64_t m, int64_t k, int64_t n) {
  return Guard([&] {
    accel::QuantPlane p;
    p.q = static_cast<const int8_t*>(B(s, q).data);
    p.scale = static_cast<const float*>(B(s, scale).data);
    p.zero = zero >= 0 ? static_cast<const int8_t*>(B(s, zero).data) : nullptr;
    p.shape.assign(shape, shape + nshape);
    p.axis = axis;
    p.offset = offset;
    D(s).MatMulQ8(B(s, a), p, B(s, c), m, k, n);
  });
}

}  // extern "C"
