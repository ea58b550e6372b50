// The one-matmul C API of AccelEP (include/accel/sim_api.h:15-37 of the
// reference) served straight from the kernel ABI.
//
// A Sim owns a CUDA stream on the device that was current when it was made
// and one device staging area that holds a call's left operand and result
// back to back; the area grows when a call needs more and is reused
// otherwise, so a steady stream of products allocates nothing. An uploaded
// matrix is a device allocation of its own. A product copies `a` in, runs the
// bit-exact MatMul kernel (accel_b200_matmul: src/sim_device.cc:185-196
// through PackedMatMul, :331-369) and copies `c` out on the Sim's stream,
// then waits for that stream alone. The process-wide counters move as the
// reference's do: one kernel matmul per product, plus the bytes that crossed
// the host boundary.
#include <cuda_runtime.h>

#include <cstdint>
#include <limits>
#include <mutex>
#include <new>
#include <stdexcept>
#include <string>

#include "accel_b200.h"
#include "accel_b200_llama.h"
#include "stats.h"

namespace {

thread_local std::string t_sim_error;

// A CUDA failure as an exception carrying the runtime's message.
void OrThrow(cudaError_t err, const char* what) {
  if (err == cudaSuccess) return;
  cudaGetLastError();
  if (err == cudaErrorMemoryAllocation) throw std::bad_alloc();
  throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(err));
}

// Bytes of `count` floats, or an overflow error (the reference's
// CheckedBytes, src/sim_device.cc:44-60, rejects the same sizes).
size_t FloatBytes(int64_t count) {
  if (count < 0 || static_cast<uint64_t>(count) > std::numeric_limits<size_t>::max() / sizeof(float)) {
    throw std::overflow_error("buffer size overflows");
  }
  return static_cast<size_t>(count) * sizeof(float);
}

size_t ProductBytes(int64_t rows, int64_t cols) {
  if (rows != 0 && cols > std::numeric_limits<int64_t>::max() / rows) throw std::overflow_error("buffer size overflows");
  return FloatBytes(rows * cols);
}

// Runs `body` as one API call: the thread's error text is cleared on
// success and set from the exception otherwise.
template <typename F>
bool Call(F&& body) {
  try {
    body();
    t_sim_error.clear();
    return true;
  } catch (const std::exception& ex) {
    t_sim_error = ex.what();
    return false;
  }
}

}  // namespace

struct AccelBuf {
  float* data = nullptr;
  int64_t count = 0;
};

struct AccelSim {
  int ordinal = 0;
  cudaStream_t stream = nullptr;
  void* staging = nullptr;  // a's floats, then c's
  size_t staging_bytes = 0;
  std::mutex mu;

  AccelSim() {
    OrThrow(cudaGetDevice(&ordinal), "current device");
    OrThrow(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "stream");
  }
  ~AccelSim() {
    Scope scope(ordinal);
    cudaStreamSynchronize(stream);
    if (staging != nullptr) cudaFree(staging);
    cudaStreamDestroy(stream);
  }

  // Makes the Sim's device current for one call and restores the caller's.
  struct Scope {
    int previous = 0;
    explicit Scope(int ordinal) {
      cudaGetDevice(&previous);
      if (previous != ordinal) cudaSetDevice(ordinal);
    }
    ~Scope() { cudaSetDevice(previous); }
  };

  void* Staging(size_t bytes) {
    if (bytes <= staging_bytes) return staging;
    if (staging != nullptr) {
      OrThrow(cudaStreamSynchronize(stream), "staging");
      cudaFree(staging);
      staging = nullptr;
      staging_bytes = 0;
    }
    OrThrow(cudaMalloc(&staging, bytes), "staging");
    staging_bytes = bytes;
    return staging;
  }
};

extern "C" {

ACCEL_B200_API AccelSim* accel_sim_create(void) {
  AccelSim* sim = nullptr;
  Call([&] {
    int devices = 0;
    if (cudaGetDeviceCount(&devices) != cudaSuccess || devices == 0) {
      cudaGetLastError();
      throw std::runtime_error("no CUDA device is available for the B200 backend");
    }
    sim = new AccelSim();
  });
  return sim;
}

ACCEL_B200_API void accel_sim_destroy(AccelSim* sim) { delete sim; }

ACCEL_B200_API AccelBuf* accel_sim_upload(AccelSim* sim, const float* data, int64_t count) {
  if (sim == nullptr || count < 0 || (count > 0 && data == nullptr)) {
    t_sim_error = "invalid upload";
    return nullptr;
  }
  AccelBuf* buf = nullptr;
  Call([&] {
    std::lock_guard<std::mutex> lock(sim->mu);
    AccelSim::Scope scope(sim->ordinal);
    const size_t bytes = FloatBytes(count);
    float* dev = nullptr;
    OrThrow(cudaMalloc(&dev, bytes == 0 ? 1 : bytes), "upload");
    const cudaError_t err = bytes == 0 ? cudaSuccess : cudaMemcpy(dev, data, bytes, cudaMemcpyHostToDevice);
    if (err != cudaSuccess) cudaFree(dev);
    OrThrow(err, "upload");
    accel_b200::NoteBytesToDevice(bytes);
    buf = new AccelBuf{dev, count};
  });
  return buf;
}

ACCEL_B200_API void accel_sim_release(AccelSim* sim, AccelBuf* buf) {
  if (sim == nullptr || buf == nullptr) return;
  std::lock_guard<std::mutex> lock(sim->mu);
  AccelSim::Scope scope(sim->ordinal);
  cudaStreamSynchronize(sim->stream);  // a product may still read it
  cudaFree(buf->data);
  delete buf;
}

ACCEL_B200_API int accel_sim_matmul(AccelSim* sim, const float* a, int64_t m, int64_t k, AccelBuf* b, int64_t n,
                                    float* c) {
  if (sim == nullptr || b == nullptr || m < 0 || k < 0 || n < 0 || (m > 0 && k > 0 && a == nullptr) ||
      (m > 0 && n > 0 && c == nullptr)) {
    t_sim_error = "invalid matmul";
    return 1;
  }
  const bool ok = Call([&] {
    std::lock_guard<std::mutex> lock(sim->mu);
    const size_t a_bytes = ProductBytes(m, k);
    const size_t c_bytes = ProductBytes(m, n);
    // src/sim_device.cc RequireBytes: the uploaded matrix must hold k * n.
    if (ProductBytes(k, n) > FloatBytes(b->count)) throw std::invalid_argument("MatMul B is out of range");
    AccelSim::Scope scope(sim->ordinal);
    // a's floats, then c's, at a 256-byte boundary.
    const size_t c_off = (a_bytes + 255) / 256 * 256;
    char* area = static_cast<char*>(sim->Staging(c_off + c_bytes + 1));
    float* dev_a = reinterpret_cast<float*>(area);
    float* dev_c = reinterpret_cast<float*>(area + c_off);
    if (a_bytes > 0) {
      OrThrow(cudaMemcpyAsync(dev_a, a, a_bytes, cudaMemcpyHostToDevice, sim->stream), "host-to-device copy");
      accel_b200::NoteBytesToDevice(a_bytes);
    }
    if (accel_b200_matmul(dev_a, b->data, dev_c, m, k, n, sim->stream) != ACCEL_B200_OK) {
      throw std::invalid_argument(accel_b200_last_error());
    }
    accel_b200::NoteKernelMatmuls(1);
    if (c_bytes > 0) {
      OrThrow(cudaMemcpyAsync(c, dev_c, c_bytes, cudaMemcpyDeviceToHost, sim->stream), "device-to-host copy");
    }
    OrThrow(cudaStreamSynchronize(sim->stream), "matmul");
    accel_b200::NoteBytesToHost(c_bytes);
  });
  return ok ? 0 : 1;
}

ACCEL_B200_API void accel_sim_reset_stats(void) { accel_b200::ResetCounters(); }
ACCEL_B200_API int64_t accel_sim_matmuls(void) { return accel_b200::GetCounters().kernel_matmuls; }
ACCEL_B200_API int64_t accel_sim_bytes_to_device(void) { return accel_b200::GetCounters().bytes_to_device; }
ACCEL_B200_API int64_t accel_sim_bytes_to_host(void) { return accel_b200::GetCounters().bytes_to_host; }
ACCEL_B200_API const char* accel_sim_last_error(void) { return t_sim_error.c_str(); }

}  // extern "C"
