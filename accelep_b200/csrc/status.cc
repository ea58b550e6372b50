// Error and launch bookkeeping shared by every C entry point of the library.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <string>

#include "accel_b200.h"
#include "status.h"

namespace accel_b200 {
namespace {
thread_local std::string g_error;
std::atomic<int64_t> g_launches{0};
}  // namespace

int SetError(int code, const std::string& message) {
  g_error = message;
  return code;
}

int ClearError() {
  g_error.clear();
  return ACCEL_B200_OK;
}

void NoteLaunches(int64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

bool PdlEnabled() {
  static const bool on = [] {
    const char* v = std::getenv("ACCEL_B200_PDL");
    return v == nullptr || std::strcmp(v, "0") != 0;
  }();
  return on;
}

// Checks a launch made through cudaLaunchKernelEx (its return code) and the
// error state.
int CheckLaunchEx(cudaError_t err, const char* what) {
  if (err != cudaSuccess) {
    cudaGetLastError();
    return SetError(ACCEL_B200_ECUDA, std::string(what) + ": " + cudaGetErrorString(err));
  }
  return CheckLaunch(what);
}

int CheckLaunch(const char* what) {
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    return SetError(ACCEL_B200_ECUDA, std::string(what) + ": " + cudaGetErrorString(err));
  }
  NoteLaunches(1);
  return ACCEL_B200_OK;
}

}  // namespace accel_b200

extern "C" ACCEL_B200_API const char* accel_b200_last_error(void) { return accel_b200::g_error.c_str(); }

extern "C" ACCEL_B200_API int64_t accel_b200_launch_count(void) {
  return accel_b200::g_launches.load(std::memory_order_relaxed);
}
