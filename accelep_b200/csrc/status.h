// Host-side error and launch bookkeeping of the kernel ABI (status.cc).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>

namespace accel_b200 {

// Records a failure for accel_b200_last_error() and returns its code.
int SetError(int code, const std::string& message);
int ClearError();
// Adds n to the process-wide launch count (accel_b200_launch_count).
void NoteLaunches(int64_t n);
// Checks the launch just issued; returns ACCEL_B200_OK or ACCEL_B200_ECUDA.
int CheckLaunch(const char* what);
// The same for a launch whose cudaLaunchKernelEx returned `err`.
int CheckLaunchEx(cudaError_t err, const char* what);

}  // namespace accel_b200
