// accel_b200_device.h: the B200 implementation of AccelEP's accel::Device.
//
// B200Device keeps its heap in HBM of one CUDA device and runs every device
// call as a kernel on one stream. Results of Device calls are complete when
// CopyDeviceToHost returns (it synchronizes the stream), which is the only
// point where the reference's callers read data back
// (src/runtime.cc:171-180, src/sim_api.cc:98).
//
// The accel::Device contract itself is declared by the host project in
// accel/device.h (include/accel/device.h:24-125 of the reference). Builds of
// this library on its own use the mirror in accel_b200_contract.h, which
// declares the same types and virtual functions; a host project builds
// src/b200_device.cc with -DACCEL_B200_USE_HOST_CONTRACT and its own header,
// which needs the one added virtual MatMulQ8.
#pragma once

#include <cstdint>
#include <memory>

#ifdef ACCEL_B200_USE_HOST_CONTRACT
#include "accel/device.h"
#include "accel/runtime.h"
#else
#include "accel_b200_contract.h"
#endif

#if defined(__GNUC__)
#define ACCEL_B200_CXX_API __attribute__((visibility("default")))
#else
#define ACCEL_B200_CXX_API
#endif

namespace accel_b200 {

// Creates a device on CUDA ordinal `ordinal` (-1: the current device).
// Throws std::runtime_error when no CUDA device is usable.
ACCEL_B200_CXX_API std::unique_ptr<accel::Device> CreateB200Device(int ordinal = -1);

// Process-wide count of B200Device allocations not yet freed.
ACCEL_B200_CXX_API int64_t LiveB200Allocs();

}  // namespace accel_b200
