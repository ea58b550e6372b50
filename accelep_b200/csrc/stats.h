// Process-wide counters the AccelEP API reports (include/accel/runtime.h:11-33
// of the reference: kernel matmuls and bytes across the host boundary).
#pragma once

#include <cstddef>
#include <cstdint>

namespace accel_b200 {

struct Counters {
  int64_t kernel_matmuls;
  int64_t bytes_to_device;
  int64_t bytes_to_host;
};

void ResetCounters();
Counters GetCounters();
void NoteKernelMatmuls(int64_t n);
void NoteBytesToDevice(size_t bytes);
void NoteBytesToHost(size_t bytes);

}  // namespace accel_b200
