#include "stats.h"

#include <atomic>

namespace accel_b200 {
namespace {
std::atomic<int64_t> g_matmuls{0};
std::atomic<int64_t> g_to_device{0};
std::atomic<int64_t> g_to_host{0};
}  // namespace

void ResetCounters() {
  g_matmuls.store(0);
  g_to_device.store(0);
  g_to_host.store(0);
}

Counters GetCounters() { return Counters{g_matmuls.load(), g_to_device.load(), g_to_host.load()}; }

void NoteKernelMatmuls(int64_t n) { g_matmuls.fetch_add(n); }
void NoteBytesToDevice(size_t bytes) { g_to_device.fetch_add(static_cast<int64_t>(bytes)); }
void NoteBytesToHost(size_t bytes) { g_to_host.fetch_add(static_cast<int64_t>(bytes)); }

}  // namespace accel_b200
