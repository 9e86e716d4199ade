// Host helpers shared by the extern "C" entry points: run a call on the device
// that owns its tensors, and set a kernel attribute once per device.
#pragma once

#include <cuda_runtime.h>

#include <atomic>

namespace osor {

// Makes the device that owns `ptr` current for the guard's lifetime (so callers
// need not set it) and restores the previous device afterwards. Host or
// unregistered pointers leave the current device alone.
class DeviceOf {
 public:
  explicit DeviceOf(const void* ptr) {
    cudaGetDevice(&prev_);
    cudaPointerAttributes attr;
    if (ptr && cudaPointerGetAttributes(&attr, ptr) == cudaSuccess &&
        attr.type == cudaMemoryTypeDevice && attr.device != prev_) {
      cudaSetDevice(attr.device);
      switched_ = true;
    }
    cudaGetLastError();
  }
  ~DeviceOf() {
    if (switched_) cudaSetDevice(prev_);
  }
  DeviceOf(const DeviceOf&) = delete;
  DeviceOf& operator=(const DeviceOf&) = delete;

 private:
  int prev_ = 0;
  bool switched_ = false;
};

constexpr int kMaxDevices = 64;

// Per-device "done" flags for one-time set-up such as cudaFuncSetAttribute.
// Atomic so that host threads calling the same entry point concurrently do not
// race on them; two threads may both run the (idempotent) set-up once.
struct PerDeviceOnce {
  std::atomic<bool> done[kMaxDevices] = {};

  // Runs `setup()` (returning cudaError_t) on the current device unless it
  // already succeeded there.
  template <typename F>
  cudaError_t run(F setup) {
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return e;
    if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
    if (done[device].load(std::memory_order_acquire)) return cudaSuccess;
    e = setup();
    if (e == cudaSuccess) done[device].store(true, std::memory_order_release);
    return e;
  }
};

}  // namespace osor
