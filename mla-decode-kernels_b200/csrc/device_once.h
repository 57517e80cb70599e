// Host-side "once per device" for kernel attribute setup.
//
// A kernel's dynamic shared memory limit (cudaFuncSetAttribute) belongs to
// the kernel as loaded on one device, so a process that launches on several
// devices must set it on each of them.  DeviceOnce runs its setup the first
// time it is asked on the current device and remembers only a success: a
// failed setup (for example during stream capture) is retried on the next
// call instead of failing every later launch.
#ifndef GQA_DEVICE_ONCE_H
#define GQA_DEVICE_ONCE_H

#include <cuda_runtime.h>

#include <atomic>
#include <mutex>

namespace gqa {

class DeviceOnce {
 public:
  static constexpr int kMaxDevices = 64;

  template <typename Setup>
  cudaError_t run(Setup&& setup) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    if (done_[dev].load(std::memory_order_acquire)) return cudaSuccess;
    std::lock_guard<std::mutex> lock(mu_);
    if (done_[dev].load(std::memory_order_relaxed)) return cudaSuccess;
    e = setup();
    if (e == cudaSuccess) done_[dev].store(true, std::memory_order_release);
    return e;
  }

 private:
  std::mutex mu_;
  std::atomic<bool> done_[kMaxDevices] = {};
};

}  // namespace gqa

#endif  // GQA_DEVICE_ONCE_H
