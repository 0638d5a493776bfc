// launch_state.h -- per-device, thread-safe launcher state.
//
// cudaFuncSetAttribute and device attributes apply to one device, and a
// drop-in host may drive several GPUs from several host threads in one
// process (one thread per GPU).  So every launcher keeps what it has set up
// per device, and the set-up itself runs under a mutex: a second device
// gets its own opt-in, and two threads never race on the record.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>
#include <mutex>

namespace ctts {

constexpr int kMaxDevices = 64;

inline int current_device() {
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess) {
    (void)cudaGetLastError();
    return -1;
  }
  return d;
}

// Largest dynamic shared memory one kernel has been opted in to, per device.
// ensure() raises the opt-in when a launch needs more than recorded (and, for
// kernels launched on clusters of more than 8 CTAs, allows the non-portable
// cluster size once).  One instance per kernel (a function-local static at
// the launch site).
class SmemOptIn {
 public:
  cudaError_t ensure(const void* fn, size_t smem, bool nonportable_cluster = false) {
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    if (smem <= done_[dev].load(std::memory_order_acquire)) return cudaSuccess;
    std::lock_guard<std::mutex> lk(mu_);
    if (smem <= done_[dev].load(std::memory_order_relaxed)) return cudaSuccess;
    cudaError_t e = cudaSuccess;
    if (nonportable_cluster) e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      return e;
    }
    done_[dev].store(smem, std::memory_order_release);
    return cudaSuccess;
  }

 private:
  std::mutex mu_;
  std::atomic<size_t> done_[kMaxDevices] = {};
};

// One integer device attribute, read once per device (value + 1 stored, so
// 0 means "not read yet"; a racing second read stores the same value).
class DeviceAttrCache {
 public:
  explicit DeviceAttrCache(cudaDeviceAttr a) : attr_(a) {}
  int get() {
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) return 0;
    int v = val_[dev].load(std::memory_order_acquire);
    if (v) return v - 1;
    int x = 0;
    if (cudaDeviceGetAttribute(&x, attr_, dev) != cudaSuccess) {
      (void)cudaGetLastError();
      return 0;
    }
    val_[dev].store(x + 1, std::memory_order_release);
    return x;
  }

 private:
  cudaDeviceAttr attr_;
  std::atomic<int> val_[kMaxDevices] = {};
};

// An integer computed once per device by the caller's function (an
// occupancy figure, for instance) and cached; concurrent first calls may
// both compute it, with the same result.
class PerDeviceInt {
 public:
  template <class F>
  int get(F&& fn) {
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) return fn();
    int v = val_[dev].load(std::memory_order_acquire);
    if (v) return v - 1;
    const int x = fn();
    val_[dev].store(x + 1, std::memory_order_release);
    return x;
  }

 private:
  std::atomic<int> val_[kMaxDevices] = {};
};

// SM count of the current device (cached per device).
inline int device_sms() {
  static DeviceAttrCache c(cudaDevAttrMultiProcessorCount);
  return c.get();
}
// Whether the current device supports cooperative launches.
inline bool device_coop() {
  static DeviceAttrCache c(cudaDevAttrCooperativeLaunch);
  return c.get() != 0;
}

}  // namespace ctts
