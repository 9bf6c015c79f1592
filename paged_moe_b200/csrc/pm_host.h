// pm_host.h -- host-side helpers shared by the library's translation units:
// the thread's last CUDA error, the current device, per-device one-time
// setup and the SM count.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <mutex>

#include "../../include/pm_sample.h"

namespace pmh {

constexpr int kMaxDevices = 64;

// The last CUDA error seen by this thread (pm_last_cuda_error).
inline int& last_cuda() {
  static thread_local int v = 0;
  return v;
}

inline int cuda_fail(cudaError_t e) {
  last_cuda() = (int)e;
  return PM_ERR_CUDA;
}

inline int current_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess) {
    cudaGetLastError();
    d = 0;
  }
  return d;
}

// One-time setup per device: kernel attributes (the dynamic shared memory
// limit) and occupancy queries belong to the device that is current, so a
// process that drives several GPUs repeats them on each.
class DeviceOnce {
 public:
  template <class F>
  void operator()(F&& f) {
    const int d = current_device();
    if (d < 0 || d >= kMaxDevices) {
      f();
      return;
    }
    if (done_[d].load(std::memory_order_acquire)) return;
    std::lock_guard<std::mutex> g(mu_);
    if (!done_[d].load(std::memory_order_relaxed)) {
      f();
      done_[d].store(true, std::memory_order_release);
    }
  }

 private:
  std::mutex mu_;
  std::atomic<bool> done_[kMaxDevices] = {};
};

// SMs of the current device (148 on B200 when the query fails).
inline int num_sms() {
  static int sms[kMaxDevices] = {};
  static DeviceOnce once;
  const int d = current_device();
  int* slot = (d >= 0 && d < kMaxDevices) ? &sms[d] : nullptr;
  int local = 0;
  once([&] {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, d) != cudaSuccess || v <= 0) {
      cudaGetLastError();
      v = 148;
    }
    if (slot) *slot = v;
    local = v;
  });
  return slot ? *slot : (local ? local : 148);
}

}  // namespace pmh

namespace pm {
struct SampleArgs;
}

// The masked gather pass (pm_masked.cu): rows with an allowed-token mask
// whose logits can be fetched as aligned 4-byte words.
int pm_launch_masked(int dtype, int KC, const pm::SampleArgs& a, cudaStream_t st);

// The processors' device lists (penalty overrides by tile, logit-bias tile
// offsets) for a pass of another translation unit (pm_lmhead.cu): bytes of
// the region (0: a history window beyond the build's cap), and the prep
// kernels that fill it and the processor fields of `a` (a.status must be set).
size_t pm_prep_bytes(const pm_rows* r, int n_tiles);
int pm_prep_launch(const pm_rows* r, int n_tiles, unsigned char* region, pm::SampleArgs& a, cudaStream_t st);

// The row merges (pm_sample.cu) over parts that a pass of another
// translation unit wrote (pm_lmhead.cu).
int pm_launch_merges(int KC, const pm::SampleArgs& a, cudaStream_t st);
