// Kernel launches with programmatic dependent launch (PDL).
//
// A kernel launched through launchPdl may begin while the previous kernel in
// the stream is still finishing: every such kernel calls tc::pdlTrigger() on
// entry (its dependents may be scheduled once all of its CTAs have started)
// and tc::pdlWait() before its first access to memory an earlier kernel
// writes or reads (griddepcontrol.wait returns once the previous grid has
// completed and its writes are visible). The prologue before the wait
// (barrier init, TMEM allocation, shared-memory tables) then overlaps the
// previous kernel's tail, and the launch latency between dependent kernels
// is hidden. Kernels launched without the attribute are unaffected by both
// calls.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <utility>

namespace fpb {

// Per-device state of the launch helpers. The group API runs one host thread
// per GPU, so kernel attributes and device properties are kept per device
// index (a node may mix parts or MIG slices). Devices past the table are
// served uncached: the setup simply runs on every call.
constexpr int kMaxDevices = 64;

inline int currentDevice() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

// A non-zero int computed once per device by f(device).
struct DeviceValue {
  std::atomic<int> v[kMaxDevices] = {};
  template <class F>
  int get(F&& f) {
    const int dev = currentDevice();
    if (dev < 0 || dev >= kMaxDevices) return f(dev);
    int x = v[dev].load(std::memory_order_acquire);
    if (x == 0) {
      x = f(dev);  // a racing thread computes the same value
      v[dev].store(x, std::memory_order_release);
    }
    return x;
  }
};

// A setup step (returning cudaError_t) that must succeed once per device, such
// as raising a kernel's dynamic shared-memory limit. A failure is returned and
// not recorded, so the next call retries.
struct DeviceOnce {
  std::atomic<bool> done[kMaxDevices] = {};
  template <class F>
  cudaError_t run(F&& setup) {
    const int dev = currentDevice();
    const bool cached = dev >= 0 && dev < kMaxDevices;
    if (cached && done[dev].load(std::memory_order_acquire)) return cudaSuccess;
    const cudaError_t e = setup();
    if (e == cudaSuccess && cached) done[dev].store(true, std::memory_order_release);
    return e;
  }
};

template <typename... KArgs, typename... Args>
cudaError_t launchPdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                      Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace fpb
