// Allocation-free variant of the frame preprocessing + initial-translation
// chain (fpk_initial_translation_noalloc, declared in include/fpk.h).
//
// Who needs it: some callers may not allocate device memory at all once they
// are running -- real-time control loops and safety-reviewed deployments that
// freeze their memory footprint at start-up, and plugin hosts (perception graph
// nodes, inference servers) that hand every buffer to a library from their own
// arena. They can pass in the frame and receive the translation, but cannot let
// this library cudaMalloc the scratch the chain needs. Here that scratch (the
// filtered depth map and the 65,536-bin depth histogram) lives in fixed-size
// device arrays of this library's module, on every GPU that uses it:
// MaxPixels * 4 bytes + 65,544 * 4 bytes, about 3.8 MiB, held until exit.
//
// Host code cannot use the arrays' names as device addresses (in host code the
// name is a host-side stand-in), so the first call on each device looks the
// addresses up with cudaGetSymbolAddress while that device is current and
// caches them. With CUDA's default lazy module loading, that first lookup is
// also when the driver loads the module on the device and sets the arrays'
// memory aside, so the first call on each device is the one that may take
// device memory: make one warm-up call per device at start-up, before the
// footprint is frozen and before any stream capture (or run with
// CUDA_MODULE_LOADING=EAGER, which reserves the arrays when the library's
// module is loaded).
// Every call reuses the same arrays: the histogram is cleared at the start of
// each call, and calls that overlap on the GPU (different streams, or several
// host threads on one device) race on the arrays and must be serialised by
// the caller.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>

#include "fpk.h"

namespace fpb {
int fail(const std::string& msg);
}

// The scratch: filtered depth (one frame) and the translation statistics.
static __device__ __align__(256) float g_noalloc_depth[FPK_NOALLOC_MAX_PIXELS];
static __device__ __align__(256) int32_t g_noalloc_stats[FPK_STATS_INTS];

namespace {

constexpr int kNoAllocMaxPixels = FPK_NOALLOC_MAX_PIXELS;
constexpr int kMaxDevices = 64;

struct Scratch {
  float* depth = nullptr;
  int32_t* stats = nullptr;
};

std::mutex g_mu;
Scratch g_scratch[kMaxDevices];

// Device addresses of the scratch arrays for the current device (looked up once).
int scratchForCurrentDevice(Scratch* out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fpb::fail(std::string("fpk noalloc: cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fpb::fail("fpk noalloc: device index out of range");
  std::lock_guard<std::mutex> lock(g_mu);
  Scratch& s = g_scratch[dev];
  if (s.depth == nullptr || s.stats == nullptr) {
    void* d = nullptr;
    void* st = nullptr;
    e = cudaGetSymbolAddress(&d, g_noalloc_depth);
    if (e != cudaSuccess) {
      return fpb::fail(std::string("fpk noalloc: cudaGetSymbolAddress(depth): ") + cudaGetErrorString(e));
    }
    e = cudaGetSymbolAddress(&st, g_noalloc_stats);
    if (e != cudaSuccess) {
      return fpb::fail(std::string("fpk noalloc: cudaGetSymbolAddress(stats): ") + cudaGetErrorString(e));
    }
    s.depth = static_cast<float*>(d);
    s.stats = static_cast<int32_t*>(st);
  }
  *out = s;
  return 0;
}

}  // namespace

extern "C" int fpk_initial_translation_noalloc(const float* depth_raw, const uint8_t* mask, int width,
                                               int height, fpk_intrinsics_t k, const fpk_params_t* p,
                                               float* t0, void* stream) {
  if (depth_raw == nullptr || mask == nullptr || t0 == nullptr) {
    return fpb::fail("fpk_initial_translation_noalloc: depth, mask and t0 are required");
  }
  if (width <= 0 || height <= 0) {
    return fpb::fail("fpk_initial_translation_noalloc: image dimensions must be positive");
  }
  if (static_cast<long long>(width) * height > kNoAllocMaxPixels) {
    return fpb::fail("fpk_initial_translation_noalloc: frame of " + std::to_string(width) + "x" +
                     std::to_string(height) + " exceeds the built-in scratch of " +
                     std::to_string(kNoAllocMaxPixels) + " pixels (1280x720)");
  }
  Scratch s;
  if (scratchForCurrentDevice(&s) != 0) return 1;
  // fpk_preprocess clears the histogram (a memset, no allocation) and runs the
  // fused erode/bilateral/statistics pass; fpk_seed_poses with no rotations
  // only reduces the histogram to the translation.
  if (fpk_preprocess(depth_raw, mask, width, height, k, p, s.depth, nullptr, nullptr, s.stats, stream) != 0) {
    return 1;
  }
  return fpk_seed_poses(s.stats, nullptr, 0, k, p, t0, nullptr, stream);
}
