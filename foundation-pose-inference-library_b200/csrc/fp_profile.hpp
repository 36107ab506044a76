// Stage timing and launch counting for benchmarks (internal). When enabled,
// every instrumented stage records a CUDA event pair on the stream it runs on
// and its algorithmic work (FLOPs or bytes); fpk_profile_read() resolves them.
#pragma once

#include <cuda_runtime.h>

namespace fpb {
namespace prof {

enum Kind { kGemm = 0, kRender = 1, kAttention = 2, kOther = 3, kPreprocess = 4, kKinds = 5 };

void countLaunch(int kind, int n = 1);
bool enabled();

// Records a start event at construction and an end event at destruction.
class Scope {
 public:
  Scope(int kind, double work, cudaStream_t s);
  ~Scope();
  Scope(const Scope&) = delete;
  Scope& operator=(const Scope&) = delete;

 private:
  int kind_;
  double work_;
  cudaStream_t s_;
  cudaEvent_t a_ = nullptr;
};

}  // namespace prof
}  // namespace fpb
