// Inference seam (reference include/foundation_pose_nvidia/inference_runner.hpp:12-30).
// rendered / observed are NCHW [batch, 6, H, W] fp32 device tensors; outputs are
// [batch, 3] translation / axis-angle deltas (pre-tanh) and [batch] scores.
#pragma once

#include <cuda_runtime_api.h>

#pragma GCC visibility push(default)
namespace foundation_pose_nvidia {

class IInferenceRunner {
 public:
  virtual ~IInferenceRunner() = default;
  virtual void prepareForBatch(int batch_size) { (void)batch_size; }
  virtual void enqueueRefine(const float* rendered, const float* observed, float* delta_translation,
                             float* delta_rotation, int batch_size, cudaStream_t stream) = 0;
  virtual void enqueueScore(const float* rendered, const float* observed, float* scores,
                            int batch_size, cudaStream_t stream) = 0;
};

}  // namespace foundation_pose_nvidia
#pragma GCC visibility pop
