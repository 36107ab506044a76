// The built-in inference backend behind the IInferenceRunner seam, under the
// reference's class name (reference include/foundation_pose_nvidia/
// tensorrt_runner.hpp:20-56) so code that constructs it keeps compiling.
// Here it runs RefineNet / ScoreNet as this library's tcgen05 kernels from
// weight packs (RuntimeOptions::refine_model_path / score_model_path name
// .fpw files); TensorRT is not used. Precision follows
// Config::tensorrt_precision; the micro-batch is min(batch_size, max_batch)
// and must divide max_batch, as in the reference.
#pragma once

#include <memory>

#include <cuda_runtime_api.h>

#include "foundation_pose_nvidia/config.hpp"
#include "foundation_pose_nvidia/device_buffer.hpp"
#include "foundation_pose_nvidia/inference_runner.hpp"

#pragma GCC visibility push(default)
namespace foundation_pose_nvidia {

class TensorRtRunner final : public IInferenceRunner {
 public:
  TensorRtRunner(RuntimeOptions options, Config config, int max_batch);
  ~TensorRtRunner() override;
  TensorRtRunner(const TensorRtRunner&) = delete;
  TensorRtRunner& operator=(const TensorRtRunner&) = delete;

  void prepareForBatch(int batch_size) override;
  void enqueueRefine(const float* rendered, const float* observed, float* delta_translation,
                     float* delta_rotation, int batch_size, cudaStream_t stream) override;
  void enqueueScore(const float* rendered, const float* observed, float* scores, int batch_size,
                    cudaStream_t stream) override;

  struct Impl;
  Impl& impl() { return *impl_; }

 private:
  std::unique_ptr<Impl> impl_;
};

}  // namespace foundation_pose_nvidia
#pragma GCC visibility pop
