// Estimator (reference include/foundation_pose_nvidia/foundation_pose.hpp:24-66):
// register / track on one object, with injectable renderer and inference
// backends. With the built-in backends the render, crop-warp and pack run as
// one fused kernel writing the networks' input layout directly; injected
// backends go through the NCHW fp32 seam exactly as in the reference.
#pragma once

#include <cstdint>
#include <filesystem>
#include <memory>
#include <span>

#include "foundation_pose_nvidia/config.hpp"
#include "foundation_pose_nvidia/inference_runner.hpp"
#include "foundation_pose_nvidia/mesh.hpp"
#include "foundation_pose_nvidia/renderer.hpp"
#include "foundation_pose_nvidia/types.hpp"

#pragma GCC visibility push(default)
namespace foundation_pose_nvidia {

class FoundationPose {
 public:
  FoundationPose(PreprocessedMesh mesh, RuntimeOptions runtime_options, Config config = {});
  FoundationPose(PreprocessedMesh mesh, RuntimeOptions runtime_options,
                 std::unique_ptr<IInferenceRunner> inference_runner,
                 std::unique_ptr<IRenderer> renderer, Config config = {});
  ~FoundationPose();
  FoundationPose(const FoundationPose&) = delete;
  FoundationPose& operator=(const FoundationPose&) = delete;
  FoundationPose(FoundationPose&&) noexcept;
  FoundationPose& operator=(FoundationPose&&) noexcept;

  static FoundationPose createFromCadFile(const std::filesystem::path& cad_path,
                                          RuntimeOptions runtime_options, Config config = {});
  static FoundationPose createFromReferenceImages(std::span<const ModelFreeReferenceView> references,
                                                  RuntimeOptions runtime_options,
                                                  Config config = {});

  void prepareForBatch(int batch_size);

  PoseEstimate registerFrame(const std::uint8_t* rgb_u8, const float* depth_m,
                             const std::uint8_t* mask_u8, int width, int height,
                             CameraIntrinsics intrinsics, int n_refine = -1, int n_hypotheses = -1);

  PoseEstimate trackFrame(const std::uint8_t* rgb_u8, const float* depth_m, int width, int height,
                          CameraIntrinsics intrinsics, int n_refine = -1);

  // Register split across estimators on several GPUs (no counterpart in the
  // reference; the multi-GPU form of registerFrame). Every shard takes the
  // same frame and hypothesis count and refines its contiguous range
  // [shard_begin, shard_begin + shard_count) of the seeded hypotheses, then
  // writes, into device memory of this estimator's GPU, its ScoreNet features
  // (shard_count x kScoreFeatureDim floats) and refined object-centred poses
  // (shard_count x 16 floats, row-major). Requires the built-in renderer and
  // networks. Returns after the outputs are complete.
  static constexpr int kScoreFeatureDim = 512;
  void registerShardBegin(const std::uint8_t* rgb_u8, const float* depth_m, const std::uint8_t* mask_u8,
                          int width, int height, CameraIntrinsics intrinsics, int n_refine,
                          int n_hypotheses, int shard_begin, int shard_count, float* features,
                          float* poses);
  // Cross-hypothesis ScoreNet head and arg-max over all n_hypotheses shards'
  // outputs, concatenated in hypothesis order (device memory on this GPU).
  // The result (and the pose track continues from) equals registerFrame's.
  PoseEstimate registerShardFinish(const float* features, const float* poses, int n_hypotheses);

  const PreprocessedMesh& mesh() const;
  const Config& config() const;

  struct Impl;

 private:
  std::unique_ptr<Impl> impl_;
};

}  // namespace foundation_pose_nvidia
#pragma GCC visibility pop
