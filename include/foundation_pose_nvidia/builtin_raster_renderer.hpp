// The built-in renderer behind the IRenderer seam (reference
// include/foundation_pose_nvidia/builtin_raster_renderer.hpp): the sm_100a
// rasterizer of this library (vertex pass, one thread per (hypothesis,
// triangle) into an L2-resident 64-bit z-buffer, per-pixel resolve and shading).
// An estimator given this renderer together with the built-in networks
// (TensorRtRunner) runs render, crop-warp and pack as one fused pass; with any
// other runner it renders through the NCHW fp32 seam.
#pragma once

#include <memory>

#include <cuda_runtime_api.h>

#include "foundation_pose_nvidia/config.hpp"
#include "foundation_pose_nvidia/cuda_pipeline.hpp"
#include "foundation_pose_nvidia/device_buffer.hpp"
#include "foundation_pose_nvidia/renderer.hpp"
#include "foundation_pose_nvidia/types.hpp"

#pragma GCC visibility push(default)
namespace foundation_pose_nvidia {

class BuiltinRasterRenderer final : public IRenderer {
 public:
  BuiltinRasterRenderer(const Config& config, int device_id, int max_batch);
  ~BuiltinRasterRenderer() override;
  BuiltinRasterRenderer(const BuiltinRasterRenderer&) = delete;
  BuiltinRasterRenderer& operator=(const BuiltinRasterRenderer&) = delete;

  void reserveForMesh(int num_vertices, int num_faces) override;
  void render(const DeviceMesh& mesh, const float* poses, const float* crop_boxes, int batch_size,
              CameraIntrinsics intrinsics, int image_width, int image_height, float3* out_rgb,
              float3* out_xyz, cudaStream_t stream) override;

  struct Impl;

 private:
  std::unique_ptr<Impl> impl_;
};

}  // namespace foundation_pose_nvidia
#pragma GCC visibility pop
