// Device-side types shared by the estimator and renderers (reference
// include/foundation_pose_nvidia/cuda_pipeline.hpp:21-41): the uploaded mesh
// (DeviceMesh, declared with the renderer seam) and the selected pose. The
// reference's free kernel wrappers (runDepthPreprocess, prepareNetworkInputs,
// ...) are replaced by the kernel-level C ABI in fpk.h.
#pragma once

#include "foundation_pose_nvidia/device_buffer.hpp"
#include "foundation_pose_nvidia/mesh.hpp"
#include "foundation_pose_nvidia/renderer.hpp"
#include "foundation_pose_nvidia/types.hpp"

#pragma GCC visibility push(default)
namespace foundation_pose_nvidia {

struct DevicePoseResult {
  Mat4f pose;
  float score = 0.0f;
  int index = -1;
};

}  // namespace foundation_pose_nvidia
#pragma GCC visibility pop
