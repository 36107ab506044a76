// Renderer seam (reference include/foundation_pose_nvidia/renderer.hpp:15-34 and the
// DeviceMesh of cuda_pipeline.hpp:21-35). A renderer draws every hypothesis pose
// of the centred mesh into its crop box and writes NHWC float3 RGB in [0,1] and
// camera-space XYZ in metres (background: zeros), stream-ordered, without
// owning the mesh.
#pragma once

#include <cuda_runtime_api.h>
#include <vector_types.h>

#include "foundation_pose_nvidia/device_buffer.hpp"
#include "foundation_pose_nvidia/types.hpp"

#pragma GCC visibility push(default)
namespace foundation_pose_nvidia {

struct DeviceMesh {
  int num_vertices = 0;
  int num_faces = 0;
  int texture_width = 0;
  int texture_height = 0;
  bool has_texture = false;
  bool has_uvs = false;
  DeviceBuffer vertices;     // float3[num_vertices], centred mesh frame
  DeviceBuffer normals;      // float3[num_vertices]
  DeviceBuffer uvs;          // float2[num_vertices], optional
  DeviceBuffer colors;       // float3[num_vertices], [0, 1]
  DeviceBuffer faces;        // int3[num_faces]
  DeviceBuffer texture_rgb;  // float3[texture_width * texture_height], optional
};

class IRenderer {
 public:
  virtual ~IRenderer() = default;
  virtual void reserveForMesh(int num_vertices, int num_faces) {
    (void)num_vertices;
    (void)num_faces;
  }
  virtual void render(const DeviceMesh& mesh, const float* poses, const float* crop_boxes,
                      int batch_size, CameraIntrinsics intrinsics, int image_width,
                      int image_height, float3* out_rgb, float3* out_xyz, cudaStream_t stream) = 0;
};

}  // namespace foundation_pose_nvidia
#pragma GCC visibility pop
