// Test renderer plugin for the FP_RENDERER loader (the runtime's counterpart of
// reference src/foundation_pose.cpp:40-68, whose real plugin is
// src/nvdiffrast_renderer.cu:180-187). Built by tests/test_renderer_plugin.py
// as a shared object with soname libfoundation_pose_nvdiffrast.so.
//
// The renderer draws through fpk_render of the main library, so the estimator
// runs its unfused IRenderer path (NHWC fp32 render -> NCHW pack -> networks)
// with the built-in rasterizer's exact images. Compile-time variants exercise
// the loader's error paths:
//   FP_TEST_PLUGIN_NO_FACTORY    exports no fp_plugin_create_renderer
//   FP_TEST_PLUGIN_NULL_FACTORY  the factory returns NULL
#include <atomic>
#include <string>

#include "foundation_pose_nvidia/config.hpp"
#include "foundation_pose_nvidia/renderer.hpp"
#include "fpk.h"

namespace {

std::atomic<int> g_render_calls{0};
std::atomic<int> g_created{0};
int g_device_id = -1;
int g_max_batch = -1;

using namespace foundation_pose_nvidia;

class PluginRenderer final : public IRenderer {
 public:
  explicit PluginRenderer(const Config& c) {
    fpk_default_params(&params_);
    params_.input_width = c.input_width;
    params_.input_height = c.input_height;
    params_.znear = c.znear;
    params_.zfar = c.zfar;
    params_.ambient_weight = c.ambient_weight;
    params_.diffuse_weight = c.diffuse_weight;
  }

  void render(const DeviceMesh& mesh, const float* poses, const float* crop_boxes, int batch_size,
              CameraIntrinsics k, int, int, float3* out_rgb, float3* out_xyz, cudaStream_t stream) override {
    fpk_mesh_t m{};
    m.vertices = mesh.vertices.as<float>();
    m.normals = mesh.normals.as<float>();
    m.colors = mesh.colors.as<float>();
    const bool tex = mesh.has_texture && mesh.has_uvs;
    m.uvs = tex ? mesh.uvs.as<float>() : nullptr;
    m.texture = tex ? mesh.texture_rgb.as<float>() : nullptr;
    m.faces = mesh.faces.as<int32_t>();
    m.n_vertices = mesh.num_vertices;
    m.n_faces = mesh.num_faces;
    m.texture_width = tex ? mesh.texture_width : 0;
    m.texture_height = tex ? mesh.texture_height : 0;
    const fpk_intrinsics_t kk{k.fx, k.fy, k.cx, k.cy};
    if (fpk_render(&m, poses, crop_boxes, batch_size, kk, &params_, reinterpret_cast<float*>(out_rgb),
                   reinterpret_cast<float*>(out_xyz), nullptr, nullptr, 0, stream) != 0) {
      throw FoundationPoseError(std::string("test plugin render: ") + fpk_last_error());
    }
    g_render_calls.fetch_add(1);
  }

 private:
  fpk_params_t params_{};
};

}  // namespace

extern "C" {

#ifndef FP_TEST_PLUGIN_NO_FACTORY
__attribute__((visibility("default"))) IRenderer* fp_plugin_create_renderer(const Config* config, int device_id,
                                                                             int max_batch) {
#ifdef FP_TEST_PLUGIN_NULL_FACTORY
  (void)config;
  (void)device_id;
  (void)max_batch;
  return nullptr;
#else
  try {
    g_device_id = device_id;
    g_max_batch = max_batch;
    g_created.fetch_add(1);
    return new PluginRenderer(*config);
  } catch (...) {
    return nullptr;
  }
#endif
}
#endif

__attribute__((visibility("default"))) int fp_test_plugin_render_calls() { return g_render_calls.load(); }
__attribute__((visibility("default"))) int fp_test_plugin_created() { return g_created.load(); }
__attribute__((visibility("default"))) int fp_test_plugin_device_id() { return g_device_id; }
__attribute__((visibility("default"))) int fp_test_plugin_max_batch() { return g_max_batch; }

}  // extern "C"
