// Test-oracle shim (not product code): drives the reference's own CUDA kernels
// (src/cuda_pipeline.cu, src/builtin_raster_renderer.cu, src/raster_kernels.cuh,
// compiled unmodified for sm_100a by oracle/Makefile into
// oracle/_ref/libfpref_gpu.so) on host buffers, so GPU parity tests can compare
// the product kernels against the reference implementation on identical
// inputs. The renderer source is included into this translation unit so the
// shim can also read the reference's intermediate rast buffer (triangle ids),
// which BuiltinRasterRenderer keeps private. Only tests load this library.
#include <cstdint>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

#include "builtin_raster_renderer.cu"
#include "foundation_pose_nvidia/cuda_pipeline.hpp"

namespace fpn = foundation_pose_nvidia;

extern "C" {

// Flat mirror of the fields of the reference Config (config.hpp:20-67) that the
// hot path reads; the shim starts from Config{} and overrides these.
typedef struct refcfg {
  float depth_min, depth_max;
  int erosion_radius, bilateral_radius;
  float depth_diff_threshold, erosion_ratio_threshold, bilateral_sigma_d, bilateral_sigma_r;
  float crop_ratio;
  int input_width, input_height;
  float rotation_normalizer_rad, znear, zfar, ambient_weight, diffuse_weight;
} refcfg_t;

}  // extern "C"

namespace {

std::string g_error;

fpn::Config toConfig(const refcfg_t* c, int max_w, int max_h) {
  fpn::Config cfg;
  cfg.depth_min = c->depth_min;
  cfg.depth_max = c->depth_max;
  cfg.erosion_radius = c->erosion_radius;
  cfg.bilateral_radius = c->bilateral_radius;
  cfg.depth_diff_threshold = c->depth_diff_threshold;
  cfg.erosion_ratio_threshold = c->erosion_ratio_threshold;
  cfg.bilateral_sigma_d = c->bilateral_sigma_d;
  cfg.bilateral_sigma_r = c->bilateral_sigma_r;
  cfg.crop_ratio = c->crop_ratio;
  cfg.input_width = c->input_width;
  cfg.input_height = c->input_height;
  cfg.rotation_normalizer_rad = c->rotation_normalizer_rad;
  cfg.znear = c->znear;
  cfg.zfar = c->zfar;
  cfg.ambient_weight = c->ambient_weight;
  cfg.diffuse_weight = c->diffuse_weight;
  cfg.max_image_width = max_w;
  cfg.max_image_height = max_h;
  return cfg;
}

void d2h(void* dst, const void* src, std::size_t bytes) {
  fpn::checkCuda(cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost), "shim d2h");
}
void h2d(void* dst, const void* src, std::size_t bytes) {
  fpn::checkCuda(cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice), "shim h2d");
}

}  // namespace

extern "C" {

const char* refgpu_last_error(void) { return g_error.c_str(); }

// Depth preprocess + initial translation + pose seeding, exactly as
// FoundationPose::registerFrame sequences them (foundation_pose.cpp:344-349).
// Outputs (host): eroded/filtered depth [h*w], xyz [h*w*3], t0[3],
// seeded poses [n_seed*16] from the given rotations [n_seed*9].
int refgpu_preprocess(const std::uint8_t* rgb, const float* depth, const std::uint8_t* mask, int w,
                      int h, const float* k4, const refcfg_t* c, const float* rotations,
                      int n_seed, float* eroded, float* filtered, float* xyz, float* t0,
                      float* seeded) {
  try {
    const fpn::Config cfg = toConfig(c, w, h);
    fpn::GpuWorkspace ws(cfg, n_seed > 0 ? n_seed : 1);
    const fpn::CameraIntrinsics k{k4[0], k4[1], k4[2], k4[3]};
    fpn::uploadFrameToDevice(rgb, depth, mask, w, h, ws, nullptr);
    fpn::runDepthPreprocess(ws, w, h, cfg, nullptr);
    fpn::runDepthToXyz(ws, w, h, k, cfg, nullptr);
    if (mask != nullptr) {
      fpn::runInitialTranslation(ws, w, h, k, cfg, nullptr);
      if (n_seed > 0) {
        std::vector<fpn::Mat3f> rots(static_cast<std::size_t>(n_seed));
        for (int i = 0; i < n_seed; ++i) {
          std::memcpy(rots[i].values.data(), rotations + 9 * i, 9 * sizeof(float));
        }
        fpn::uploadRotationGridToDevice(rots, ws, nullptr);
        fpn::seedPosesFromRotations(ws, n_seed, nullptr);
      }
    }
    fpn::checkCuda(cudaDeviceSynchronize(), "shim preprocess sync");
    const std::size_t px = static_cast<std::size_t>(w) * h;
    d2h(eroded, ws.depth_eroded.data(), px * sizeof(float));
    d2h(filtered, ws.depth_filtered.data(), px * sizeof(float));
    d2h(xyz, ws.xyz_map.data(), px * 3 * sizeof(float));
    if (mask != nullptr) {
      d2h(t0, ws.init_translation.data(), 3 * sizeof(float));
      if (n_seed > 0) {
        d2h(seeded, ws.poses.data(), static_cast<std::size_t>(n_seed) * 16 * sizeof(float));
      }
    }
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return 1;
  }
}

// One prepareNetworkInputs pass (foundation_pose.cpp:429-443): crop boxes (K8),
// the built-in rasterizer (K9-K13, also returning the private rast buffer) and
// the network-input pack (K14). The frame is preprocessed first (K1-K3).
// Mesh colours are u8 and go through uploadMeshToDevice like fp_create does.
int refgpu_render_pass(const float* verts, const float* normals, const std::uint8_t* colors,
                       int n_verts, const std::int32_t* faces, int n_faces, float diameter,
                       const float* poses, int batch, const std::uint8_t* rgb, const float* depth,
                       int w, int h, const float* k4, const refcfg_t* c, float invalid_threshold,
                       float* boxes, float* out_rgb, float* out_xyz, float* out_rast,
                       float* net_rendered, float* net_observed) {
  try {
    const fpn::Config cfg = toConfig(c, w, h);
    const fpn::CameraIntrinsics k{k4[0], k4[1], k4[2], k4[3]};
    fpn::GpuWorkspace ws(cfg, batch);
    fpn::Mesh mesh;
    for (int i = 0; i < n_verts; ++i) {
      mesh.vertices.push_back({verts[3 * i], verts[3 * i + 1], verts[3 * i + 2]});
      mesh.normals.push_back({normals[3 * i], normals[3 * i + 1], normals[3 * i + 2]});
      mesh.vertex_colors.push_back({colors[3 * i], colors[3 * i + 1], colors[3 * i + 2]});
    }
    for (int i = 0; i < n_faces; ++i) {
      mesh.faces.push_back({static_cast<std::uint32_t>(faces[3 * i]),
                            static_cast<std::uint32_t>(faces[3 * i + 1]),
                            static_cast<std::uint32_t>(faces[3 * i + 2])});
    }
    fpn::DeviceMesh dm;
    fpn::uploadMeshToDevice(mesh, dm, nullptr);
    fpn::uploadFrameToDevice(rgb, depth, nullptr, w, h, ws, nullptr);
    fpn::runDepthPreprocess(ws, w, h, cfg, nullptr);
    fpn::runDepthToXyz(ws, w, h, k, cfg, nullptr);
    h2d(ws.poses.data(), poses, static_cast<std::size_t>(batch) * 16 * sizeof(float));
    fpn::computeCropBoxesOnDevice(ws.poses.as<float>(), batch, k, diameter, cfg,
                                  ws.crop_boxes.as<float>(), nullptr);

    // The renderer sequence of BuiltinRasterRenderer::render (builtin_raster_renderer.cu:218-281),
    // kept step by step so the rast buffer is observable.
    const int cw = cfg.input_width;
    const int ch = cfg.input_height;
    fpn::DeviceBuffer clip(static_cast<std::size_t>(batch) * n_verts * sizeof(float4));
    fpn::DeviceBuffer campos(static_cast<std::size_t>(batch) * n_verts * sizeof(float3));
    fpn::DeviceBuffer camnrm(static_cast<std::size_t>(batch) * n_verts * sizeof(float3));
    const std::size_t pixels = static_cast<std::size_t>(batch) * cw * ch;
    fpn::DeviceBuffer zbuf(pixels * sizeof(unsigned long long));
    fpn::DeviceBuffer rast(pixels * sizeof(float4));
    const int tv = batch * n_verts;
    fpn::raster_kernels::buildRenderVerticesKernel<<<(tv + 255) / 256, 256>>>(
        dm.vertices.as<float3>(), dm.normals.as<float3>(), ws.poses.as<float>(),
        ws.crop_boxes.as<float4>(), n_verts, batch, k, cfg, clip.as<float4>(),
        campos.as<float3>(), camnrm.as<float3>());
    fpn::checkCuda(cudaMemset(zbuf.data(), 0xFF, pixels * sizeof(unsigned long long)), "memset");
    const int tt = batch * n_faces;
    fpn::rasterTrianglesKernel<<<(tt + 255) / 256, 256>>>(clip.as<float4>(), dm.faces.as<int3>(),
                                                          n_verts, n_faces, batch, cw, ch,
                                                          zbuf.as<unsigned long long>());
    const int tp = static_cast<int>(pixels);
    fpn::resolveRastKernel<<<(tp + 255) / 256, 256>>>(zbuf.as<unsigned long long>(),
                                                      clip.as<float4>(), dm.faces.as<int3>(),
                                                      n_verts, batch, cw, ch, rast.as<float4>());
    fpn::raster_kernels::shadeRasterKernel<<<(tp + 255) / 256, 256>>>(
        rast.as<float4>(), dm.faces.as<int3>(), campos.as<float3>(), camnrm.as<float3>(),
        dm.uvs.as<float2>(), dm.colors.as<float3>(), dm.texture_rgb.as<float3>(),
        dm.texture_width, dm.texture_height, n_verts, n_faces, batch, cw, ch, dm.has_texture,
        dm.has_uvs, cfg, ws.rendered_rgb.as<float3>(), ws.rendered_xyz.as<float3>());
    fpn::checkCuda(cudaGetLastError(), "shim render launch");
    fpn::prepareNetworkInputsOnDevice(ws, ws.poses.as<float>(), batch, w, h, diameter,
                                      invalid_threshold, nullptr);
    fpn::checkCuda(cudaDeviceSynchronize(), "shim render sync");
    d2h(boxes, ws.crop_boxes.data(), static_cast<std::size_t>(batch) * 4 * sizeof(float));
    d2h(out_rgb, ws.rendered_rgb.data(), pixels * 3 * sizeof(float));
    d2h(out_xyz, ws.rendered_xyz.data(), pixels * 3 * sizeof(float));
    d2h(out_rast, rast.data(), pixels * 4 * sizeof(float));
    d2h(net_rendered, ws.network_rendered.data(), pixels * 6 * sizeof(float));
    d2h(net_observed, ws.network_observed.data(), pixels * 6 * sizeof(float));
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return 1;
  }
}

// K15 applyPoseDeltasOnDevice (cuda_pipeline.cu:847-858) on host buffers, in place.
int refgpu_apply_deltas(float* poses, const float* dt, const float* dr, int batch, float diameter,
                        float rotation_normalizer_rad) {
  try {
    fpn::Config cfg;
    cfg.rotation_normalizer_rad = rotation_normalizer_rad;
    fpn::DeviceBuffer p(static_cast<std::size_t>(batch) * 16 * sizeof(float));
    fpn::DeviceBuffer t(static_cast<std::size_t>(batch) * 3 * sizeof(float));
    fpn::DeviceBuffer r(static_cast<std::size_t>(batch) * 3 * sizeof(float));
    h2d(p.data(), poses, p.bytes());
    h2d(t.data(), dt, t.bytes());
    h2d(r.data(), dr, r.bytes());
    fpn::applyPoseDeltasOnDevice(p.as<float>(), t.as<float>(), r.as<float>(), batch, diameter,
                                 cfg, nullptr);
    fpn::checkCuda(cudaDeviceSynchronize(), "shim delta sync");
    d2h(poses, p.data(), p.bytes());
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return 1;
  }
}

// K16 selectBestPoseOnDevice (cuda_pipeline.cu:860-868): pose16, score, index.
int refgpu_select_best(const float* poses, const float* scores, int batch, const float* center3,
                       float* out_pose, float* out_score, int* out_index) {
  try {
    fpn::DeviceBuffer p(static_cast<std::size_t>(batch) * 16 * sizeof(float));
    fpn::DeviceBuffer s(static_cast<std::size_t>(batch) * sizeof(float));
    fpn::DeviceBuffer res(sizeof(fpn::DevicePoseResult));
    h2d(p.data(), poses, p.bytes());
    h2d(s.data(), scores, s.bytes());
    fpn::selectBestPoseOnDevice(p.as<float>(), s.as<float>(), batch,
                                fpn::Vec3f{center3[0], center3[1], center3[2]},
                                res.as<fpn::DevicePoseResult>(), nullptr);
    fpn::DevicePoseResult host;
    fpn::checkCuda(cudaDeviceSynchronize(), "shim select sync");
    d2h(&host, res.data(), sizeof(host));
    std::memcpy(out_pose, host.pose.values.data(), 16 * sizeof(float));
    *out_score = host.score;
    *out_index = host.index;
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return 1;
  }
}

}  // extern "C"
