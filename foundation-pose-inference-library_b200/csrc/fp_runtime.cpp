// Estimator runtime and the stable fp_* C ABI.
//
// Register (reference src/foundation_pose.cpp:312-377) and track (:379-410)
// sequence the sm_100a kernels of fpk_pipeline.cu and the networks of
// fp_network.cu on the estimator's own stream. With the built-in renderer and
// networks, each refinement pass is
//   fpk_render_pack (crop boxes + raster + shade + crop-warp + pack, one launch)
//   -> RefineNet (tcgen05 GEMMs) -> fpk_apply_deltas
// with no host synchronisation until the final pose read. Injected IRenderer /
// IInferenceRunner backends are driven through the reference's NCHW fp32 seam.
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <algorithm>
#include <condition_variable>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <format>
#include <functional>
#include <latch>
#include <memory>
#include <mutex>
#include <string>
#include <string_view>
#include <thread>
#include <utility>
#include <vector>

#include "foundation_pose_nvidia/builtin_raster_renderer.hpp"
#include "foundation_pose_nvidia/c_api.h"
#include "foundation_pose_nvidia/foundation_pose.hpp"
#include "foundation_pose_nvidia/tensorrt_runner.hpp"
#include "fp_host.hpp"
#include "fp_network.hpp"
#include "fpk.h"

namespace fpb {
int fail(const std::string& msg);
}

namespace foundation_pose_nvidia {

void checkCuda(cudaError_t status, const char* what) {
  if (status != cudaSuccess) {
    throw FoundationPoseError(std::string(what) + ": " + cudaGetErrorString(status));
  }
}

DeviceBuffer::DeviceBuffer(DeviceBuffer&& o) noexcept
    : ptr_(std::exchange(o.ptr_, nullptr)), bytes_(std::exchange(o.bytes_, 0)) {}
DeviceBuffer& DeviceBuffer::operator=(DeviceBuffer&& o) noexcept {
  if (this != &o) {
    reset();
    ptr_ = std::exchange(o.ptr_, nullptr);
    bytes_ = std::exchange(o.bytes_, 0);
  }
  return *this;
}
DeviceBuffer::~DeviceBuffer() { reset(); }
void DeviceBuffer::allocate(std::size_t bytes) {
  reset();
  if (bytes == 0) return;
  checkCuda(cudaMalloc(&ptr_, bytes), "cudaMalloc");
  bytes_ = bytes;
  checkCuda(cudaMemset(ptr_, 0, bytes), "cudaMemset");
}
void DeviceBuffer::reset() {
  if (ptr_ != nullptr) cudaFree(ptr_);
  ptr_ = nullptr;
  bytes_ = 0;
}

CudaStream::CudaStream(unsigned int flags) {
  checkCuda(cudaStreamCreateWithFlags(&stream_, flags), "cudaStreamCreateWithFlags");
}
CudaStream::CudaStream(CudaStream&& o) noexcept : stream_(std::exchange(o.stream_, nullptr)) {}
CudaStream& CudaStream::operator=(CudaStream&& o) noexcept {
  if (this != &o) {
    if (stream_ != nullptr) cudaStreamDestroy(stream_);
    stream_ = std::exchange(o.stream_, nullptr);
  }
  return *this;
}
CudaStream::~CudaStream() {
  if (stream_ != nullptr) cudaStreamDestroy(stream_);
}
void CudaStream::synchronize() const { checkCuda(cudaStreamSynchronize(stream_), "cudaStreamSynchronize"); }

namespace {

void fpkCheck(int rc) {
  if (rc != 0) throw FoundationPoseError(fpk_last_error());
}

fpk_params_t toParams(const Config& c) {
  fpk_params_t p;
  p.depth_min = c.depth_min;
  p.depth_max = c.depth_max;
  p.erosion_radius = c.erosion_radius;
  p.bilateral_radius = c.bilateral_radius;
  p.depth_diff_threshold = c.depth_diff_threshold;
  p.erosion_ratio_threshold = c.erosion_ratio_threshold;
  p.bilateral_sigma_d = c.bilateral_sigma_d;
  p.bilateral_sigma_r = c.bilateral_sigma_r;
  p.crop_ratio = c.crop_ratio;
  p.input_width = c.input_width;
  p.input_height = c.input_height;
  p.rotation_normalizer_rad = c.rotation_normalizer_rad;
  p.znear = c.znear;
  p.zfar = c.zfar;
  p.ambient_weight = c.ambient_weight;
  p.diffuse_weight = c.diffuse_weight;
  return p;
}

fpk_intrinsics_t toK(CameraIntrinsics k) { return {k.fx, k.fy, k.cx, k.cy}; }

fpk_mesh_t meshView(const DeviceMesh& m) {
  fpk_mesh_t v{};
  v.vertices = m.vertices.as<float>();
  v.normals = m.normals.as<float>();
  v.colors = m.colors.as<float>();
  const bool tex = m.has_texture && m.has_uvs;
  v.uvs = tex ? m.uvs.as<float>() : nullptr;
  v.texture = tex ? m.texture_rgb.as<float>() : nullptr;
  v.faces = m.faces.as<int32_t>();
  v.n_vertices = m.num_vertices;
  v.n_faces = m.num_faces;
  v.texture_width = tex ? m.texture_width : 0;
  v.texture_height = tex ? m.texture_height : 0;
  return v;
}

void uploadMesh(const Mesh& mesh, DeviceMesh& dst, cudaStream_t s) {
  const std::size_t nv = mesh.vertices.size();
  dst.num_vertices = static_cast<int>(nv);
  dst.num_faces = static_cast<int>(mesh.faces.size());
  dst.texture_width = mesh.texture_width;
  dst.texture_height = mesh.texture_height;
  dst.has_texture = mesh.hasTexture();
  dst.has_uvs = !mesh.uvs.empty();
  std::vector<float> v(3 * nv), n(3 * nv), c(3 * nv), uv(2 * nv);
  for (std::size_t i = 0; i < nv; ++i) {
    v[3 * i] = mesh.vertices[i].x;
    v[3 * i + 1] = mesh.vertices[i].y;
    v[3 * i + 2] = mesh.vertices[i].z;
    const Vec3f nn = i < mesh.normals.size() ? mesh.normals[i] : Vec3f{0.0f, 0.0f, 1.0f};
    n[3 * i] = nn.x;
    n[3 * i + 1] = nn.y;
    n[3 * i + 2] = nn.z;
    const Vec3u8 cc = i < mesh.vertex_colors.size() ? mesh.vertex_colors[i] : Vec3u8{128, 128, 128};
    c[3 * i] = static_cast<float>(cc.r) / 255.0f;
    c[3 * i + 1] = static_cast<float>(cc.g) / 255.0f;
    c[3 * i + 2] = static_cast<float>(cc.b) / 255.0f;
    const Vec2f u = i < mesh.uvs.size() ? mesh.uvs[i] : Vec2f{};
    uv[2 * i] = u.x;
    uv[2 * i + 1] = u.y;
  }
  std::vector<int32_t> f(3 * mesh.faces.size());
  for (std::size_t i = 0; i < mesh.faces.size(); ++i) {
    for (int k = 0; k < 3; ++k) {
      if (mesh.faces[i][k] >= nv) throw FoundationPoseError("Mesh face references a missing vertex");
      f[3 * i + k] = static_cast<int32_t>(mesh.faces[i][k]);
    }
  }
  auto put = [&](DeviceBuffer& b, const void* src, std::size_t bytes) {
    b.allocate(bytes);
    checkCuda(cudaMemcpyAsync(b.data(), src, bytes, cudaMemcpyHostToDevice, s), "upload mesh");
  };
  put(dst.vertices, v.data(), v.size() * 4);
  put(dst.normals, n.data(), n.size() * 4);
  put(dst.colors, c.data(), c.size() * 4);
  put(dst.uvs, uv.data(), uv.size() * 4);
  put(dst.faces, f.data(), f.size() * 4);
  if (dst.has_texture) {
    std::vector<float> t(3 * mesh.texture_rgb.size());
    for (std::size_t i = 0; i < mesh.texture_rgb.size(); ++i) {
      t[3 * i] = static_cast<float>(mesh.texture_rgb[i].r) / 255.0f;
      t[3 * i + 1] = static_cast<float>(mesh.texture_rgb[i].g) / 255.0f;
      t[3 * i + 2] = static_cast<float>(mesh.texture_rgb[i].b) / 255.0f;
    }
    put(dst.texture_rgb, t.data(), t.size() * 4);
  }
  checkCuda(cudaStreamSynchronize(s), "upload mesh");
}

}  // namespace

// Built-in renderer behind the IRenderer seam (fpk_render into the caller's
// NHWC buffers; the estimator fuses it with the pack when it also runs the
// built-in networks).
struct BuiltinRasterRenderer::Impl {
  fpk_params_t params;
  int max_batch;
  DeviceBuffer workspace;
};

BuiltinRasterRenderer::BuiltinRasterRenderer(const Config& config, int device_id, int max_batch)
    : impl_(std::make_unique<Impl>(Impl{toParams(config), std::max(1, max_batch), DeviceBuffer{}})) {
  int current = -1;
  checkCuda(cudaGetDevice(&current), "cudaGetDevice");
  if (current != device_id) checkCuda(cudaSetDevice(device_id), "cudaSetDevice");
}

BuiltinRasterRenderer::~BuiltinRasterRenderer() = default;

void BuiltinRasterRenderer::reserveForMesh(int num_vertices, int) {
  const std::size_t bytes = fpk_render_workspace_bytes(impl_->max_batch, num_vertices, &impl_->params);
  if (bytes > impl_->workspace.bytes()) impl_->workspace.allocate(bytes);
}

void BuiltinRasterRenderer::render(const DeviceMesh& mesh, const float* poses, const float* crop_boxes,
                                   int batch_size, CameraIntrinsics k, int, int, float3* out_rgb, float3* out_xyz,
                                   cudaStream_t stream) {
  if (mesh.num_vertices <= 0 || mesh.num_faces <= 0) {
    throw FoundationPoseError("builtin renderer received an empty mesh");
  }
  const std::size_t need = fpk_render_workspace_bytes(batch_size, mesh.num_vertices, &impl_->params);
  if (need > impl_->workspace.bytes()) {
    checkCuda(cudaStreamSynchronize(stream), "renderer workspace resize");
    impl_->workspace.allocate(need);
  }
  const fpk_mesh_t m = meshView(mesh);
  fpkCheck(fpk_render(&m, poses, crop_boxes, batch_size, toK(k), &impl_->params, reinterpret_cast<float*>(out_rgb),
                      reinterpret_cast<float*>(out_xyz), nullptr, impl_->workspace.data(), impl_->workspace.bytes(),
                      stream));
}

namespace {

// Default-renderer selection (reference src/foundation_pose.cpp:40-68): the
// built-in rasterizer unless FP_RENDERER=nvdiffrast, which loads the renderer
// plugin libfoundation_pose_nvdiffrast.so with dlopen and builds the renderer
// through its extern "C" factory
//   IRenderer* fp_plugin_create_renderer(const Config*, int device_id, int max_batch).
// The plugin is looked up on the dynamic loader's path first, then in the
// directory of this library. It is loaded once per process and never unloaded
// (renderers it created may outlive any estimator).
constexpr const char* kRendererPluginName = "libfoundation_pose_nvdiffrast.so";
using PluginRendererFactory = IRenderer* (*)(const Config*, int, int);

struct RendererPlugin {
  void* handle = nullptr;
  std::string error;
};

const RendererPlugin& rendererPlugin() {
  static const RendererPlugin plugin = [] {
    RendererPlugin p;
    p.handle = dlopen(kRendererPluginName, RTLD_NOW | RTLD_LOCAL);
    if (p.handle != nullptr) return p;
    const char* first = dlerror();
    p.error = first != nullptr ? first : "not found";
    Dl_info self{};
    if (dladdr(reinterpret_cast<const void*>(&rendererPlugin), &self) != 0 && self.dli_fname != nullptr) {
      std::string dir(self.dli_fname);
      const std::size_t slash = dir.rfind('/');
      dir = slash == std::string::npos ? std::string(".") : dir.substr(0, slash);
      p.handle = dlopen((dir + "/" + kRendererPluginName).c_str(), RTLD_NOW | RTLD_LOCAL);
      if (p.handle == nullptr) {
        const char* second = dlerror();
        if (second != nullptr) p.error += std::string("; ") + second;
      }
    }
    return p;
  }();
  return plugin;
}

std::unique_ptr<IRenderer> makeDefaultRenderer(const Config& config, int device_id, int max_batch) {
  const char* choice = std::getenv("FP_RENDERER");
  if (choice == nullptr || std::string_view(choice) != "nvdiffrast") {
    return std::make_unique<BuiltinRasterRenderer>(config, device_id, max_batch);
  }
  const RendererPlugin& plugin = rendererPlugin();
  if (plugin.handle == nullptr) {
    throw FoundationPoseError(
        "FP_RENDERER=nvdiffrast requested but the renderer plugin could not be loaded (keep " +
        std::string(kRendererPluginName) + " on the loader path or next to the main library): " + plugin.error);
  }
  auto factory = reinterpret_cast<PluginRendererFactory>(dlsym(plugin.handle, "fp_plugin_create_renderer"));
  if (factory == nullptr) {
    throw FoundationPoseError("nvdiffrast renderer plugin is missing fp_plugin_create_renderer");
  }
  std::unique_ptr<IRenderer> renderer(factory(&config, device_id, max_batch));
  if (!renderer) throw FoundationPoseError("nvdiffrast renderer plugin failed to create a renderer");
  return renderer;
}

fpb::NetPrecision toNetPrecision(TensorrtPrecision p) {
  switch (p) {
    case TensorrtPrecision::kFP16:
      return fpb::NetPrecision::kFP16;
    case TensorrtPrecision::kBF16:
      return fpb::NetPrecision::kBF16;
    case TensorrtPrecision::kTF32:
      return fpb::NetPrecision::kTF32;
    default:
      return fpb::NetPrecision::kFP32;
  }
}

}  // namespace

// Exceptions of the network code surface as FoundationPoseError.
template <class F>
void runNet(F&& f) {
  try {
    f();
  } catch (const FoundationPoseError&) {
    throw;
  } catch (const std::exception& e) {
    throw FoundationPoseError(e.what());
  }
}

// Built-in RefineNet/ScoreNet behind the IInferenceRunner seam. The networks
// are created on first use (like the reference's lazily built engines).
struct TensorRtRunner::Impl {
  RuntimeOptions opts;
  Config cfg;
  int max_batch = 0;
  int engine_batch = 0;
  std::unique_ptr<fpb::NetworkRunner> net_;

  fpb::NetworkRunner& net() {
    if (!net_) {
      if (opts.refine_model_path.empty()) throw FoundationPoseError("refine_model_path is required");
      if (opts.score_model_path.empty()) throw FoundationPoseError("score_model_path is required");
      runNet([&] {
        net_ = std::make_unique<fpb::NetworkRunner>(opts.refine_model_path, opts.score_model_path,
                                                    toNetPrecision(cfg.tensorrt_precision), max_batch,
                                                    cfg.input_width, cfg.input_height);
      });
    }
    return *net_;
  }
};

TensorRtRunner::TensorRtRunner(RuntimeOptions options, Config config, int max_batch)
    : impl_(std::make_unique<Impl>()) {
  Impl& I = *impl_;
  I.opts = std::move(options);
  I.cfg = config;
  I.max_batch = max_batch;
  const int bs = config.batch_size > 0 ? config.batch_size : max_batch;
  I.engine_batch = std::min(max_batch, bs);
  if (I.engine_batch <= 0 || max_batch % I.engine_batch != 0) {
    throw FoundationPoseError("max_batch (" + std::to_string(max_batch) + ") must be divisible by effective_bs (" +
                              std::to_string(I.engine_batch) + ")");
  }
  checkCuda(cudaSetDevice(I.opts.device_id), "cudaSetDevice");
}

TensorRtRunner::~TensorRtRunner() = default;

void TensorRtRunner::prepareForBatch(int batch_size) {
  if (batch_size <= 0 || batch_size > impl_->max_batch) {
    throw FoundationPoseError("prepare batch size exceeds configured maximum");
  }
  (void)impl_->net();
}

void TensorRtRunner::enqueueRefine(const float* rendered, const float* observed, float* dt, float* dr, int batch,
                                   cudaStream_t stream) {
  Impl& I = *impl_;
  if (batch <= 0 || batch > I.max_batch) throw FoundationPoseError("refine batch size exceeds configured maximum");
  const std::size_t stride = static_cast<std::size_t>(6) * I.cfg.input_width * I.cfg.input_height;
  for (int off = 0; off < batch; off += I.engine_batch) {
    const int chunk = std::min(I.engine_batch, batch - off);
    I.net().loadNchw(rendered + off * stride, observed + off * stride, chunk, stream);
    runNet([&] { I.net().refine(chunk, 0, dt + 3 * off, dr + 3 * off, stream); });
  }
}

void TensorRtRunner::enqueueScore(const float* rendered, const float* observed, float* scores, int batch,
                                  cudaStream_t stream) {
  Impl& I = *impl_;
  if (batch <= 0 || batch > I.max_batch) throw FoundationPoseError("score batch size exceeds configured maximum");
  I.net().loadNchw(rendered, observed, batch, stream);
  runNet([&] { I.net().score(batch, scores, stream); });
}

struct FoundationPose::Impl {
  PreprocessedMesh mesh;
  RuntimeOptions opts;
  Config cfg;
  fpk_params_t params{};
  int max_hyp = 0;
  int active = 0;
  bool has_prev = false;
  std::unique_ptr<CudaStream> stream;
  DeviceMesh dmesh;
  std::unique_ptr<IInferenceRunner> inference;
  std::unique_ptr<IRenderer> renderer;
  TensorRtRunner::Impl* builtin_runner = nullptr;  // the built-in networks, when injected or default
  bool fused = false;  // built-in renderer + networks: fused render/pack path
  int rotation_count = 0;
  DeviceBuffer rgb, mask, depth_raw, depth_filtered, stats, rotations, poses, prev_pose, boxes;
  DeviceBuffer dt, dr, scores, best, one, seeded;
  DeviceBuffer render_ws;  // fused path: fpk_render_pack workspace for max_hyp hypotheses
  DeviceBuffer rend_rgb, rend_xyz, net_rendered, net_observed;  // seam path only
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t graph_exec = nullptr;
  int graph_batch = 0, graph_w = 0, graph_h = 0;
  CameraIntrinsics graph_k{};
  // Whole track call (preprocess -> previous pose -> passes -> select) as one
  // graph, kept apart from the register's refinement graph so alternating
  // register and track calls re-capture neither.
  cudaGraphExec_t track_exec = nullptr;
  int track_iters = -1, track_w = 0, track_h = 0;
  CameraIntrinsics track_k{};

  ~Impl() {
    destroyGraph();
    destroyTrackGraph();
  }

  void destroyTrackGraph() noexcept {
    if (track_exec != nullptr) cudaGraphExecDestroy(track_exec);
    track_exec = nullptr;
    track_iters = -1;
  }

  void destroyGraph() noexcept {
    if (graph_exec != nullptr) cudaGraphExecDestroy(graph_exec);
    if (graph != nullptr) cudaGraphDestroy(graph);
    graph_exec = nullptr;
    graph = nullptr;
    graph_batch = graph_w = graph_h = 0;
  }

  cudaStream_t s() const { return stream->get(); }

  void validateFrame(const void* rgb_u8, const float* depth_m, const void* mask_u8, int w, int h,
                     bool need_mask) const {
    if (rgb_u8 == nullptr || depth_m == nullptr || (need_mask && mask_u8 == nullptr)) {
      throw FoundationPoseError("RGB, depth, and mask pointers are required");
    }
    if (w <= 0 || h <= 0) throw FoundationPoseError("Image dimensions must be positive");
    if (w > cfg.max_image_width || h > cfg.max_image_height) {
      throw FoundationPoseError("Image exceeds configured max_image_width/max_image_height");
    }
  }

  void upload(const std::uint8_t* rgb_u8, const float* depth_m, const std::uint8_t* mask_u8, int w, int h) {
    const std::size_t px = static_cast<std::size_t>(w) * h;
    checkCuda(cudaMemcpyAsync(rgb.data(), rgb_u8, px * 3, cudaMemcpyDefault, s()), "cudaMemcpyAsync rgb");
    checkCuda(cudaMemcpyAsync(depth_raw.data(), depth_m, px * 4, cudaMemcpyDefault, s()), "cudaMemcpyAsync depth");
    if (mask_u8 != nullptr) {
      checkCuda(cudaMemcpyAsync(mask.data(), mask_u8, px, cudaMemcpyDefault, s()), "cudaMemcpyAsync mask");
    }
  }

  // One refinement pass over n hypotheses in chunks of `chunk`.
  void refinePass(int n, int chunk, int w, int h, CameraIntrinsics k) {
    if (fused) {
      fpb::NetworkRunner& net = builtin_runner->net();
      const fpk_mesh_t m = meshView(dmesh);
      for (int off = 0; off < n; off += chunk) {
        const int c = std::min(chunk, n - off);
        fpkCheck(fpk_render_pack(&m, poses.as<float>() + 16 * off, c, rgb.as<uint8_t>(),
                                 depth_filtered.as<float>(), w, h, toK(k), &params, mesh.diameter,
                                 cfg.depth_min, net.dtype(), net.stem().base, net.stem().plane_stride,
                                 boxes.as<float>() + 4 * off, render_ws.data(), render_ws.bytes(), s()));
        runNet(
            [&] { net.refine(c, 0, dt.as<float>() + 3 * off, dr.as<float>() + 3 * off, s()); });
      }
    } else {
      prepareSeamInputs(n, w, h, k, cfg.depth_min);
      inference->enqueueRefine(net_rendered.as<float>(), net_observed.as<float>(), dt.as<float>(),
                               dr.as<float>(), n, s());
    }
    fpkCheck(fpk_apply_deltas(poses.as<float>(), dt.as<float>(), dr.as<float>(), n, mesh.diameter,
                              &params, s()));
  }

  void prepareSeamInputs(int n, int w, int h, CameraIntrinsics k, float threshold) {
    fpkCheck(fpk_crop_boxes(poses.as<float>(), n, toK(k), mesh.diameter, &params, boxes.as<float>(), s()));
    renderer->render(dmesh, poses.as<float>(), boxes.as<float>(), n, k, w, h,
                     rend_rgb.as<float3>(), rend_xyz.as<float3>(), s());
    fpkCheck(fpk_pack(rgb.as<uint8_t>(), depth_filtered.as<float>(), w, h, toK(k), &params,
                      rend_rgb.as<float>(), rend_xyz.as<float>(), poses.as<float>(), boxes.as<float>(),
                      n, mesh.diameter, threshold, net_rendered.as<float>(), net_observed.as<float>(),
                      s()));
  }

  void scorePass(int n, int w, int h, CameraIntrinsics k) {
    if (fused) {
      fpb::NetworkRunner& net = builtin_runner->net();
      const fpk_mesh_t m = meshView(dmesh);
      fpkCheck(fpk_render_pack(&m, poses.as<float>(), n, rgb.as<uint8_t>(), depth_filtered.as<float>(),
                               w, h, toK(k), &params, mesh.diameter, 0.1f, net.dtype(), net.stem().base,
                               net.stem().plane_stride, boxes.as<float>(), render_ws.data(), render_ws.bytes(), s()));
      runNet([&] { net.score(n, scores.as<float>(), s()); });
    } else {
      prepareSeamInputs(n, w, h, k, 0.1f);
      inference->enqueueScore(net_rendered.as<float>(), net_observed.as<float>(), scores.as<float>(), n, s());
    }
  }

  void refinementLoop(int iters, int n, int chunk, int w, int h, CameraIntrinsics k) {
    if (iters <= 0) return;
    if (cfg.capture_cuda_graph) {
      const bool stale = graph_exec == nullptr || graph_batch != n || graph_w != w || graph_h != h ||
                         graph_k.fx != k.fx || graph_k.fy != k.fy || graph_k.cx != k.cx || graph_k.cy != k.cy;
      if (stale) captureGraph(n, chunk, w, h, k);
      for (int i = 0; i < iters; ++i) checkCuda(cudaGraphLaunch(graph_exec, s()), "cudaGraphLaunch refinement graph");
      return;
    }
    for (int i = 0; i < iters; ++i) refinePass(n, chunk, w, h, k);
  }

  void captureGraph(int n, int chunk, int w, int h, CameraIntrinsics k) {
    destroyGraph();
    inference->prepareForBatch(n);
    // One uncaptured pass would change the poses; warm the launch attributes instead.
    checkCuda(cudaStreamBeginCapture(s(), cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
    bool open = true;
    try {
      refinePass(n, chunk, w, h, k);
      checkCuda(cudaStreamEndCapture(s(), &graph), "cudaStreamEndCapture");
      open = false;
      checkCuda(cudaGraphInstantiate(&graph_exec, graph, 0), "cudaGraphInstantiate");
    } catch (...) {
      if (open) {
        cudaGraph_t abandoned = nullptr;
        cudaStreamEndCapture(s(), &abandoned);
        if (abandoned != nullptr) cudaGraphDestroy(abandoned);
      }
      destroyGraph();
      throw;
    }
    graph_batch = n;
    graph_w = w;
    graph_h = h;
    graph_k = k;
  }

  // Device work of one track call after the frame upload (reference
  // src/foundation_pose.cpp:379-410).
  void trackBody(int iters, int w, int h, CameraIntrinsics k) {
    fpkCheck(fpk_preprocess(depth_raw.as<float>(), nullptr, w, h, toK(k), &params, depth_filtered.as<float>(),
                            nullptr, nullptr, nullptr, s()));
    checkCuda(cudaMemcpyAsync(poses.data(), prev_pose.data(), 64, cudaMemcpyDeviceToDevice, s()),
              "cudaMemcpyAsync device pose");
    for (int i = 0; i < iters; ++i) refinePass(1, 1, w, h, k);
    const float center[3] = {mesh.center.x, mesh.center.y, mesh.center.z};
    fpkCheck(fpk_select_best(poses.as<float>(), one.as<float>(), 1, center, best.as<float>(), s()));
    checkCuda(cudaMemcpyAsync(prev_pose.data(), poses.data(), 64, cudaMemcpyDeviceToDevice, s()),
              "cudaMemcpyAsync device pose");
  }

  void trackCall(int iters, int w, int h, CameraIntrinsics k) {
    if (!cfg.capture_cuda_graph) {
      trackBody(iters, w, h, k);
      return;
    }
    const bool stale = track_exec == nullptr || track_iters != iters || track_w != w || track_h != h ||
                       track_k.fx != k.fx || track_k.fy != k.fy || track_k.cx != k.cx || track_k.cy != k.cy;
    if (stale) {
      destroyTrackGraph();
      inference->prepareForBatch(1);
      checkCuda(cudaStreamBeginCapture(s(), cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
      cudaGraph_t g = nullptr;
      try {
        trackBody(iters, w, h, k);
      } catch (...) {
        cudaStreamEndCapture(s(), &g);
        if (g != nullptr) cudaGraphDestroy(g);
        throw;
      }
      checkCuda(cudaStreamEndCapture(s(), &g), "cudaStreamEndCapture");
      const cudaError_t e = cudaGraphInstantiate(&track_exec, g, 0);
      cudaGraphDestroy(g);
      if (e != cudaSuccess) {
        track_exec = nullptr;
        checkCuda(e, "cudaGraphInstantiate track graph");
      }
      track_iters = iters;
      track_w = w;
      track_h = h;
      track_k = k;
    }
    checkCuda(cudaGraphLaunch(track_exec, s()), "cudaGraphLaunch track graph");
  }

  void checkNetworkErrors() {
    if (builtin_runner == nullptr) return;
    int* flag = builtin_runner->net().errorFlag();
    int host = 0;
    checkCuda(cudaMemcpyAsync(&host, flag, sizeof(int), cudaMemcpyDeviceToHost, s()), "read error flag");
    stream->synchronize();
    if (host != 0) {
      runNet([&] { builtin_runner->net().clearError(s()); });
      stream->synchronize();
      throw FoundationPoseError("network kernel pipeline timed out (code " + std::to_string(host) + ")");
    }
  }

  PoseEstimate readBest() {
    float host[18];
    checkCuda(cudaMemcpyAsync(host, best.data(), sizeof(host), cudaMemcpyDeviceToHost, s()), "cudaMemcpyAsync best result");
    stream->synchronize();
    if (fused || builtin_runner != nullptr) checkNetworkErrors();
    PoseEstimate e;
    std::memcpy(e.pose.values.data(), host, 16 * sizeof(float));
    e.score = host[16];
    int idx = 0;
    std::memcpy(&idx, host + 17, sizeof(int));
    last_index = idx;
    return e;
  }

  int last_index = 0;
};

namespace {

CameraIntrinsics validateIntrinsics(CameraIntrinsics k) {
  if (k.fx <= 0.0f || k.fy <= 0.0f) throw FoundationPoseError("Camera intrinsics must have positive focal lengths");
  return k;
}

int maxHypothesesFor(const Config& c) { return std::max(1, c.n_hypotheses); }

}  // namespace

FoundationPose::FoundationPose(PreprocessedMesh mesh, RuntimeOptions runtime_options, Config config)
    : FoundationPose(std::move(mesh), runtime_options,
                     std::make_unique<TensorRtRunner>(runtime_options, config, maxHypothesesFor(config)),
                     makeDefaultRenderer(config, runtime_options.device_id, maxHypothesesFor(config)),
                     config) {}

FoundationPose::FoundationPose(PreprocessedMesh mesh, RuntimeOptions runtime_options,
                               std::unique_ptr<IInferenceRunner> inference_runner,
                               std::unique_ptr<IRenderer> renderer, Config config)
    : impl_(std::make_unique<Impl>()) {
  Impl& I = *impl_;
  if (!inference_runner || !renderer) {
    throw FoundationPoseError("FoundationPose requires inference and renderer backends");
  }
  I.mesh = std::move(mesh);
  I.opts = std::move(runtime_options);
  I.cfg = config;
  I.params = toParams(config);
  I.max_hyp = maxHypothesesFor(config);
  int current = -1;
  checkCuda(cudaGetDevice(&current), "cudaGetDevice");
  if (current != I.opts.device_id) checkCuda(cudaSetDevice(I.opts.device_id), "cudaSetDevice");
  I.stream = std::make_unique<CudaStream>();
  I.inference = std::move(inference_runner);
  I.renderer = std::move(renderer);
  if (auto* r = dynamic_cast<TensorRtRunner*>(I.inference.get())) I.builtin_runner = &r->impl();
  I.fused = I.builtin_runner != nullptr && dynamic_cast<BuiltinRasterRenderer*>(I.renderer.get()) != nullptr;

  const std::size_t px = static_cast<std::size_t>(config.max_image_width) * config.max_image_height;
  if (px == 0 || config.input_width <= 0 || config.input_height <= 0) {
    throw FoundationPoseError("Invalid GPU workspace dimensions");
  }
  const std::size_t B = static_cast<std::size_t>(I.max_hyp);
  I.rgb.allocate(px * 3);
  I.mask.allocate(px);
  I.depth_raw.allocate(px * 4);
  I.depth_filtered.allocate(px * 4);
  I.stats.allocate(FPK_STATS_INTS * 4);
  I.poses.allocate(B * 16 * 4);
  I.prev_pose.allocate(16 * 4);
  I.boxes.allocate(B * 4 * 4);
  I.dt.allocate(B * 3 * 4);
  I.dr.allocate(B * 3 * 4);
  I.scores.allocate(B * 4);
  I.best.allocate(18 * 4);
  I.seeded.allocate(B * 16 * 4);
  I.one.allocate(4);
  const float one = 1.0f;
  checkCuda(cudaMemcpy(I.one.data(), &one, 4, cudaMemcpyHostToDevice), "upload constant");
  if (!I.fused) {
    const std::size_t cp = static_cast<std::size_t>(config.input_width) * config.input_height;
    I.rend_rgb.allocate(B * cp * 12);
    I.rend_xyz.allocate(B * cp * 12);
    I.net_rendered.allocate(B * 6 * cp * 4);
    I.net_observed.allocate(B * 6 * cp * 4);
  }
  uploadMesh(I.mesh.centered_mesh, I.dmesh, I.s());
  if (I.dmesh.num_faces >= (1 << 24)) throw FoundationPoseError("meshes are limited to 2^24 triangles");
  I.renderer->reserveForMesh(I.dmesh.num_vertices, I.dmesh.num_faces);
  if (I.fused) I.render_ws.allocate(fpk_render_workspace_bytes(I.max_hyp, I.dmesh.num_vertices, &I.params));
  std::vector<Mat3f> rots = fpb_host::makeRotationGrid(config);
  if (rots.empty()) throw FoundationPoseError("Rotation grid generation returned no hypotheses");
  if (static_cast<int>(rots.size()) > I.max_hyp) rots.resize(static_cast<std::size_t>(I.max_hyp));
  I.rotation_count = static_cast<int>(rots.size());
  std::vector<float> flat;
  for (const Mat3f& r : rots) flat.insert(flat.end(), r.values.begin(), r.values.end());
  I.rotations.allocate(flat.size() * 4);
  checkCuda(cudaMemcpy(I.rotations.data(), flat.data(), flat.size() * 4, cudaMemcpyHostToDevice), "upload rotations");
}

FoundationPose::~FoundationPose() = default;
FoundationPose::FoundationPose(FoundationPose&&) noexcept = default;
FoundationPose& FoundationPose::operator=(FoundationPose&&) noexcept = default;

const PreprocessedMesh& FoundationPose::mesh() const { return impl_->mesh; }
const Config& FoundationPose::config() const { return impl_->cfg; }

FoundationPose FoundationPose::createFromCadFile(const std::filesystem::path& cad_path,
                                                 RuntimeOptions runtime_options, Config config) {
  Mesh mesh = loadMesh(cad_path);
  if (runtime_options.mesh_unit_scale != 1.0f) {
    for (Vec3f& v : mesh.vertices) v = v * runtime_options.mesh_unit_scale;
  }
  return FoundationPose(preprocessMesh(mesh, config), std::move(runtime_options), config);
}

FoundationPose FoundationPose::createFromReferenceImages(std::span<const ModelFreeReferenceView> refs,
                                                         RuntimeOptions runtime_options, Config config) {
  Mesh mesh = fpb_host::reconstructReferenceMesh(refs, config);
  return FoundationPose(preprocessMesh(mesh, config), std::move(runtime_options), config);
}

void FoundationPose::prepareForBatch(int batch_size) {
  if (batch_size <= 0 || batch_size > impl_->max_hyp) {
    throw FoundationPoseError("prepare batch size exceeds configured maximum");
  }
  impl_->inference->prepareForBatch(batch_size);
}

namespace {

// Active hypothesis count of a register call (reference foundation_pose.cpp:330-342 rules).
int activeHypotheses(const FoundationPose::Impl& I, int n_hypotheses) {
  int active = n_hypotheses > 0 ? std::min(n_hypotheses, I.rotation_count)
                                : std::min(I.cfg.n_hypotheses, I.rotation_count);
  active = std::min(active, I.max_hyp);
  if (active <= 0) throw FoundationPoseError("No active hypotheses available");
  return active;
}

// Micro-batch for refining n hypotheses, with the reference's divisibility
// and graph-capture rules.
int refineChunk(const FoundationPose::Impl& I, int n) {
  const int bs = I.cfg.batch_size > 0 ? I.cfg.batch_size : n;
  const int eff = std::min(n, bs);
  if (eff > 0 && n % eff != 0) {
    throw FoundationPoseError("active_hypotheses (" + std::to_string(n) +
                              ") must be divisible by batch_size (" + std::to_string(eff) + ")");
  }
  if (I.cfg.capture_cuda_graph && eff < n) {
    throw FoundationPoseError("capture_cuda_graph is not supported when batch_size (" + std::to_string(eff) +
                              ") < active_hypotheses (" + std::to_string(n) + ")");
  }
  return eff;
}

}  // namespace

void FoundationPose::registerShardBegin(const std::uint8_t* rgb_u8, const float* depth_m,
                                        const std::uint8_t* mask_u8, int width, int height,
                                        CameraIntrinsics intrinsics, int n_refine, int n_hypotheses,
                                        int shard_begin, int shard_count, float* features, float* poses) {
  Impl& I = *impl_;
  if (!I.fused) throw FoundationPoseError("sharded register requires the built-in renderer and networks");
  I.validateFrame(rgb_u8, depth_m, mask_u8, width, height, true);
  intrinsics = validateIntrinsics(intrinsics);
  if (features == nullptr || poses == nullptr) throw FoundationPoseError("shard outputs are required");
  const int iters = n_refine >= 0 ? n_refine : I.cfg.n_refine_iters;
  const int active = activeHypotheses(I, n_hypotheses);
  if (shard_begin < 0 || shard_count <= 0 || shard_begin + shard_count > active) {
    throw FoundationPoseError("shard [" + std::to_string(shard_begin) + ", " +
                              std::to_string(shard_begin + shard_count) + ") is outside the " +
                              std::to_string(active) + " active hypotheses");
  }
  // The reference's batch rules apply to the register as a whole (all active
  // hypotheses); a shard then refines in micro-batches of that size counted
  // from its own first hypothesis, the last one possibly shorter (a 63-
  // hypothesis shard of a batch-42 register runs 42 + 21).
  const int eff = std::min(refineChunk(I, active), shard_count);
  I.upload(rgb_u8, depth_m, mask_u8, width, height);
  fpkCheck(fpk_preprocess(I.depth_raw.as<float>(), I.mask.as<uint8_t>(), width, height, toK(intrinsics),
                          &I.params, I.depth_filtered.as<float>(), nullptr, nullptr, I.stats.as<int32_t>(), I.s()));
  // Seeding is deterministic, so every shard seeds all hypotheses and keeps its range.
  fpkCheck(fpk_seed_poses(I.stats.as<int32_t>(), I.rotations.as<float>(), active, toK(intrinsics), &I.params,
                          nullptr, I.seeded.as<float>(), I.s()));
  checkCuda(cudaMemcpyAsync(I.poses.data(), I.seeded.as<float>() + 16 * shard_begin,
                            static_cast<std::size_t>(shard_count) * 64, cudaMemcpyDeviceToDevice, I.s()),
            "cudaMemcpyAsync shard poses");
  I.active = shard_count;
  I.refinementLoop(iters, shard_count, eff, width, height, intrinsics);
  fpb::NetworkRunner& net = I.builtin_runner->net();
  const fpk_mesh_t m = meshView(I.dmesh);
  fpkCheck(fpk_render_pack(&m, I.poses.as<float>(), shard_count, I.rgb.as<uint8_t>(), I.depth_filtered.as<float>(),
                           width, height, toK(intrinsics), &I.params, I.mesh.diameter, 0.1f, net.dtype(),
                           net.stem().base, net.stem().plane_stride, I.boxes.as<float>(), I.render_ws.data(),
                           I.render_ws.bytes(), I.s()));
  runNet([&] { net.scoreFeatures(shard_count, features, I.s()); });
  checkCuda(cudaMemcpyAsync(poses, I.poses.data(), static_cast<std::size_t>(shard_count) * 64,
                            cudaMemcpyDeviceToDevice, I.s()),
            "cudaMemcpyAsync shard poses out");
  I.stream->synchronize();
  I.checkNetworkErrors();
}

PoseEstimate FoundationPose::registerShardFinish(const float* features, const float* poses, int n_hypotheses) {
  Impl& I = *impl_;
  if (!I.fused) throw FoundationPoseError("sharded register requires the built-in renderer and networks");
  if (features == nullptr || poses == nullptr) throw FoundationPoseError("gathered features and poses are required");
  if (n_hypotheses <= 0 || n_hypotheses > I.max_hyp) {
    throw FoundationPoseError("n_hypotheses must be in [1, " + std::to_string(I.max_hyp) + "]");
  }
  fpb::NetworkRunner& net = I.builtin_runner->net();
  runNet([&] { net.scoreHead(n_hypotheses, features, I.scores.as<float>(), I.s()); });
  const float center[3] = {I.mesh.center.x, I.mesh.center.y, I.mesh.center.z};
  fpkCheck(fpk_select_best(poses, I.scores.as<float>(), n_hypotheses, center, I.best.as<float>(), I.s()));
  PoseEstimate e = I.readBest();
  checkCuda(cudaMemcpyAsync(I.prev_pose.data(), poses + 16 * I.last_index, 64, cudaMemcpyDeviceToDevice, I.s()),
            "cudaMemcpyAsync previous pose");
  I.stream->synchronize();
  I.has_prev = true;
  return e;
}

PoseEstimate FoundationPose::registerFrame(const std::uint8_t* rgb_u8, const float* depth_m,
                                           const std::uint8_t* mask_u8, int width, int height,
                                           CameraIntrinsics intrinsics, int n_refine, int n_hypotheses) {
  Impl& I = *impl_;
  I.validateFrame(rgb_u8, depth_m, mask_u8, width, height, true);
  intrinsics = validateIntrinsics(intrinsics);
  const int iters = n_refine >= 0 ? n_refine : I.cfg.n_refine_iters;
  const int active = activeHypotheses(I, n_hypotheses);
  I.active = active;
  const int eff = refineChunk(I, active);
  I.upload(rgb_u8, depth_m, mask_u8, width, height);
  fpkCheck(fpk_preprocess(I.depth_raw.as<float>(), I.mask.as<uint8_t>(), width, height, toK(intrinsics),
                          &I.params, I.depth_filtered.as<float>(), nullptr, nullptr, I.stats.as<int32_t>(), I.s()));
  fpkCheck(fpk_seed_poses(I.stats.as<int32_t>(), I.rotations.as<float>(), active, toK(intrinsics), &I.params,
                          nullptr, I.poses.as<float>(), I.s()));
  I.refinementLoop(iters, active, eff, width, height, intrinsics);
  I.scorePass(active, width, height, intrinsics);
  const float center[3] = {I.mesh.center.x, I.mesh.center.y, I.mesh.center.z};
  fpkCheck(fpk_select_best(I.poses.as<float>(), I.scores.as<float>(), active, center, I.best.as<float>(), I.s()));
  PoseEstimate e = I.readBest();
  checkCuda(cudaMemcpyAsync(I.prev_pose.data(), I.poses.as<float>() + 16 * I.last_index, 64,
                            cudaMemcpyDeviceToDevice, I.s()),
            "cudaMemcpyAsync previous pose");
  I.has_prev = true;
  return e;
}

PoseEstimate FoundationPose::trackFrame(const std::uint8_t* rgb_u8, const float* depth_m, int width,
                                        int height, CameraIntrinsics intrinsics, int n_refine) {
  Impl& I = *impl_;
  I.validateFrame(rgb_u8, depth_m, nullptr, width, height, false);
  intrinsics = validateIntrinsics(intrinsics);
  if (!I.has_prev) throw FoundationPoseError("No previous pose. Call registerFrame before trackFrame.");
  const int iters = n_refine >= 0 ? n_refine : I.cfg.n_track_iters;
  I.upload(rgb_u8, depth_m, nullptr, width, height);
  I.trackCall(iters, width, height, intrinsics);
  return I.readBest();
}

}  // namespace foundation_pose_nvidia

// ---------------------------------------------------------------------------
// C ABI (reference src/c_api.cpp:262-542).
// ---------------------------------------------------------------------------

using foundation_pose_nvidia::CameraIntrinsics;
using foundation_pose_nvidia::Config;
using foundation_pose_nvidia::FoundationPose;
using foundation_pose_nvidia::FoundationPoseError;
using foundation_pose_nvidia::Mat4f;
using foundation_pose_nvidia::ModelFreeReferenceView;
using foundation_pose_nvidia::PoseEstimate;
using foundation_pose_nvidia::RuntimeOptions;
using foundation_pose_nvidia::TensorrtPrecision;

struct fp_handle {
  std::unique_ptr<FoundationPose> estimator;
};

namespace {

// The group's host side: one long-lived worker thread per object, bound to
// that object's device for its whole life (the estimator's stream, workspace
// and graphs live there). A group call gives every active worker one job and
// returns when all of them have finished, so a frame costs two condition-
// variable hand-offs per object instead of a thread start and join (the
// reference starts one std::jthread per object per call, c_api.cpp:203-237).
class GroupWorkers {
 public:
  explicit GroupWorkers(const std::vector<int>& devices) : slots_(devices.size()) {
    for (std::size_t i = 0; i < devices.size(); ++i) {
      slots_[i].thread = std::thread([this, i, dev = devices[i]] { loop(slots_[i], dev); });
    }
  }
  ~GroupWorkers() {
    for (Slot& w : slots_) {
      {
        std::lock_guard<std::mutex> lock(w.mu);
        w.stop = true;
      }
      w.cv.notify_one();
    }
    for (Slot& w : slots_) w.thread.join();
  }
  GroupWorkers(const GroupWorkers&) = delete;
  GroupWorkers& operator=(const GroupWorkers&) = delete;

  // Runs job(i) on worker i for every i with active[i]; errors[i] receives
  // the message of a job that threw ("" when it returned).
  void run(const std::vector<bool>& active, const std::function<void(std::size_t)>& job,
           std::vector<std::string>& errors) {
    std::ptrdiff_t n = 0;
    for (bool a : active) n += a ? 1 : 0;
    std::latch done(n);
    for (std::size_t i = 0; i < slots_.size(); ++i) {
      if (!active[i]) continue;
      Slot& w = slots_[i];
      {
        std::lock_guard<std::mutex> lock(w.mu);
        w.task = [&, i] {
          try {
            job(i);
          } catch (const std::exception& e) {
            errors[i] = e.what();
            if (errors[i].empty()) errors[i] = "unknown error";
          }
          done.count_down();
        };
      }
      w.cv.notify_one();
    }
    done.wait();
  }

 private:
  struct Slot {
    std::thread thread;
    std::mutex mu;
    std::condition_variable cv;
    std::function<void()> task;
    bool stop = false;
  };

  static void loop(Slot& w, int device) {
    // Bind once; a job re-selects (and reports) the device if this failed.
    if (cudaSetDevice(device) != cudaSuccess) cudaGetLastError();
    for (;;) {
      std::function<void()> task;
      {
        std::unique_lock<std::mutex> lock(w.mu);
        w.cv.wait(lock, [&] { return w.stop || static_cast<bool>(w.task); });
        if (!w.task) return;  // stop requested and nothing pending
        task = std::move(w.task);
        w.task = nullptr;
      }
      task();
    }
  }

  std::vector<Slot> slots_;
};

}  // namespace

struct fp_group {
  std::vector<std::unique_ptr<fp_handle>> handles;
  std::vector<int> device_ids;
  std::unique_ptr<GroupWorkers> workers;  // declared last: stopped before the handles go
};

static_assert(sizeof(fp_config_t) == 14 * 4, "fp_config_t layout");
static_assert(offsetof(fp_config_t, batch_size) == 13 * 4, "fp_config_t layout");
static_assert(sizeof(fp_pose_result_t) == 17 * 4, "fp_pose_result_t layout");
static_assert(offsetof(fp_create_options_t, mesh_unit_scale) == 12, "fp_create_options_t layout");
static_assert(sizeof(fp_create_options_t) == 96, "fp_create_options_t layout");
static_assert(sizeof(fp_image_view_t) == 40, "fp_image_view_t layout");
static_assert(sizeof(fp_reference_image_view_t) == 48, "fp_reference_image_view_t layout");

namespace {

void writeError(char* buf, size_t size, std::string_view msg) {
  if (buf == nullptr || size == 0) return;
  const size_t n = std::min(size - 1, msg.size());
  std::memcpy(buf, msg.data(), n);
  buf[n] = '\0';
}

// "<= 0 keeps the default", except the iteration counts (>= 0 accepted) and the
// flags, exactly as the reference's toConfig (src/c_api.cpp:58-117).
Config toConfig(const fp_config_t* in) {
  Config c;
  if (in == nullptr) return c;
  if (in->n_hypotheses > 0) c.n_hypotheses = in->n_hypotheses;
  if (in->n_refine_iters >= 0) c.n_refine_iters = in->n_refine_iters;
  if (in->n_track_iters >= 0) c.n_track_iters = in->n_track_iters;
  if (in->crop_ratio > 0.0f) c.crop_ratio = in->crop_ratio;
  if (in->input_width > 0) c.input_width = in->input_width;
  if (in->input_height > 0) c.input_height = in->input_height;
  if (in->max_image_width > 0) c.max_image_width = in->max_image_width;
  if (in->max_image_height > 0) c.max_image_height = in->max_image_height;
  c.capture_cuda_graph = in->capture_cuda_graph != 0;
  if (in->model_free_sample_stride > 0) c.model_free_sample_stride = in->model_free_sample_stride;
  if (in->model_free_max_vertices > 0) c.model_free_max_vertices = in->model_free_max_vertices;
  if (in->model_free_depth_edge_threshold > 0.0f) c.model_free_depth_edge_threshold = in->model_free_depth_edge_threshold;
  switch (in->tensorrt_precision) {
    case FP_PRECISION_TF32:
      c.tensorrt_precision = TensorrtPrecision::kTF32;
      break;
    case FP_PRECISION_FP16:
      c.tensorrt_precision = TensorrtPrecision::kFP16;
      break;
    case FP_PRECISION_BF16:
      c.tensorrt_precision = TensorrtPrecision::kBF16;
      break;
    default:
      c.tensorrt_precision = TensorrtPrecision::kFP32;
  }
  if (in->batch_size > 0) c.batch_size = in->batch_size;
  return c;
}

std::string strOrEmpty(const char* s) { return s == nullptr ? std::string{} : std::string(s); }

RuntimeOptions toOptions(const fp_create_options_t& in) {
  RuntimeOptions o;
  o.device_id = in.device_id;
  if (in.mesh_unit_scale > 0.0f) o.mesh_unit_scale = in.mesh_unit_scale;
  o.refine_model_path = strOrEmpty(in.refine_model_path);
  o.score_model_path = strOrEmpty(in.score_model_path);
  o.engine_cache_dir = strOrEmpty(in.engine_cache_dir);
  if (in.refine_model_name) o.refine_model_name = in.refine_model_name;
  if (in.score_model_name) o.score_model_name = in.score_model_name;
  if (in.rendered_input_name) o.rendered_input_name = in.rendered_input_name;
  if (in.observed_input_name) o.observed_input_name = in.observed_input_name;
  if (in.refine_translation_output_name) o.refine_translation_output_name = in.refine_translation_output_name;
  if (in.refine_rotation_output_name) o.refine_rotation_output_name = in.refine_rotation_output_name;
  if (in.score_output_name) o.score_output_name = in.score_output_name;
  return o;
}

CameraIntrinsics intrinsicsOf(const fp_image_view_t& v) {
  if (v.k_row_major == nullptr) throw FoundationPoseError("k_row_major is required");
  return CameraIntrinsics::fromRowMajor(v.k_row_major);
}

void writeResult(const PoseEstimate& e, fp_pose_result_t* r) {
  if (r == nullptr) return;
  for (int i = 0; i < 16; ++i) r->pose_row_major[i] = e.pose.values[static_cast<size_t>(i)];
  r->score = e.score;
}

// The C reference views (host buffers) as the estimator's view type; a NULL
// camera_to_world is the identity (reference c_api.cpp fp_create_model_free).
std::vector<ModelFreeReferenceView> referenceViews(const fp_reference_image_view_t* refs, size_t count) {
  std::vector<ModelFreeReferenceView> views(count);
  for (size_t i = 0; i < count; ++i) {
    const fp_reference_image_view_t& r = refs[i];
    if (r.k_row_major == nullptr) throw FoundationPoseError("Reference k_row_major is required");
    ModelFreeReferenceView& v = views[i];
    v.width = r.width;
    v.height = r.height;
    v.rgb_u8 = r.rgb_u8;
    v.depth_m = r.depth_m;
    v.mask_u8 = r.mask_u8;
    v.intrinsics = CameraIntrinsics::fromRowMajor(r.k_row_major);
    v.camera_to_world = Mat4f::identity();
    if (r.camera_to_world_row_major != nullptr) {
      std::copy(r.camera_to_world_row_major, r.camera_to_world_row_major + 16, v.camera_to_world.values.begin());
    }
  }
  return views;
}

// A group call over the objects not skipped: per-object statuses, the number
// of failures as the result and the first failure's message prefixed with its
// object index (reference c_api.cpp:203-258 behaviour).
int runGroup(fp_group* g, const std::vector<bool>& skip, fp_pose_result_t* results, int* statuses,
             char* err, size_t err_size, const std::function<PoseEstimate(FoundationPose&, size_t)>& eval) {
  const size_t n = g->handles.size();
  std::vector<bool> active(n);
  for (size_t i = 0; i < n; ++i) active[i] = !skip[i];
  std::vector<std::string> errors(n);
  std::vector<char> failed(n, 0);
  g->workers->run(active, [&](size_t i) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != g->device_ids[i]) {
      foundation_pose_nvidia::checkCuda(cudaSetDevice(g->device_ids[i]), "cudaSetDevice");
    }
    try {
      const PoseEstimate est = eval(*g->handles[i]->estimator, i);
      if (results != nullptr) writeResult(est, results + i);
    } catch (...) {
      failed[i] = 1;
      throw;
    }
  }, errors);
  int failures = 0;
  std::string first;
  for (size_t i = 0; i < n; ++i) {
    const int st = skip[i] ? FP_OBJECT_SKIPPED : (failed[i] ? FP_OBJECT_FAILED : FP_OBJECT_OK);
    if (statuses != nullptr) statuses[i] = st;
    if (st == FP_OBJECT_FAILED && failures++ == 0) first = std::format("object {}: {}", i, errors[i]);
  }
  writeError(err, err_size, first);
  return failures;
}

}  // namespace

extern "C" {

void fp_default_config(fp_config_t* config) {
  if (config == nullptr) return;
  const Config d;
  config->n_hypotheses = d.n_hypotheses;
  config->n_refine_iters = d.n_refine_iters;
  config->n_track_iters = d.n_track_iters;
  config->crop_ratio = d.crop_ratio;
  config->input_width = d.input_width;
  config->input_height = d.input_height;
  config->max_image_width = d.max_image_width;
  config->max_image_height = d.max_image_height;
  config->capture_cuda_graph = d.capture_cuda_graph ? 1 : 0;
  config->model_free_sample_stride = d.model_free_sample_stride;
  config->model_free_max_vertices = d.model_free_max_vertices;
  config->model_free_depth_edge_threshold = d.model_free_depth_edge_threshold;
  config->tensorrt_precision = static_cast<int>(d.tensorrt_precision);
  config->batch_size = d.batch_size;
}

fp_handle_t* fp_create(const fp_create_options_t* options, const fp_config_t* config, char* err,
                       size_t err_size) {
  try {
    if (options == nullptr || options->cad_path == nullptr) throw FoundationPoseError("cad_path is required");
    auto h = std::make_unique<fp_handle>();
    h->estimator = std::make_unique<FoundationPose>(
        FoundationPose::createFromCadFile(options->cad_path, toOptions(*options), toConfig(config)));
    writeError(err, err_size, "");
    return h.release();
  } catch (const std::exception& e) {
    writeError(err, err_size, e.what());
    return nullptr;
  }
}

fp_handle_t* fp_create_model_free(const fp_reference_image_view_t* refs, size_t count,
                                  const fp_create_options_t* options, const fp_config_t* config,
                                  char* err, size_t err_size) {
  try {
    if (refs == nullptr || count == 0) throw FoundationPoseError("At least one model-free reference image is required");
    if (options == nullptr) throw FoundationPoseError("create options are required");
    const std::vector<ModelFreeReferenceView> views = referenceViews(refs, count);
    auto h = std::make_unique<fp_handle>();
    h->estimator = std::make_unique<FoundationPose>(
        FoundationPose::createFromReferenceImages(views, toOptions(*options), toConfig(config)));
    writeError(err, err_size, "");
    return h.release();
  } catch (const std::exception& e) {
    writeError(err, err_size, e.what());
    return nullptr;
  }
}

int fp_prepare(fp_handle_t* handle, int batch_size, char* err, size_t err_size) {
  try {
    if (handle == nullptr || !handle->estimator) throw FoundationPoseError("Invalid handle");
    handle->estimator->prepareForBatch(batch_size);
    writeError(err, err_size, "");
    return 0;
  } catch (const std::exception& e) {
    writeError(err, err_size, e.what());
    return 1;
  }
}

void fp_destroy(fp_handle_t* handle) { delete handle; }

int fp_register_frame(fp_handle_t* handle, const fp_image_view_t* image, int n_refine, int n_hypotheses,
                      fp_pose_result_t* result, char* err, size_t err_size) {
  try {
    if (handle == nullptr || !handle->estimator || image == nullptr) throw FoundationPoseError("Invalid handle or image");
    writeResult(handle->estimator->registerFrame(image->rgb_u8, image->depth_m, image->mask_u8, image->width,
                                                 image->height, intrinsicsOf(*image), n_refine, n_hypotheses),
                result);
    writeError(err, err_size, "");
    return 0;
  } catch (const std::exception& e) {
    writeError(err, err_size, e.what());
    return 1;
  }
}

int fp_register_shard_begin(fp_handle_t* handle, const fp_image_view_t* image, int n_refine, int n_hypotheses,
                            int shard_begin, int shard_count, float* features, float* poses, char* err,
                            size_t err_size) {
  try {
    if (handle == nullptr || !handle->estimator || image == nullptr) throw FoundationPoseError("Invalid handle or image");
    handle->estimator->registerShardBegin(image->rgb_u8, image->depth_m, image->mask_u8, image->width,
                                          image->height, intrinsicsOf(*image), n_refine, n_hypotheses,
                                          shard_begin, shard_count, features, poses);
    writeError(err, err_size, "");
    return 0;
  } catch (const std::exception& e) {
    writeError(err, err_size, e.what());
    return 1;
  }
}

int fp_register_shard_finish(fp_handle_t* handle, const float* features, const float* poses, int n_hypotheses,
                             fp_pose_result_t* result, char* err, size_t err_size) {
  try {
    if (handle == nullptr || !handle->estimator) throw FoundationPoseError("Invalid handle");
    writeResult(handle->estimator->registerShardFinish(features, poses, n_hypotheses), result);
    writeError(err, err_size, "");
    return 0;
  } catch (const std::exception& e) {
    writeError(err, err_size, e.what());
    return 1;
  }
}

int fp_track_frame(fp_handle_t* handle, const fp_image_view_t* image, int n_refine, fp_pose_result_t* result,
                   char* err, size_t err_size) {
  try {
    if (handle == nullptr || !handle->estimator || image == nullptr) throw FoundationPoseError("Invalid handle or image");
    writeResult(handle->estimator->trackFrame(image->rgb_u8, image->depth_m, image->width, image->height,
                                              intrinsicsOf(*image), n_refine),
                result);
    writeError(err, err_size, "");
    return 0;
  } catch (const std::exception& e) {
    writeError(err, err_size, e.what());
    return 1;
  }
}

fp_group_t* fp_group_create(const fp_create_options_t* objects, size_t count, const fp_config_t* config,
                            char* err, size_t err_size) {
  try {
    if (objects == nullptr || count == 0) throw FoundationPoseError("At least one object is required");
    auto g = std::make_unique<fp_group>();
    for (size_t i = 0; i < count; ++i) {
      if (objects[i].cad_path == nullptr) throw FoundationPoseError(std::format("object {}: cad_path is required", i));
      auto h = std::make_unique<fp_handle>();
      h->estimator = std::make_unique<FoundationPose>(
          FoundationPose::createFromCadFile(objects[i].cad_path, toOptions(objects[i]), toConfig(config)));
      g->handles.push_back(std::move(h));
      g->device_ids.push_back(objects[i].device_id);
    }
    g->workers = std::make_unique<GroupWorkers>(g->device_ids);
    writeError(err, err_size, "");
    return g.release();
  } catch (const std::exception& e) {
    writeError(err, err_size, e.what());
    return nullptr;
  }
}

size_t fp_group_size(const fp_group_t* group) { return group == nullptr ? 0 : group->handles.size(); }

fp_handle_t* fp_group_handle(fp_group_t* group, size_t index) {
  if (group == nullptr || index >= group->handles.size()) return nullptr;
  return group->handles[index].get();
}

int fp_group_prepare(fp_group_t* group, int batch_size, char* err, size_t err_size) {
  if (group == nullptr) {
    writeError(err, err_size, "Invalid group");
    return 1;
  }
  const std::vector<bool> skip(group->handles.size(), false);
  return runGroup(group, skip, nullptr, nullptr, err, err_size, [batch_size](FoundationPose& e, size_t) {
    e.prepareForBatch(batch_size);
    return PoseEstimate{};
  });
}

int fp_group_register_frame(fp_group_t* group, const fp_image_view_t* image, const uint8_t* const* masks,
                            int n_refine, int n_hypotheses, fp_pose_result_t* results, int* statuses,
                            char* err, size_t err_size) {
  try {
    if (group == nullptr || image == nullptr || masks == nullptr || results == nullptr) {
      throw FoundationPoseError("Invalid group, image, masks, or results");
    }
    const CameraIntrinsics k = intrinsicsOf(*image);
    std::vector<bool> skip(group->handles.size());
    for (size_t i = 0; i < skip.size(); ++i) skip[i] = masks[i] == nullptr;
    return runGroup(group, skip, results, statuses, err, err_size,
                    [image, masks, k, n_refine, n_hypotheses](FoundationPose& e, size_t i) {
                      return e.registerFrame(image->rgb_u8, image->depth_m, masks[i], image->width,
                                             image->height, k, n_refine, n_hypotheses);
                    });
  } catch (const std::exception& e) {
    writeError(err, err_size, e.what());
    return group == nullptr ? 1 : static_cast<int>(group->handles.size());
  }
}

int fp_group_track_frame(fp_group_t* group, const fp_image_view_t* image, const int* active, int n_refine,
                         fp_pose_result_t* results, int* statuses, char* err, size_t err_size) {
  try {
    if (group == nullptr || image == nullptr || results == nullptr) {
      throw FoundationPoseError("Invalid group, image, or results");
    }
    const CameraIntrinsics k = intrinsicsOf(*image);
    std::vector<bool> skip(group->handles.size());
    for (size_t i = 0; i < skip.size(); ++i) skip[i] = active != nullptr && active[i] == 0;
    return runGroup(group, skip, results, statuses, err, err_size, [image, k, n_refine](FoundationPose& e, size_t) {
      return e.trackFrame(image->rgb_u8, image->depth_m, image->width, image->height, k, n_refine);
    });
  } catch (const std::exception& e) {
    writeError(err, err_size, e.what());
    return group == nullptr ? 1 : static_cast<int>(group->handles.size());
  }
}

void fp_group_destroy(fp_group_t* group) { delete group; }

int fp_synchronize_device(char* err, size_t err_size) {
  try {
    const cudaError_t s = cudaDeviceSynchronize();
    if (s != cudaSuccess) throw FoundationPoseError(cudaGetErrorString(s));
    writeError(err, err_size, "");
    return 0;
  } catch (const std::exception& e) {
    writeError(err, err_size, e.what());
    return 1;
  }
}

int fpk_model_free_mesh(const fp_reference_image_view_t* refs, size_t count, const fp_config_t* config,
                        int* n_vertices, int* n_faces, float* vertices, uint8_t* colors, float* normals,
                        int32_t* faces) {
  try {
    if (refs == nullptr || count == 0) throw FoundationPoseError("At least one model-free reference image is required");
    if (n_vertices == nullptr || n_faces == nullptr) throw FoundationPoseError("fpk_model_free_mesh: count outputs are required");
    const std::vector<ModelFreeReferenceView> views = referenceViews(refs, count);
    const foundation_pose_nvidia::Mesh m = foundation_pose_nvidia::fpb_host::reconstructReferenceMesh(views, toConfig(config));
    *n_vertices = static_cast<int>(m.vertices.size());
    *n_faces = static_cast<int>(m.faces.size());
    for (size_t i = 0; i < m.vertices.size(); ++i) {
      if (vertices != nullptr) {
        vertices[3 * i] = m.vertices[i].x;
        vertices[3 * i + 1] = m.vertices[i].y;
        vertices[3 * i + 2] = m.vertices[i].z;
      }
      if (colors != nullptr) {
        colors[3 * i] = m.vertex_colors[i].r;
        colors[3 * i + 1] = m.vertex_colors[i].g;
        colors[3 * i + 2] = m.vertex_colors[i].b;
      }
      if (normals != nullptr) {
        normals[3 * i] = m.normals[i].x;
        normals[3 * i + 1] = m.normals[i].y;
        normals[3 * i + 2] = m.normals[i].z;
      }
    }
    if (faces != nullptr) {
      for (size_t i = 0; i < m.faces.size(); ++i)
        for (int k = 0; k < 3; ++k) faces[3 * i + k] = static_cast<int32_t>(m.faces[i][k]);
    }
    return 0;
  } catch (const std::exception& e) {
    return fpb::fail(e.what());
  }
}

const char* fp_build_info(void) {
  return "foundation-pose B200 runtime (sm_100a: fused raster/pack, tcgen05 RefineNet/ScoreNet FP16/BF16)";
}

}  // extern "C"
