// Model-free object mesh from reference RGB-D views, built on the GPU.
//
// Replaces the reference's CPU reconstruction behind
// FoundationPose::createFromReferenceImages (src/foundation_pose.cpp:91-182,
// 296-300); the result is the same mesh, vertex for vertex and face for face:
//   * every stride-th pixel of each view (stride from the configuration and
//     the vertex budget) whose mask is set and whose depth is valid becomes a
//     vertex, back-projected with the view's intrinsics and moved to the world
//     frame by its camera_to_world pose; vertices are numbered in view order,
//     then row-major sample order, until the budget is spent;
//   * every 2 x 2 cell of a view's sample lattice contributes up to two
//     triangles (upper-left and lower-right halves) whose three corners are
//     vertices of that view with depths within the edge threshold of each other.
// Here each view is one pass of three small kernels: a lattice kernel marks
// valid samples and candidate triangles, a single-CTA scan turns the marks
// into vertex and face numbers (in the order above), and an emit kernel
// writes the vertices, colours and faces at those numbers. Positions use
// separately rounded multiplies and adds (no FMA contraction) and an IEEE
// division, which is how the reference's host build evaluates them.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <span>
#include <string>
#include <vector>

#include "foundation_pose_nvidia/device_buffer.hpp"
#include "foundation_pose_nvidia/foundation_pose.hpp"
#include "fp_host.hpp"

namespace foundation_pose_nvidia {
namespace fpb_host {
namespace {

constexpr int kScanThreads = 1024;

struct ViewGeom {
  int width, height, stride;
  int gw, gh;  // sample lattice: x = gx * stride < width, y = gy * stride < height
  float fx, fy, cx, cy;
  float m[12];  // camera_to_world rows 0-2
  float depth_min, depth_max, edge;
};

__device__ __forceinline__ bool validZ(float z, const ViewGeom& g) {
  return isfinite(z) && z >= g.depth_min && z < g.depth_max;
}

// Marks: sample_flag[s] = 1 for a masked, valid-depth lattice sample;
// sample_z[s] its depth.
__global__ void latticeKernel(const float* __restrict__ depth, const uint8_t* __restrict__ mask, ViewGeom g,
                              int* __restrict__ sample_flag, float* __restrict__ sample_z) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= g.gw * g.gh) return;
  const int gy = s / g.gw;
  const int gx = s - gy * g.gw;
  const size_t px = static_cast<size_t>(gy * g.stride) * g.width + gx * g.stride;
  const float z = depth[px];
  const bool ok = mask[px] != 0 && validZ(z, g);
  sample_flag[s] = ok ? 1 : 0;
  sample_z[s] = z;
}

// Exclusive scan of n flags by one CTA, in chunks of kScanThreads: index[i] =
// base + number of set flags before i when flag i is set and that number is
// below `cap - base`, else -1. count_out receives the number kept.
__global__ void __launch_bounds__(kScanThreads) scanKernel(const int* __restrict__ flags, int n, int base, int cap,
                                                           int* __restrict__ index, int* __restrict__ count_out) {
  __shared__ int warp_tot[kScanThreads / 32];
  __shared__ int carry;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  if (tid == 0) carry = 0;
  __syncthreads();
  for (int c0 = 0; c0 < n; c0 += kScanThreads) {
    const int i = c0 + tid;
    const int f = i < n ? flags[i] : 0;
    int incl = f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int t = warp_tot[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, t, o);
        if (lane >= o) t += v;
      }
      warp_tot[lane] = t;  // inclusive over warps
    }
    __syncthreads();
    const int before = carry + (warp > 0 ? warp_tot[warp - 1] : 0) + incl - f;
    if (i < n) index[i] = (f != 0 && base + before < cap) ? base + before : -1;
    __syncthreads();
    if (tid == kScanThreads - 1) carry += warp_tot[31];
    __syncthreads();
  }
  if (tid == 0) *count_out = min(carry, max(cap - base, 0));
}

__device__ __forceinline__ float affineRow(const float* r, float x, float y, float z) {
  // ((r0 x + r1 y) + r2 z) + r3 with every product and sum rounded on its own.
  return __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(r[0], x), __fmul_rn(r[1], y)), __fmul_rn(r[2], z)), r[3]);
}

// Vertices of the kept samples, and the candidate-triangle flags of every
// lattice cell (two per cell: corners (a, b, c) and (b, d, c)).
__global__ void emitVerticesKernel(const uint8_t* __restrict__ rgb, ViewGeom g, const int* __restrict__ vindex,
                                   const float* __restrict__ sample_z, float* __restrict__ verts,
                                   uint8_t* __restrict__ colors, int* __restrict__ face_flag) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= g.gw * g.gh) return;
  const int gy = s / g.gw;
  const int gx = s - gy * g.gw;
  const int v = vindex[s];
  if (v >= 0) {
    const int x = gx * g.stride;
    const int y = gy * g.stride;
    const float z = sample_z[s];
    const float px = __fdiv_rn(__fmul_rn(__fsub_rn(static_cast<float>(x), g.cx), z), g.fx);
    const float py = __fdiv_rn(__fmul_rn(__fsub_rn(static_cast<float>(y), g.cy), z), g.fy);
    verts[3 * v + 0] = affineRow(g.m + 0, px, py, z);
    verts[3 * v + 1] = affineRow(g.m + 4, px, py, z);
    verts[3 * v + 2] = affineRow(g.m + 8, px, py, z);
    const size_t p = (static_cast<size_t>(y) * g.width + x) * 3;
    colors[3 * v + 0] = rgb[p];
    colors[3 * v + 1] = rgb[p + 1];
    colors[3 * v + 2] = rgb[p + 2];
  }
  if (gx + 1 < g.gw && gy + 1 < g.gh) {
    const int cells_w = g.gw - 1;
    const int cell = gy * cells_w + gx;
    const int sa = s, sb = s + 1, sc = s + g.gw, sd = s + g.gw + 1;
    const int a = v, b = vindex[sb], c = vindex[sc], d = vindex[sd];
    const float za = sample_z[sa], zb = sample_z[sb], zc = sample_z[sc], zd = sample_z[sd];
    auto smooth = [&](float p, float q, float r) {
      return fabsf(p - q) <= g.edge && fabsf(p - r) <= g.edge && fabsf(q - r) <= g.edge;
    };
    face_flag[2 * cell + 0] = (a >= 0 && b >= 0 && c >= 0 && smooth(za, zb, zc)) ? 1 : 0;
    face_flag[2 * cell + 1] = (b >= 0 && d >= 0 && c >= 0 && smooth(zb, zd, zc)) ? 1 : 0;
  }
}

__global__ void emitFacesKernel(ViewGeom g, const int* __restrict__ vindex, const int* __restrict__ findex,
                                int32_t* __restrict__ faces) {
  const int cell = blockIdx.x * blockDim.x + threadIdx.x;
  const int cells_w = g.gw - 1;
  if (cells_w <= 0 || cell >= cells_w * (g.gh - 1)) return;
  const int cy = cell / cells_w;
  const int cx = cell - cy * cells_w;
  const int s = cy * g.gw + cx;
  const int a = vindex[s], b = vindex[s + 1], c = vindex[s + g.gw], d = vindex[s + g.gw + 1];
  const int f0 = findex[2 * cell], f1 = findex[2 * cell + 1];
  if (f0 >= 0) {
    faces[3 * f0 + 0] = a;
    faces[3 * f0 + 1] = b;
    faces[3 * f0 + 2] = c;
  }
  if (f1 >= 0) {
    faces[3 * f1 + 0] = b;
    faces[3 * f1 + 1] = d;
    faces[3 * f1 + 2] = c;
  }
}

void cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw FoundationPoseError(std::string("model-free reconstruction: ") + what + ": " +
                                                  cudaGetErrorString(e));
}

}  // namespace

Mesh reconstructReferenceMesh(std::span<const ModelFreeReferenceView> refs, const Config& config) {
  if (static_cast<int>(refs.size()) < config.model_free_min_reference_images) {
    throw FoundationPoseError("Model-free mode requires at least one reference image");
  }
  std::size_t total_px = 0, max_px = 0;
  for (const ModelFreeReferenceView& r : refs) {
    if (r.intrinsics.fx <= 0.0f || r.intrinsics.fy <= 0.0f) {
      throw FoundationPoseError("Camera intrinsics must have positive focal lengths");
    }
    if (r.width <= 0 || r.height <= 0 || r.rgb_u8 == nullptr || r.depth_m == nullptr || r.mask_u8 == nullptr) {
      throw FoundationPoseError("Each model-free reference needs RGB, depth, mask, and dimensions");
    }
    const std::size_t px = static_cast<std::size_t>(r.width) * r.height;
    total_px += px;
    max_px = std::max(max_px, px);
  }
  // Sampling stride: the configured one, widened so that all views together
  // offer about the vertex budget (reference foundation_pose.cpp:106-110).
  const int budget = std::max(config.model_free_max_vertices, 4);
  const int wide = std::max(1, static_cast<int>(std::ceil(std::sqrt(static_cast<double>(total_px) / budget))));
  const int stride = std::max(config.model_free_sample_stride, wide);

  std::size_t max_samples = 0;
  for (const ModelFreeReferenceView& r : refs) {
    max_samples = std::max(max_samples, static_cast<std::size_t>((r.width + stride - 1) / stride) *
                                            ((r.height + stride - 1) / stride));
  }
  cudaStream_t s = nullptr;
  cuda(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "stream");
  struct StreamGuard {
    cudaStream_t s;
    ~StreamGuard() { cudaStreamDestroy(s); }
  } guard{s};
  DeviceBuffer d_depth(max_px * 4), d_mask(max_px), d_rgb(max_px * 3);
  DeviceBuffer d_flag(max_samples * 4), d_z(max_samples * 4), d_vidx(max_samples * 4);
  DeviceBuffer d_fflag(max_samples * 8), d_fidx(max_samples * 8), d_count(16);
  DeviceBuffer d_verts(static_cast<std::size_t>(budget) * 12), d_colors(static_cast<std::size_t>(budget) * 3);
  std::vector<int32_t> faces;
  int n_verts = 0;
  for (const ModelFreeReferenceView& r : refs) {
    const std::size_t px = static_cast<std::size_t>(r.width) * r.height;
    cuda(cudaMemcpyAsync(d_depth.data(), r.depth_m, px * 4, cudaMemcpyDefault, s), "depth upload");
    cuda(cudaMemcpyAsync(d_mask.data(), r.mask_u8, px, cudaMemcpyDefault, s), "mask upload");
    cuda(cudaMemcpyAsync(d_rgb.data(), r.rgb_u8, px * 3, cudaMemcpyDefault, s), "rgb upload");
    ViewGeom g{};
    g.width = r.width;
    g.height = r.height;
    g.stride = stride;
    g.gw = (r.width + stride - 1) / stride;
    g.gh = (r.height + stride - 1) / stride;
    g.fx = r.intrinsics.fx;
    g.fy = r.intrinsics.fy;
    g.cx = r.intrinsics.cx;
    g.cy = r.intrinsics.cy;
    for (int i = 0; i < 12; ++i) g.m[i] = r.camera_to_world.values[static_cast<std::size_t>(i)];
    g.depth_min = config.depth_min;
    g.depth_max = config.depth_max;
    g.edge = config.model_free_depth_edge_threshold;
    const int samples = g.gw * g.gh;
    const int cells = std::max(0, g.gw - 1) * std::max(0, g.gh - 1);
    const int blocks = (samples + 255) / 256;
    latticeKernel<<<blocks, 256, 0, s>>>(d_depth.as<float>(), d_mask.as<std::uint8_t>(), g, d_flag.as<int>(),
                                        d_z.as<float>());
    scanKernel<<<1, kScanThreads, 0, s>>>(d_flag.as<int>(), samples, n_verts, budget, d_vidx.as<int>(),
                                          d_count.as<int>());
    emitVerticesKernel<<<blocks, 256, 0, s>>>(d_rgb.as<std::uint8_t>(), g, d_vidx.as<int>(), d_z.as<float>(),
                                              d_verts.as<float>(), d_colors.as<std::uint8_t>(), d_fflag.as<int>());
    const int base_f = static_cast<int>(faces.size() / 3);
    scanKernel<<<1, kScanThreads, 0, s>>>(d_fflag.as<int>(), 2 * cells, base_f, INT32_MAX, d_fidx.as<int>(),
                                          d_count.as<int>() + 1);
    cuda(cudaGetLastError(), "kernel launch");
    int counts[2] = {0, 0};
    cuda(cudaMemcpyAsync(counts, d_count.data(), sizeof(counts), cudaMemcpyDeviceToHost, s), "counts");
    cuda(cudaStreamSynchronize(s), "sync");
    n_verts += counts[0];
    if (counts[1] > 0) {
      DeviceBuffer d_faces(static_cast<std::size_t>(base_f + counts[1]) * 12);
      emitFacesKernel<<<(cells + 255) / 256, 256, 0, s>>>(g, d_vidx.as<int>(), d_fidx.as<int>(),
                                                          d_faces.as<int32_t>());
      cuda(cudaGetLastError(), "face kernel launch");
      faces.resize(static_cast<std::size_t>(base_f + counts[1]) * 3);
      cuda(cudaMemcpyAsync(faces.data() + static_cast<std::size_t>(base_f) * 3,
                           d_faces.as<int32_t>() + static_cast<std::size_t>(base_f) * 3,
                           static_cast<std::size_t>(counts[1]) * 12, cudaMemcpyDeviceToHost, s),
           "faces download");
      cuda(cudaStreamSynchronize(s), "sync");
    }
  }
  Mesh mesh;
  mesh.source_path = "model_free_references";
  std::vector<float> v(static_cast<std::size_t>(n_verts) * 3);
  std::vector<std::uint8_t> c(static_cast<std::size_t>(n_verts) * 3);
  if (n_verts > 0) {
    cuda(cudaMemcpy(v.data(), d_verts.data(), v.size() * 4, cudaMemcpyDeviceToHost), "vertex download");
    cuda(cudaMemcpy(c.data(), d_colors.data(), c.size(), cudaMemcpyDeviceToHost), "colour download");
  }
  mesh.vertices.resize(static_cast<std::size_t>(n_verts));
  mesh.vertex_colors.resize(static_cast<std::size_t>(n_verts));
  for (int i = 0; i < n_verts; ++i) {
    mesh.vertices[i] = Vec3f{v[3 * i], v[3 * i + 1], v[3 * i + 2]};
    mesh.vertex_colors[i] = Vec3u8{c[3 * i], c[3 * i + 1], c[3 * i + 2]};
  }
  mesh.faces.resize(faces.size() / 3);
  for (std::size_t i = 0; i < mesh.faces.size(); ++i) {
    mesh.faces[i] = {static_cast<std::uint32_t>(faces[3 * i]), static_cast<std::uint32_t>(faces[3 * i + 1]),
                     static_cast<std::uint32_t>(faces[3 * i + 2])};
  }
  if (mesh.vertices.size() < 4 || mesh.faces.empty()) {
    throw FoundationPoseError("Model-free reconstruction produced too little geometry; check masks and depth");
  }
  computeVertexNormals(mesh);
  return mesh;
}

}  // namespace fpb_host
}  // namespace foundation_pose_nvidia
