// sm_100a pipeline kernels of the render-and-compare hot path, exported through
// the fpk_* C ABI (include/fpk.h).
//
//  * fpk_preprocess   one tiled pass: erode -> bilateral -> (xyz) -> mask stats
//  * fpk_seed_poses   parallel histogram-median + pose seeding (one CTA)
//  * fpk_render[_pack] vertex pass (crop box, clip and pixel position per
//                     (hypothesis, vertex), z-buffer clear), one raster thread
//                     per (hypothesis, triangle) with 64-bit depth keys in an
//                     L2-resident z-buffer, warp-per-triangle pass for large
//                     triangles, then per-pixel resolve + shade and (fused
//                     variant) crop-warp + pack straight into the network's
//                     input layout
//  * fpk_apply_deltas / fpk_select_best  pose update and arg-max
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <atomic>
#include <cstdint>
#include <cstdio>
#include <string>
#include <type_traits>

#include "fp_device.cuh"
#include "fp_launch.hpp"
#include "fp_tc.cuh"
#include "fp_profile.hpp"
#include "fpk.h"

namespace fpb {

thread_local std::string g_fpk_error;

int fail(const std::string& msg) {
  g_fpk_error = msg;
  return 1;
}

int checkLaunch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return fail(std::string(what) + ": " + cudaGetErrorString(e));
  }
  return 0;
}

// ---------------------------------------------------------------------------
// Preprocess: erode -> bilateral -> xyz -> statistics, one frame pass.
// ---------------------------------------------------------------------------

constexpr int kPreTileW = 32;
constexpr int kPreTileH = 16;
constexpr int kMaxRadius = 4;
constexpr int kMaxHalo = 2 * kMaxRadius;
constexpr int kHistBins = 65536;

// Statistics layout in the int32 scratch: [0] max(INT_MAX - x) over mask
// pixels, [1] max(x + 1), [2] max(INT_MAX - y), [3] max(y + 1), [4] count of
// valid masked depths, [8 .. 8+65536) depth histogram. All updates are
// order-independent integer atomics, so the result is deterministic.
__global__ void __launch_bounds__(256) preprocessKernel(const float* __restrict__ depth_raw,
                                                        const uint8_t* __restrict__ mask,
                                                        int width, int height, fpk_intrinsics_t k,
                                                        fpk_params_t p,
                                                        float* __restrict__ depth_filtered,
                                                        float* __restrict__ eroded_out,
                                                        float* __restrict__ xyz_out,
                                                        int32_t* __restrict__ stats) {
  __shared__ float raw[kPreTileH + 2 * kMaxHalo][kPreTileW + 2 * kMaxHalo];
  __shared__ float ero[kPreTileH + 2 * kMaxRadius][kPreTileW + 2 * kMaxRadius];
  const int er = p.erosion_radius;
  const int br = p.bilateral_radius;
  const int halo = er + br;
  const int x0 = blockIdx.x * kPreTileW;
  const int y0 = blockIdx.y * kPreTileH;
  const int tid = threadIdx.y * blockDim.x + threadIdx.x;

  // Stage the raw depth tile with its halo (out-of-image cells are never read:
  // every stencil below clamps its window to the image like the reference).
  const int rw = kPreTileW + 2 * halo;
  const int rh = kPreTileH + 2 * halo;
  for (int i = tid; i < rw * rh; i += 256) {
    const int ly = i / rw;
    const int lx = i - ly * rw;
    const int gy = y0 - halo + ly;
    const int gx = x0 - halo + lx;
    float v = 0.0f;
    if (gx >= 0 && gy >= 0 && gx < width && gy < height) {
      v = __ldg(depth_raw + gy * width + gx);
    }
    raw[ly][lx] = v;
  }
  __syncthreads();

  // Erode the tile + bilateral halo (reference cuda_pipeline.cu:87-120).
  const int ew = kPreTileW + 2 * br;
  const int eh = kPreTileH + 2 * br;
  for (int i = tid; i < ew * eh; i += 256) {
    const int ly = i / ew;
    const int lx = i - ly * ew;
    const int y = y0 - br + ly;
    const int x = x0 - br + lx;
    if (x < 0 || y < 0 || x >= width || y >= height) {
      ero[ly][lx] = 0.0f;
      continue;
    }
    const float center = raw[ly + er][lx + er];
    float out = center;
    if (!validDepth(center, p.depth_min, p.depth_max)) {
      out = 0.0f;
    } else {
      int bad = 0;
      int total = 0;
      for (int yy = max(0, y - er); yy <= min(height - 1, y + er); ++yy) {
        for (int xx = max(0, x - er); xx <= min(width - 1, x + er); ++xx) {
          const float z = raw[yy - (y0 - halo)][xx - (x0 - halo)];
          ++total;
          if (!validDepth(z, p.depth_min, p.depth_max) ||
              fabsf(z - center) > p.depth_diff_threshold) {
            ++bad;
          }
        }
      }
      out = (total > 0 && static_cast<float>(bad) / static_cast<float>(total) >
                              p.erosion_ratio_threshold)
                ? 0.0f
                : center;
    }
    ero[ly][lx] = out;
  }
  __syncthreads();

  // Bilateral (reference cuda_pipeline.cu:122-171), xyz (:173-192), statistics.
  const float sigma_d2 = 2.0f * p.bilateral_sigma_d * p.bilateral_sigma_d;
  const float sigma_r2 = 2.0f * p.bilateral_sigma_r * p.bilateral_sigma_r;
  int s_minx = 0, s_maxx = 0, s_miny = 0, s_maxy = 0, s_count = 0;
  for (int i = tid; i < kPreTileW * kPreTileH; i += 256) {
    const int ly = i / kPreTileW;
    const int lx = i - ly * kPreTileW;
    const int y = y0 + ly;
    const int x = x0 + lx;
    if (x >= width || y >= height) {
      continue;
    }
    float mean = 0.0f;
    int valid = 0;
    for (int yy = max(0, y - br); yy <= min(height - 1, y + br); ++yy) {
      for (int xx = max(0, x - br); xx <= min(width - 1, x + br); ++xx) {
        const float z = ero[yy - (y0 - br)][xx - (x0 - br)];
        if (validDepth(z, p.depth_min, p.depth_max)) {
          mean += z;
          ++valid;
        }
      }
    }
    float result = 0.0f;
    if (valid != 0) {
      mean /= static_cast<float>(valid);
      float weighted = 0.0f;
      float weight_sum = 0.0f;
      for (int yy = max(0, y - br); yy <= min(height - 1, y + br); ++yy) {
        for (int xx = max(0, x - br); xx <= min(width - 1, x + br); ++xx) {
          const float z = ero[yy - (y0 - br)][xx - (x0 - br)];
          if (!validDepth(z, p.depth_min, p.depth_max)) {
            continue;
          }
          const float dx = static_cast<float>(xx - x);
          const float dy = static_cast<float>(yy - y);
          const float range = z - mean;
          const float w = expf(-(dx * dx + dy * dy) / sigma_d2) * expf(-(range * range) / sigma_r2);
          weighted += w * z;
          weight_sum += w;
        }
      }
      result = weight_sum > 0.0f ? weighted / weight_sum : 0.0f;
    }
    const int idx = y * width + x;
    depth_filtered[idx] = result;
    if (eroded_out != nullptr) {
      eroded_out[idx] = ero[ly + br][lx + br];
    }
    const bool dvalid = validDepth(result, p.depth_min, p.depth_max);
    if (xyz_out != nullptr) {
      float3 v = make_float3(0.0f, 0.0f, 0.0f);
      if (dvalid) {
        v = make_float3((static_cast<float>(x) - k.cx) * result / k.fx,
                        (static_cast<float>(y) - k.cy) * result / k.fy, result);
      }
      xyz_out[3 * idx + 0] = v.x;
      xyz_out[3 * idx + 1] = v.y;
      xyz_out[3 * idx + 2] = v.z;
    }
    if (mask != nullptr && __ldg(mask + idx) != 0) {
      s_minx = max(s_minx, INT_MAX - x);
      s_maxx = max(s_maxx, x + 1);
      s_miny = max(s_miny, INT_MAX - y);
      s_maxy = max(s_maxy, y + 1);
      if (dvalid) {
        ++s_count;
        // reference cuda_pipeline.cu:295-298
        const float normalized = (result - p.depth_min) / (p.depth_max - p.depth_min);
        const int bin = min(max(static_cast<int>(normalized * kHistBins), 0), kHistBins - 1);
        atomicAdd(stats + 8 + bin, 1);
      }
    }
  }
  if (mask != nullptr) {
    s_minx = __reduce_max_sync(0xffffffffu, s_minx);
    s_maxx = __reduce_max_sync(0xffffffffu, s_maxx);
    s_miny = __reduce_max_sync(0xffffffffu, s_miny);
    s_maxy = __reduce_max_sync(0xffffffffu, s_maxy);
    s_count = __reduce_add_sync(0xffffffffu, s_count);
    if ((tid & 31) == 0 && s_maxx > 0) {
      atomicMax(stats + 0, s_minx);
      atomicMax(stats + 1, s_maxx);
      atomicMax(stats + 2, s_miny);
      atomicMax(stats + 3, s_maxy);
      atomicAdd(stats + 4, s_count);
    }
  }
}

// Median bin of the histogram (parallel scan over 65,536 bins), translation
// (reference cuda_pipeline.cu:239-278) and pose seeding (:301-327).
__global__ void __launch_bounds__(1024) seedPosesKernel(const int32_t* __restrict__ stats,
                                                        const float* __restrict__ rotations, int n,
                                                        fpk_intrinsics_t k, fpk_params_t p,
                                                        float* __restrict__ t0_out,
                                                        float* __restrict__ poses) {
  __shared__ int warp_sums[32];
  __shared__ int median_bin;
  __shared__ float t_sh[3];
  const int tid = threadIdx.x;
  const int count = stats[4];
  const bool empty = stats[1] == 0 || count <= 0;
  if (tid == 0) {
    median_bin = 0;
  }
  constexpr int kPerThread = kHistBins / 1024;
  int local = 0;
  const int* hist = stats + 8;
  if (!empty) {
    for (int j = 0; j < kPerThread; ++j) {
      local += hist[tid * kPerThread + j];
    }
  }
  // Block-wide exclusive scan of the per-thread sums.
  const int lane = tid & 31;
  const int warp = tid >> 5;
  int incl = local;
  for (int off = 1; off < 32; off <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += v;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int ws = warp_sums[lane];
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, ws, off);
      if (lane >= off) ws += v;
    }
    warp_sums[lane] = ws;  // inclusive over warps
  }
  __syncthreads();
  const int before = incl - local + (warp > 0 ? warp_sums[warp - 1] : 0);
  const int median_rank = count / 2;
  if (!empty && before <= median_rank && before + local > median_rank) {
    int cumulative = before;
    for (int j = 0; j < kPerThread; ++j) {
      cumulative += hist[tid * kPerThread + j];
      if (cumulative > median_rank) {
        median_bin = tid * kPerThread + j;
        break;
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    float3 t = make_float3(0.0f, 0.0f, 0.0f);
    if (!empty) {
      const int min_x = INT_MAX - stats[0];
      const int max_x = stats[1] - 1;
      const int min_y = INT_MAX - stats[2];
      const int max_y = stats[3] - 1;
      const float z_range = p.depth_max - p.depth_min;
      const float z = p.depth_min + (static_cast<float>(median_bin) + 0.5f) * z_range /
                                        static_cast<float>(kHistBins);
      const float u = 0.5f * (static_cast<float>(min_x) + static_cast<float>(max_x));
      const float v = 0.5f * (static_cast<float>(min_y) + static_cast<float>(max_y));
      t = make_float3((u - k.cx) * z / k.fx, (v - k.cy) * z / k.fy, z);
    }
    t_sh[0] = t.x;
    t_sh[1] = t.y;
    t_sh[2] = t.z;
    if (t0_out != nullptr) {
      t0_out[0] = t.x;
      t0_out[1] = t.y;
      t0_out[2] = t.z;
    }
  }
  __syncthreads();
  for (int i = tid; i < n; i += blockDim.x) {
    const float* r = rotations + i * 9;
    float* pose = poses + i * 16;
    pose[0] = r[0];
    pose[1] = r[1];
    pose[2] = r[2];
    pose[3] = t_sh[0];
    pose[4] = r[3];
    pose[5] = r[4];
    pose[6] = r[5];
    pose[7] = t_sh[1];
    pose[8] = r[6];
    pose[9] = r[7];
    pose[10] = r[8];
    pose[11] = t_sh[2];
    pose[12] = 0.0f;
    pose[13] = 0.0f;
    pose[14] = 0.0f;
    pose[15] = 1.0f;
  }
}

__global__ void cropBoxesKernel(const float* __restrict__ poses, int n, fpk_intrinsics_t k,
                                float diameter, float crop_ratio, float4* __restrict__ boxes) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    boxes[i] = cropBox(poses + 16 * i, k, diameter, crop_ratio);
  }
}

// ---------------------------------------------------------------------------
// Rasterizer: one thread per (hypothesis, triangle), z-buffer resident in L2.
// ---------------------------------------------------------------------------

// A triangle thread tests its own bounding-box pixels up to this many pixels.
// Larger triangles are queued and walked by a whole warp each, so one large
// triangle never holds the other 31 lanes of its warp (the common triangle of
// the 50k-250k meshes covers 4-16 bounding-box pixels).
constexpr int kSmallTriPixels = 32;
constexpr int kRasterThreads = 256;
constexpr int kBigTriThreads = 256;

enum class RenderOut { kNhwc = 0, kS2dF32 = 1, kS2dF16 = 2, kS2dBf16 = 3, kS2dF32Exact = 4 };

struct RenderArgs {
  fpk_mesh_t mesh;
  const float* poses;
  const float* boxes_in;  // null: compute crop boxes in-kernel
  float* boxes_out;
  int n;
  fpk_intrinsics_t k;
  fpk_params_t p;
  float diameter;
  // kNhwc outputs
  float* out_rgb;
  float* out_xyz;
  int32_t* tri_ids;
  // s2d pack outputs
  const uint8_t* frame_rgb;
  const float* frame_depth;
  int img_w, img_h;
  float invalid_threshold;
  void* net;
  long long plane_stride;
  int grid_w, grid_h;  // stem space-to-depth grid (83 x 83 for 160 x 160 crops)
  // Workspace: per (hypothesis, vertex) clip position and pixel position; the
  // z-buffer [n][H][W] of packed (depth, triangle + 1) keys, rast rows
  // bottom-up (all ones = background; 51.6 MB at 252 hypotheses, so it stays
  // in the 126 MB L2 between the raster and the shading kernels); the queue of
  // large triangles as (hypothesis, triangle) pairs.
  float4* vclip;
  float2* vscr;
  unsigned long long* zbuf;
  int* big_count;
  int2* big_queue;
  int big_cap;
};

struct TriSetup {
  float4 p0, p1, p2;
  int min_x, max_x, min_y, max_y;
};

__device__ __forceinline__ float4 vertexClip(const RenderArgs& a, const HypState& hs, int vi) {
  const float3 cam = camPosition(hs.pose, loadF3(a.mesh.vertices, vi));
  return clipPosition(cam, hs.box, a.k, a.p.znear, a.p.zfar);
}

// Crop box of hypothesis `hyp`: given, or from its pose.
__device__ __forceinline__ float4 hypothesisBox(const RenderArgs& a, int hyp) {
  return a.boxes_in != nullptr ? reinterpret_cast<const float4*>(a.boxes_in)[hyp]
                               : cropBox(a.poses + hyp * 16, a.k, a.diameter, a.p.crop_ratio);
}

// Triangle setup from the per-vertex workspace; reference
// src/builtin_raster_renderer.cu:53-77 (vertex fetch, projection, bbox). The
// vertex pass stored exactly the clip positions and pixel coordinates the
// reference computes per triangle.
__device__ __forceinline__ TriSetup setupTriangle(const float4* vclip, const float2* vscr, int3 f,
                                                  int width, int height) {
  TriSetup s;
  const int i0 = f.x;
  const int i1 = f.y;
  const int i2 = f.z;
  s.p0 = __ldg(vclip + i0);
  s.p1 = __ldg(vclip + i1);
  s.p2 = __ldg(vclip + i2);
  const float2 q0 = __ldg(vscr + i0);
  const float2 q1 = __ldg(vscr + i1);
  const float2 q2 = __ldg(vscr + i2);
  s.min_x = max(0, static_cast<int>(floorf(fminf(fminf(q0.x, q1.x), q2.x))));
  s.max_x = min(width - 1, static_cast<int>(ceilf(fmaxf(fmaxf(q0.x, q1.x), q2.x))));
  s.min_y = max(0, static_cast<int>(floorf(fminf(fminf(q0.y, q1.y), q2.y))));
  s.max_y = min(height - 1, static_cast<int>(ceilf(fmaxf(fmaxf(q0.y, q1.y), q2.y))));
  return s;
}

__device__ __forceinline__ int3 loadFace(const RenderArgs& a, int tri) {
  return make_int3(__ldg(a.mesh.faces + 3 * tri + 0), __ldg(a.mesh.faces + 3 * tri + 1),
                   __ldg(a.mesh.faces + 3 * tri + 2));
}

__device__ __forceinline__ TriSetup setupTriangle(const RenderArgs& a, const float4* vclip,
                                                  const float2* vscr, int tri, int width, int height) {
  return setupTriangle(vclip, vscr, loadFace(a, tri), width, height);
}

// Coverage + depth key for one pixel; reference builtin_raster_renderer.cu:85-111.
// p0y/p1y/p2y are the per-row terms the reference hoists out of its px loop.
__device__ __forceinline__ void rasterPixel(const TriSetup& s, int px, float inv_w, float p0y,
                                            float p1y, float p2y, int tri_plus_one,
                                            unsigned long long* zrow) {
  const float fx = (2.0f * px + 1.0f) * inv_w - 1.0f;
  const float p0x = s.p0.x - fx * s.p0.w;
  const float p1x = s.p1.x - fx * s.p1.w;
  const float p2x = s.p2.x - fx * s.p2.w;
  const float a0 = p1x * p2y - p1y * p2x;
  const float a1 = p2x * p0y - p2y * p0x;
  const float a2 = p0x * p1y - p0y * p1x;
  const bool inside_pos = a0 >= 0.0f && a1 >= 0.0f && a2 >= 0.0f;
  const bool inside_neg = a0 <= 0.0f && a1 <= 0.0f && a2 <= 0.0f;
  const float area = a0 + a1 + a2;
  if ((!inside_pos && !inside_neg) || area == 0.0f) {
    return;
  }
  const float z = s.p0.z * a0 + s.p1.z * a1 + s.p2.z * a2;
  const float w = s.p0.w * a0 + s.p1.w * a1 + s.p2.w * a2;
  if (w == 0.0f) {
    return;
  }
  const float zw = z / w;
  atomicMin(zrow + px, packDepthKey(zw, tri_plus_one));
}

__device__ __forceinline__ float rowTerm(float fy, const float4& q) { return q.y - fy * q.w; }

// reference src/raster_kernels.cuh:382-408 sampleTexture.
__device__ __forceinline__ float3 sampleTexture(const float* texture, int width, int height,
                                                float2 uv) {
  const float u = uv.x - floorf(uv.x);
  const float v = 1.0f - (uv.y - floorf(uv.y));
  const float x = u * static_cast<float>(width) - 0.5f;
  const float y = v * static_cast<float>(height) - 0.5f;
  const int ix0 = static_cast<int>(floorf(x));
  const int iy0 = static_cast<int>(floorf(y));
  const int x0 = (ix0 % width + width) % width;
  const int y0 = (iy0 % height + height) % height;
  const int x1 = (x0 + 1) % width;
  const int y1 = (y0 + 1) % height;
  const float tx = x - static_cast<float>(ix0);
  const float ty = y - static_cast<float>(iy0);
  const float3 c00 = loadF3(texture, y0 * width + x0);
  const float3 c10 = loadF3(texture, y0 * width + x1);
  const float3 c01 = loadF3(texture, y1 * width + x0);
  const float3 c11 = loadF3(texture, y1 * width + x1);
  return make_float3((1.0f - ty) * ((1.0f - tx) * c00.x + tx * c10.x) +
                         ty * ((1.0f - tx) * c01.x + tx * c11.x),
                     (1.0f - ty) * ((1.0f - tx) * c00.y + tx * c10.y) +
                         ty * ((1.0f - tx) * c01.y + tx * c11.y),
                     (1.0f - ty) * ((1.0f - tx) * c00.z + tx * c10.z) +
                         ty * ((1.0f - tx) * c01.z + tx * c11.z));
}

// Resolve + deferred shading of one pixel whose z-buffer winner is tri_plus_one;
// reference src/builtin_raster_renderer.cu:137-171 and raster_kernels.cuh:443-494.
__device__ __forceinline__ void shadePixel(const RenderArgs& a, const HypState& hs, const float4* vclip,
                                           int tri_plus_one, int px, int py, int width, int height,
                                           float3& rgb, float3& xyz) {
  const int tri = tri_plus_one - 1;
  const int i0 = __ldg(a.mesh.faces + 3 * tri + 0);
  const int i1 = __ldg(a.mesh.faces + 3 * tri + 1);
  const int i2 = __ldg(a.mesh.faces + 3 * tri + 2);
  const float3 c0 = camPosition(hs.pose, loadF3(a.mesh.vertices, i0));
  const float3 c1 = camPosition(hs.pose, loadF3(a.mesh.vertices, i1));
  const float3 c2 = camPosition(hs.pose, loadF3(a.mesh.vertices, i2));
  const float4 p0 = __ldg(vclip + i0);  // = clipPosition(c0, box, ...), from the vertex pass
  const float4 p1 = __ldg(vclip + i1);
  const float4 p2 = __ldg(vclip + i2);

  const float fx = (2.0f * px + 1.0f) / static_cast<float>(width) - 1.0f;
  const float fy = (2.0f * py + 1.0f) / static_cast<float>(height) - 1.0f;
  const float p0x = p0.x - fx * p0.w;
  const float p0y = p0.y - fy * p0.w;
  const float p1x = p1.x - fx * p1.w;
  const float p1y = p1.y - fy * p1.w;
  const float p2x = p2.x - fx * p2.w;
  const float p2y = p2.y - fy * p2.w;
  const float a0 = p1x * p2y - p1y * p2x;
  const float a1 = p2x * p0y - p2y * p0x;
  const float a2 = p0x * p1y - p0y * p1x;
  const float iw = 1.0f / (a0 + a1 + a2);
  float b0 = __saturatef(a0 * iw);
  float b1 = __saturatef(a1 * iw);
  const float bs = 1.0f / fmaxf(b0 + b1, 1.0f);
  b0 *= bs;
  b1 *= bs;

  const float b2 = fmaxf(0.0f, 1.0f - b0 - b1);
  xyz = make_float3(b0 * c0.x + b1 * c1.x + b2 * c2.x, b0 * c0.y + b1 * c1.y + b2 * c2.y,
                    b0 * c0.z + b1 * c1.z + b2 * c2.z);
  const float3 n0 = camNormal(hs.pose, loadF3(a.mesh.normals, i0));
  const float3 n1 = camNormal(hs.pose, loadF3(a.mesh.normals, i1));
  const float3 n2 = camNormal(hs.pose, loadF3(a.mesh.normals, i2));
  const float3 n = normalize3(make_float3(b0 * n0.x + b1 * n1.x + b2 * n2.x,
                                          b0 * n0.y + b1 * n1.y + b2 * n2.y,
                                          b0 * n0.z + b1 * n1.z + b2 * n2.z));
  float3 albedo;
  if (a.mesh.texture != nullptr && a.mesh.uvs != nullptr && a.mesh.texture_width > 0 &&
      a.mesh.texture_height > 0) {
    const float2 uv0 = make_float2(__ldg(a.mesh.uvs + 2 * i0), __ldg(a.mesh.uvs + 2 * i0 + 1));
    const float2 uv1 = make_float2(__ldg(a.mesh.uvs + 2 * i1), __ldg(a.mesh.uvs + 2 * i1 + 1));
    const float2 uv2 = make_float2(__ldg(a.mesh.uvs + 2 * i2), __ldg(a.mesh.uvs + 2 * i2 + 1));
    albedo = sampleTexture(a.mesh.texture, a.mesh.texture_width, a.mesh.texture_height,
                           make_float2(b0 * uv0.x + b1 * uv1.x + b2 * uv2.x,
                                       b0 * uv0.y + b1 * uv1.y + b2 * uv2.y));
  } else {
    const float3 q0 = loadF3(a.mesh.colors, i0);
    const float3 q1 = loadF3(a.mesh.colors, i1);
    const float3 q2 = loadF3(a.mesh.colors, i2);
    albedo = make_float3(b0 * q0.x + b1 * q1.x + b2 * q2.x, b0 * q0.y + b1 * q1.y + b2 * q2.y,
                         b0 * q0.z + b1 * q1.z + b2 * q2.z);
  }
  const float diffuse = fmaxf(0.0f, -n.z);
  const float light = fminf(fmaxf(a.p.ambient_weight + a.p.diffuse_weight * diffuse, 0.0f), 1.5f);
  rgb = make_float3(fminf(fmaxf(albedo.x * light, 0.0f), 1.0f),
                    fminf(fmaxf(albedo.y * light, 0.0f), 1.0f),
                    fminf(fmaxf(albedo.z * light, 0.0f), 1.0f));
}

// reference src/cuda_pipeline.cu:370-407 sampleRgbBilinear.
// lut255[v] holds v / 255.0f (filled with that division on the device, so
// the table lookup returns the reference's quotient bit for bit).
__device__ __forceinline__ float3 sampleRgbBilinear(const uint8_t* rgb, int width, int height,
                                                    float x, float y, const float* lut255) {
  if (x < 0.0f || y < 0.0f || x > static_cast<float>(width - 1) ||
      y > static_cast<float>(height - 1)) {
    return make_float3(0.0f, 0.0f, 0.0f);
  }
  const int x0 = min(max(static_cast<int>(floorf(x)), 0), width - 1);
  const int y0 = min(max(static_cast<int>(floorf(y)), 0), height - 1);
  const int x1 = min(x0 + 1, width - 1);
  const int y1 = min(y0 + 1, height - 1);
  const float tx = x - static_cast<float>(x0);
  const float ty = y - static_cast<float>(y0);
  const uint8_t* q00 = rgb + (y0 * width + x0) * 3;
  const uint8_t* q10 = rgb + (y0 * width + x1) * 3;
  const uint8_t* q01 = rgb + (y1 * width + x0) * 3;
  const uint8_t* q11 = rgb + (y1 * width + x1) * 3;
  const float3 c00 = make_float3(lut255[__ldg(q00 + 0)],
                                 lut255[__ldg(q00 + 1)],
                                 lut255[__ldg(q00 + 2)]);
  const float3 c10 = make_float3(lut255[__ldg(q10 + 0)],
                                 lut255[__ldg(q10 + 1)],
                                 lut255[__ldg(q10 + 2)]);
  const float3 c01 = make_float3(lut255[__ldg(q01 + 0)],
                                 lut255[__ldg(q01 + 1)],
                                 lut255[__ldg(q01 + 2)]);
  const float3 c11 = make_float3(lut255[__ldg(q11 + 0)],
                                 lut255[__ldg(q11 + 1)],
                                 lut255[__ldg(q11 + 2)]);
  return make_float3((1.0f - ty) * ((1.0f - tx) * c00.x + tx * c10.x) +
                         ty * ((1.0f - tx) * c01.x + tx * c11.x),
                     (1.0f - ty) * ((1.0f - tx) * c00.y + tx * c10.y) +
                         ty * ((1.0f - tx) * c01.y + tx * c11.y),
                     (1.0f - ty) * ((1.0f - tx) * c00.z + tx * c10.z) +
                         ty * ((1.0f - tx) * c01.z + tx * c11.z));
}

// Observed xyz at the nearest frame pixel, back-projected from the filtered
// depth (reference sampleXyzNearest cuda_pipeline.cu:409-420 over the
// depthToXyzKernel map :173-192).
__device__ __forceinline__ float3 observedXyz(const float* depth, int width, int height,
                                              fpk_intrinsics_t k, const fpk_params_t& p, float x,
                                              float y) {
  const int xx = static_cast<int>(roundf(x));
  const int yy = static_cast<int>(roundf(y));
  if (xx < 0 || yy < 0 || xx >= width || yy >= height) {
    return make_float3(0.0f, 0.0f, 0.0f);
  }
  const float z = __ldg(depth + yy * width + xx);
  if (!validDepth(z, p.depth_min, p.depth_max)) {
    return make_float3(0.0f, 0.0f, 0.0f);
  }
  return make_float3((static_cast<float>(xx) - k.cx) * z / k.fx,
                     (static_cast<float>(yy) - k.cy) * z / k.fy, z);
}

// Network-input normalisation of one crop pixel (reference cuda_pipeline.cu:458-496).
struct PackedPixel {
  float r[6];
  float o[6];
};

__device__ __forceinline__ PackedPixel packPixel(const RenderArgs& a, const HypState& hs, int x,
                                                 int y, int crop_width, int crop_height,
                                                 float3 rend_rgb, float3 rend_xyz,
                                                 const float* lut255) {
  const float4 box = hs.box;
  const float crop_w = fmaxf(box.z - box.x, 1.0f);
  const float crop_h = fmaxf(box.w - box.y, 1.0f);
  float src_x = box.x + static_cast<float>(x) * crop_w / static_cast<float>(crop_width);
  float src_y = box.y + static_cast<float>(y) * crop_h / static_cast<float>(crop_height);
  if (a.img_w > 1) {
    src_x = src_x * static_cast<float>(a.img_w) / static_cast<float>(a.img_w - 1) - 0.5f;
  }
  if (a.img_h > 1) {
    src_y = src_y * static_cast<float>(a.img_h) / static_cast<float>(a.img_h - 1) - 0.5f;
  }
  const float3 t = make_float3(hs.pose[3], hs.pose[7], hs.pose[11]);
  const float radius = fmaxf(a.diameter * 0.5f, 1e-6f);
  const float3 obs_rgb = sampleRgbBilinear(a.frame_rgb, a.img_w, a.img_h, src_x, src_y, lut255);
  float3 obs_xyz = observedXyz(a.frame_depth, a.img_w, a.img_h, a.k, a.p, src_x, src_y);
  const bool obs_invalid = obs_xyz.z < a.invalid_threshold;
  obs_xyz = make_float3((obs_xyz.x - t.x) / radius, (obs_xyz.y - t.y) / radius,
                        (obs_xyz.z - t.z) / radius);
  if (obs_invalid || fabsf(obs_xyz.x) >= 2.0f || fabsf(obs_xyz.y) >= 2.0f ||
      fabsf(obs_xyz.z) >= 2.0f) {
    obs_xyz = make_float3(0.0f, 0.0f, 0.0f);
  }
  const bool rendered_bg = rend_xyz.z < a.invalid_threshold;
  rend_xyz = make_float3((rend_xyz.x - t.x) / radius, (rend_xyz.y - t.y) / radius,
                         (rend_xyz.z - t.z) / radius);
  if (rendered_bg) {
    rend_xyz = make_float3(0.0f, 0.0f, 0.0f);
  }
  PackedPixel out;
  out.r[0] = rend_rgb.x;
  out.r[1] = rend_rgb.y;
  out.r[2] = rend_rgb.z;
  out.r[3] = rend_xyz.x;
  out.r[4] = rend_xyz.y;
  out.r[5] = rend_xyz.z;
  out.o[0] = obs_rgb.x;
  out.o[1] = obs_rgb.y;
  out.o[2] = obs_rgb.z;
  out.o[3] = obs_xyz.x;
  out.o[4] = obs_xyz.y;
  out.o[5] = obs_xyz.z;
  return out;
}

template <typename T>
__device__ __forceinline__ T fromFloat(float v);
template <>
__device__ __forceinline__ float fromFloat<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half fromFloat<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 fromFloat<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// 8 channels (6 used + 2 zero) of one crop pixel into the stem's
// space-to-depth KP8 layout: pixel (y, x) -> plane ((y+3)%2)*2 + (x+3)%2, row
// of grid cell ((y+3)/2, (x+3)/2). See fp_nets.cu for how the stem consumes it.
template <typename T, bool kExact = false>
__device__ __forceinline__ void storeS2d(void* net, long long plane_stride, int img, int y, int x,
                                         int gw, int gh, const float* v) {
  const int gy = (y + 3) >> 1;
  const int gx = (x + 3) >> 1;
  const int sub = ((y + 3) & 1) * 2 + ((x + 3) & 1);
  unsigned char* dst = reinterpret_cast<unsigned char*>(net) + sub * plane_stride +
                       ((static_cast<long long>(img) * gh + gy) * gw + gx) * 16;
  if constexpr (sizeof(T) == 2) {
    alignas(16) T tmp[8];
#pragma unroll
    for (int c = 0; c < 6; ++c) tmp[c] = fromFloat<T>(v[c]);
    tmp[6] = fromFloat<T>(0.0f);
    tmp[7] = fromFloat<T>(0.0f);
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(tmp);
  } else {
    // fp32: 8 values span two 16-byte records; the layout holds 4 channels per
    // record (KP4), so channels 0-3 go to plane 2*sub and 4-7 to plane 2*sub+1.
    unsigned char* d0 = reinterpret_cast<unsigned char*>(net) + (2 * sub) * plane_stride +
                        ((static_cast<long long>(img) * gh + gy) * gw + gx) * 16;
    if constexpr (kExact) {  // strict FP32: the stem splits its operands itself
      *reinterpret_cast<float4*>(d0) = make_float4(v[0], v[1], v[2], v[3]);
      *reinterpret_cast<float4*>(d0 + plane_stride) = make_float4(v[4], v[5], 0.0f, 0.0f);
    } else {
      // The stem reads fp32 inputs as TF32: round to nearest here, as every other
      // producer of a TF32 operand does (the NCHW seam loader included).
      *reinterpret_cast<float4*>(d0) =
          make_float4(tc::tf32Round(v[0]), tc::tf32Round(v[1]), tc::tf32Round(v[2]), tc::tf32Round(v[3]));
      *reinterpret_cast<float4*>(d0 + plane_stride) =
          make_float4(tc::tf32Round(v[4]), tc::tf32Round(v[5]), 0.0f, 0.0f);
    }
    (void)dst;
  }
}

// Vertex pass: crop box and, per vertex, clip position and pixel position
// under each hypothesis (once per vertex instead of once per triangle corner).
__global__ void __launch_bounds__(256) vertexKernel(RenderArgs a) {
  tc::pdlTrigger();
  tc::pdlWait();
  __shared__ HypState hs;
  const int hyp = blockIdx.y;
  const int tid = threadIdx.x;
  if (tid < 12) hs.pose[tid] = a.poses[hyp * 16 + tid];
  if (tid == 0) {
    hs.box = hypothesisBox(a, hyp);
    if (a.boxes_out != nullptr && blockIdx.x == 0) reinterpret_cast<float4*>(a.boxes_out)[hyp] = hs.box;
  }
  __syncthreads();
  // Clear this hypothesis's z-buffer for the raster grid, which starts only
  // after this grid has completed (the previous call's shading, which reads
  // the z-buffer, completed before this grid's wait above returned).
  const int crop_px = a.p.input_width * a.p.input_height;
  unsigned long long* z = a.zbuf + static_cast<size_t>(hyp) * crop_px;
  for (int i = blockIdx.x * blockDim.x + tid; i < crop_px; i += gridDim.x * blockDim.x) z[i] = ~0ull;
  if (hyp == 0 && blockIdx.x == 0 && tid == 0) *a.big_count = 0;
  const int v = blockIdx.x * blockDim.x + tid;
  const int nv = a.mesh.n_vertices;
  if (v >= nv) return;
  const float4 c = vertexClip(a, hs, v);
  const float half_w = 0.5f * static_cast<float>(a.p.input_width);
  const float half_h = 0.5f * static_cast<float>(a.p.input_height);
  const size_t o = static_cast<size_t>(hyp) * nv + v;
  a.vclip[o] = c;
  a.vscr[o] = make_float2((c.x / c.w + 1.0f) * half_w - 0.5f, (c.y / c.w + 1.0f) * half_h - 0.5f);
}

// Raster pass: one thread per (triangle, hypothesis). The coverage test and
// depth key repeat the reference's per-pixel expressions over the reference's
// bounding box (builtin_raster_renderer.cu:40-114), so the winning key of
// every pixel -- the minimum over the same set of keys -- is the reference's.
// The 64-bit atomicMin goes to the L2-resident z-buffer.
__global__ void __launch_bounds__(kRasterThreads) rasterTriKernel(RenderArgs a) {
  tc::pdlTrigger();
  const int hyp = blockIdx.y;
  const int tri = blockIdx.x * kRasterThreads + threadIdx.x;
  const int nf = a.mesh.n_faces;
  const int3 face = tri < nf ? loadFace(a, tri) : make_int3(0, 0, 0);  // the mesh is constant
  tc::pdlWait();  // vertex positions and the cleared z-buffer are ready from here on
  if (tri >= nf) return;
  const int width = a.p.input_width;
  const int height = a.p.input_height;
  const size_t vbase = static_cast<size_t>(hyp) * a.mesh.n_vertices;
  const TriSetup s = setupTriangle(a.vclip + vbase, a.vscr + vbase, face, width, height);
  if (s.min_x > s.max_x || s.min_y > s.max_y) return;
  const int npx = (s.max_x - s.min_x + 1) * (s.max_y - s.min_y + 1);
  if (npx > kSmallTriPixels) {
    const int slot = atomicAdd(a.big_count, 1);
    if (slot < a.big_cap) {
      a.big_queue[slot] = make_int2(hyp, tri);
      return;
    }
    // Queue full: this thread rasterizes the triangle itself (slower, same result).
  }
  // One flat loop over the bounding box (row terms refreshed on each new row):
  // a warp runs as many iterations as its largest box.
  const float inv_w = 1.0f / static_cast<float>(width);
  const float inv_h = 1.0f / static_cast<float>(height);
  int px = s.min_x;
  int py = s.min_y;
  float fy = (2.0f * py + 1.0f) * inv_h - 1.0f;
  float p0y = rowTerm(fy, s.p0);
  float p1y = rowTerm(fy, s.p1);
  float p2y = rowTerm(fy, s.p2);
  unsigned long long* zrow = a.zbuf + (static_cast<size_t>(hyp) * height + py) * width;
  for (int i = 0; i < npx; ++i) {
    rasterPixel(s, px, inv_w, p0y, p1y, p2y, tri + 1, zrow);
    if (++px > s.max_x) {
      px = s.min_x;
      ++py;
      fy = (2.0f * py + 1.0f) * inv_h - 1.0f;
      p0y = rowTerm(fy, s.p0);
      p1y = rowTerm(fy, s.p1);
      p2y = rowTerm(fy, s.p2);
      zrow += width;
    }
  }
}

// Large triangles: one warp per queued triangle, lanes over its pixels.
__global__ void __launch_bounds__(kBigTriThreads) bigTriKernel(RenderArgs a) {
  tc::pdlTrigger();
  tc::pdlWait();  // the raster grid has queued every large triangle
  const int count = min(*a.big_count, a.big_cap);
  const int lane = threadIdx.x & 31;
  const int nwarps = gridDim.x * (kBigTriThreads / 32);
  const int width = a.p.input_width;
  const int height = a.p.input_height;
  const float inv_w = 1.0f / static_cast<float>(width);
  const float inv_h = 1.0f / static_cast<float>(height);
  for (int q = (blockIdx.x * kBigTriThreads + threadIdx.x) >> 5; q < count; q += nwarps) {
    const int2 e = a.big_queue[q];
    const size_t vbase = static_cast<size_t>(e.x) * a.mesh.n_vertices;
    const TriSetup s = setupTriangle(a, a.vclip + vbase, a.vscr + vbase, e.y, width, height);
    const int bw = s.max_x - s.min_x + 1;
    const int npx = bw * (s.max_y - s.min_y + 1);
    unsigned long long* z = a.zbuf + static_cast<size_t>(e.x) * height * width;
    for (int i = lane; i < npx; i += 32) {
      const int py = s.min_y + i / bw;
      const int px = s.min_x + i % bw;
      const float fy = (2.0f * py + 1.0f) * inv_h - 1.0f;
      rasterPixel(s, px, inv_w, rowTerm(fy, s.p0), rowTerm(fy, s.p1), rowTerm(fy, s.p2), e.y + 1,
                  z + static_cast<size_t>(py) * width);
    }
  }
}

// Shade + emit: one thread per crop pixel, all hypotheses (many warps per SM
// to hide the gathers: eight 256-thread CTAs per SM, 32 registers with a few
// spills, measured 4 % faster than five). Output rows are top-down:
// y = height - 1 - py.
constexpr int kShadeThreads = 256;  // also the size of the 1/255 table it fills

template <RenderOut kOut>
__global__ void __launch_bounds__(kShadeThreads, 8) shadeKernel(RenderArgs a) {
  __shared__ HypState hs;
  __shared__ float lut255[256];
  const int width = a.p.input_width;
  const int height = a.p.input_height;
  const int hyp = blockIdx.y;  // grid: (pixel blocks, hypotheses)
  const int tid = threadIdx.x;
  tc::pdlTrigger();
  lut255[tid] = static_cast<float>(tid) / 255.0f;
  tc::pdlWait();  // the raster (triangle ids) is complete from here on
  if (tid < 12) hs.pose[tid] = a.poses[hyp * 16 + tid];
  if (tid == 0) hs.box = hypothesisBox(a, hyp);
  __syncthreads();
  const int rem = blockIdx.x * kShadeThreads + tid;
  if (rem >= width * height) return;
  const size_t idx = static_cast<size_t>(hyp) * width * height + rem;
  const int py = rem / width;
  const int px = rem - py * width;
  // Resolve: the winning key's triangle (0 = background).
  const unsigned long long key = a.zbuf[idx];
  const int t = key == ~0ull ? 0 : static_cast<int>(key & 0xFFFFFFFFull);
  const int tri_plus_one = t <= a.mesh.n_faces ? t : 0;
  float3 rgb = make_float3(0.0f, 0.0f, 0.0f);
  float3 xyz = make_float3(0.0f, 0.0f, 0.0f);
  if (tri_plus_one > 0) {
    shadePixel(a, hs, a.vclip + static_cast<size_t>(hyp) * a.mesh.n_vertices, tri_plus_one, px, py, width,
               height, rgb, xyz);
  }
  const int y = height - 1 - py;
  if constexpr (kOut == RenderOut::kNhwc) {
    const size_t o = (static_cast<size_t>(hyp) * height + y) * width + px;
    a.out_rgb[3 * o + 0] = rgb.x;
    a.out_rgb[3 * o + 1] = rgb.y;
    a.out_rgb[3 * o + 2] = rgb.z;
    a.out_xyz[3 * o + 0] = xyz.x;
    a.out_xyz[3 * o + 1] = xyz.y;
    a.out_xyz[3 * o + 2] = xyz.z;
    if (a.tri_ids != nullptr) a.tri_ids[idx] = tri_plus_one;
  } else {
    const PackedPixel pk = packPixel(a, hs, px, y, width, height, rgb, xyz, lut255);
    constexpr bool kExact = kOut == RenderOut::kS2dF32Exact;
    using T = typename std::conditional<
        kOut == RenderOut::kS2dF32 || kExact, float,
        typename std::conditional<kOut == RenderOut::kS2dF16, __half, __nv_bfloat16>::type>::type;
    storeS2d<T, kExact>(a.net, a.plane_stride, hyp, y, px, a.grid_w, a.grid_h, pk.r);
    storeS2d<T, kExact>(a.net, a.plane_stride, a.n + hyp, y, px, a.grid_w, a.grid_h, pk.o);
  }
}

// Reference-layout pack: NCHW [n,6,H,W] fp32 from NHWC renders (seam path).
__global__ void packNchwKernel(RenderArgs a, const float* __restrict__ rend_rgb,
                               const float* __restrict__ rend_xyz, float* __restrict__ net_r,
                               float* __restrict__ net_o) {
  const int width = a.p.input_width;
  const int height = a.p.input_height;
  const long long total = static_cast<long long>(a.n) * width * height;
  const long long linear = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  __shared__ float lut255[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) lut255[i] = static_cast<float>(i) / 255.0f;
  __syncthreads();
  if (linear >= total) {
    return;
  }
  const int x = static_cast<int>(linear % width);
  const int y = static_cast<int>((linear / width) % height);
  const int s = static_cast<int>(linear / (static_cast<long long>(width) * height));
  HypState hs;
  for (int i = 0; i < 12; ++i) hs.pose[i] = __ldg(a.poses + s * 16 + i);
  hs.box = reinterpret_cast<const float4*>(a.boxes_in)[s];
  const size_t o = (static_cast<size_t>(s) * height + y) * width + x;
  const float3 rgb = make_float3(rend_rgb[3 * o], rend_rgb[3 * o + 1], rend_rgb[3 * o + 2]);
  const float3 xyz = make_float3(rend_xyz[3 * o], rend_xyz[3 * o + 1], rend_xyz[3 * o + 2]);
  const PackedPixel pk = packPixel(a, hs, x, y, width, height, rgb, xyz, lut255);
  const size_t plane = static_cast<size_t>(width) * height;
  for (int c = 0; c < 6; ++c) {
    net_r[(static_cast<size_t>(s) * 6 + c) * plane + static_cast<size_t>(y) * width + x] = pk.r[c];
    net_o[(static_cast<size_t>(s) * 6 + c) * plane + static_cast<size_t>(y) * width + x] = pk.o[c];
  }
}

// ---------------------------------------------------------------------------
// Pose update and selection.
// ---------------------------------------------------------------------------

// reference src/cuda_pipeline.cu:46-85 so3ExpTranspose.
__device__ void so3ExpTranspose(float3 omega, float* out) {
  const float theta =
      sqrtf(fmaxf(omega.x * omega.x + omega.y * omega.y + omega.z * omega.z, 0.0f));
  for (int i = 0; i < 9; ++i) out[i] = 0.0f;
  out[0] = out[4] = out[8] = 1.0f;
  if (theta < 1e-6f) {
    return;
  }
  const float inv_theta = 1.0f / theta;
  const float x = omega.x * inv_theta;
  const float y = omega.y * inv_theta;
  const float z = omega.z * inv_theta;
  const float s = sinf(theta);
  const float c = cosf(theta);
  const float one_c = 1.0f - c;
  float r[9];
  r[0] = c + x * x * one_c;
  r[1] = x * y * one_c - z * s;
  r[2] = x * z * one_c + y * s;
  r[3] = y * x * one_c + z * s;
  r[4] = c + y * y * one_c;
  r[5] = y * z * one_c - x * s;
  r[6] = z * x * one_c - y * s;
  r[7] = z * y * one_c + x * s;
  r[8] = c + z * z * one_c;
  out[0] = r[0];
  out[1] = r[3];
  out[2] = r[6];
  out[3] = r[1];
  out[4] = r[4];
  out[5] = r[7];
  out[6] = r[2];
  out[7] = r[5];
  out[8] = r[8];
}

// reference src/cuda_pipeline.cu:513-547 applyPoseDeltasKernel.
__global__ void applyDeltasKernel(float* __restrict__ poses, const float* __restrict__ delta_t,
                                  const float* __restrict__ delta_r, int n, float diameter,
                                  float rotation_normalizer_rad) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) {
    return;
  }
  float* pose = poses + i * 16;
  const float3 omega = make_float3(tanhf(delta_r[i * 3 + 0]) * rotation_normalizer_rad,
                                   tanhf(delta_r[i * 3 + 1]) * rotation_normalizer_rad,
                                   tanhf(delta_r[i * 3 + 2]) * rotation_normalizer_rad);
  float dR[9];
  so3ExpTranspose(omega, dR);
  const float old_r[9] = {pose[0], pose[1], pose[2], pose[4], pose[5],
                          pose[6], pose[8], pose[9], pose[10]};
  for (int row = 0; row < 3; ++row) {
    for (int col = 0; col < 3; ++col) {
      float v = 0.0f;
      for (int kk = 0; kk < 3; ++kk) {
        v += dR[row * 3 + kk] * old_r[kk * 3 + col];
      }
      pose[row * 4 + col] = v;
    }
  }
  const float scale = diameter * 0.5f;
  pose[3] += delta_t[i * 3 + 0] * scale;
  pose[7] += delta_t[i * 3 + 1] * scale;
  pose[11] += delta_t[i * 3 + 2] * scale;
}

// Parallel arg-max with the reference's sequential semantics
// (cuda_pipeline.cu:549-582): the running best starts at scores[0] and is only
// replaced by a strictly greater score, so the first maximum wins and NaN
// scores never win (a NaN at index 0 is never replaced).
__device__ __forceinline__ bool better(float s, int i, float bs, int bi) {
  return s > bs || (s == bs && i < bi);
}

__global__ void __launch_bounds__(256) selectBestKernel(const float* __restrict__ poses,
                                                        const float* __restrict__ scores, int n,
                                                        float cx, float cy, float cz,
                                                        float* __restrict__ result) {
  __shared__ float sh_s[8];
  __shared__ int sh_i[8];
  const int tid = threadIdx.x;
  const float s0 = scores[0];
  float bs = s0;
  int bi = 0;
  if (!isnan(s0)) {
    for (int i = tid; i < n; i += 256) {
      const float s = scores[i];
      if (!isnan(s) && better(s, i, bs, bi)) {
        bs = s;
        bi = i;
      }
    }
    for (int off = 16; off > 0; off >>= 1) {
      const float os = __shfl_down_sync(0xffffffffu, bs, off);
      const int oi = __shfl_down_sync(0xffffffffu, bi, off);
      if (better(os, oi, bs, bi)) {
        bs = os;
        bi = oi;
      }
    }
    if ((tid & 31) == 0) {
      sh_s[tid >> 5] = bs;
      sh_i[tid >> 5] = bi;
    }
    __syncthreads();
    if (tid == 0) {
      for (int w = 1; w < 8; ++w) {
        if (better(sh_s[w], sh_i[w], bs, bi)) {
          bs = sh_s[w];
          bi = sh_i[w];
        }
      }
    }
  }
  if (tid == 0) {
    const float* src = poses + bi * 16;
    float dst[16];
    for (int i = 0; i < 16; ++i) dst[i] = 0.0f;
    dst[15] = 1.0f;
    for (int r = 0; r < 3; ++r)
      for (int c = 0; c < 3; ++c) dst[r * 4 + c] = src[r * 4 + c];
    const float neg_center[3] = {-cx, -cy, -cz};
    for (int r = 0; r < 3; ++r) {
      dst[r * 4 + 3] = src[r * 4 + 3] + src[r * 4 + 0] * neg_center[0] +
                       src[r * 4 + 1] * neg_center[1] + src[r * 4 + 2] * neg_center[2];
    }
    for (int i = 0; i < 16; ++i) result[i] = dst[i];
    result[16] = bs;
    reinterpret_cast<int*>(result)[17] = bi;
  }
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------

int validateParams(const fpk_params_t* p) {
  if (p == nullptr) return fail("fpk: params are required");
  if (p->erosion_radius < 0 || p->erosion_radius > kMaxRadius || p->bilateral_radius < 0 ||
      p->bilateral_radius > kMaxRadius) {
    return fail("fpk: erosion/bilateral radius must be in [0, 4]");
  }
  if (p->input_width <= 0 || p->input_height <= 0) return fail("fpk: crop size must be positive");
  return 0;
}

// SM count of the current device (cached per device).
int renderSms() {
  static DeviceValue cache;
  return cache.get([](int dev) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
  });
}

// Workspace of one render call: clip positions (16 B) and pixel positions
// (8 B) per (hypothesis, vertex), the z-buffer (8 B per crop pixel) and the
// large-triangle queue (8 B per entry; sized at a quarter of the
// (hypothesis, vertex) count -- about an eighth of the triangles of a closed
// mesh -- beyond which large triangles are rasterized by their own thread).
struct RenderWorkspace {
  size_t clip = 0, scr = 0, zbuf = 0, count = 0, queue = 0, total = 0;
  int cap = 0;
  RenderWorkspace(int n, int nv, int w, int h) {
    auto up = [](size_t b) { return (b + 255) / 256 * 256; };
    clip = up(static_cast<size_t>(n) * nv * 16);
    scr = up(static_cast<size_t>(n) * nv * 8);
    zbuf = up(static_cast<size_t>(n) * w * h * 8);
    count = 256;
    const size_t c = std::min<size_t>(static_cast<size_t>(n) * nv / 4 + 4096, size_t{1} << 28);
    cap = static_cast<int>(c);
    queue = up(c * 8);
    total = clip + scr + zbuf + count + queue;
  }
};

template <RenderOut kOut>
int launchRender(RenderArgs& a, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  const RenderWorkspace ws(a.n, a.mesh.n_vertices, a.p.input_width, a.p.input_height);
  void* mem = workspace;
  if (mem == nullptr) {
    // No caller workspace: a stream-ordered allocation, released in stream order.
    const cudaError_t e = cudaMallocAsync(&mem, ws.total, stream);
    if (e != cudaSuccess) return fail(std::string("render workspace: ") + cudaGetErrorString(e));
  } else if (workspace_bytes < ws.total || reinterpret_cast<uintptr_t>(workspace) % 256 != 0) {
    return fail("render workspace too small or not 256-byte aligned (need " + std::to_string(ws.total) +
                " bytes, see fpk_render_workspace_bytes)");
  }
  unsigned char* base = static_cast<unsigned char*>(mem);
  a.vclip = reinterpret_cast<float4*>(base);
  a.vscr = reinterpret_cast<float2*>(base + ws.clip);
  a.zbuf = reinterpret_cast<unsigned long long*>(base + ws.clip + ws.scr);
  a.big_count = reinterpret_cast<int*>(base + ws.clip + ws.scr + ws.zbuf);
  a.big_queue = reinterpret_cast<int2*>(base + ws.clip + ws.scr + ws.zbuf + ws.count);
  a.big_cap = ws.cap;
  // Algorithmic bytes: mesh once, the frame once (rgb + depth) when packing,
  // and the outputs (NHWC fp32 rgb+xyz, or both packed network inputs).
  const double px = static_cast<double>(a.n) * a.p.input_width * a.p.input_height;
  const double elt = kOut == RenderOut::kNhwc
                         ? 0.0
                         : ((kOut == RenderOut::kS2dF32 || kOut == RenderOut::kS2dF32Exact) ? 4.0 : 2.0);
  const double bytes = a.mesh.n_vertices * 36.0 + a.mesh.n_faces * 12.0 +
                       (kOut == RenderOut::kNhwc ? px * 24.0
                                                 : px * 12.0 * elt + a.img_w * static_cast<double>(a.img_h) * 7.0);
  int rc = 0;
  {
    for (int i = 0; i < 4; ++i) prof::countLaunch(prof::kRender);
    prof::Scope scope(prof::kRender, bytes, stream);
    cudaError_t e = launchPdl(vertexKernel, dim3((a.mesh.n_vertices + 255) / 256, a.n), dim3(256), 0, stream, a);
    if (e == cudaSuccess) {
      e = launchPdl(rasterTriKernel, dim3((a.mesh.n_faces + kRasterThreads - 1) / kRasterThreads, a.n),
                    dim3(kRasterThreads), 0, stream, a);
    }
    if (e == cudaSuccess) e = launchPdl(bigTriKernel, dim3(2 * renderSms()), dim3(kBigTriThreads), 0, stream, a);
    if (e == cudaSuccess) {
      e = launchPdl(shadeKernel<kOut>,
                    dim3((a.p.input_width * a.p.input_height + kShadeThreads - 1) / kShadeThreads, a.n),
                    dim3(kShadeThreads), 0, stream, a);
    }
    if (e != cudaSuccess) cudaGetLastError();
    rc = e != cudaSuccess ? fail(std::string("render kernels: ") + cudaGetErrorString(e)) : checkLaunch("render kernels");
  }
  if (workspace == nullptr) cudaFreeAsync(mem, stream);
  return rc;
}

int validateMesh(const fpk_mesh_t* m) {
  if (m == nullptr || m->vertices == nullptr || m->normals == nullptr || m->faces == nullptr ||
      m->colors == nullptr) {
    return fail("fpk: mesh vertices, normals, colors and faces are required");
  }
  if (m->n_vertices <= 0 || m->n_faces <= 0) return fail("fpk: empty mesh");
  if (m->n_faces >= (1 << 24)) return fail("fpk: meshes are limited to 2^24 triangles");
  return 0;
}

}  // namespace fpb

using namespace fpb;

extern "C" {

const char* fpk_last_error(void) { return g_fpk_error.c_str(); }

void fpk_default_params(fpk_params_t* p) {
  if (p == nullptr) return;
  p->depth_min = 0.001f;
  p->depth_max = 100.0f;
  p->erosion_radius = 2;
  p->bilateral_radius = 2;
  p->depth_diff_threshold = 0.001f;
  p->erosion_ratio_threshold = 0.8f;
  p->bilateral_sigma_d = 2.0f;
  p->bilateral_sigma_r = 100000.0f;
  p->crop_ratio = 1.2f;
  p->input_width = 160;
  p->input_height = 160;
  p->rotation_normalizer_rad = 0.3490658503988659f;
  p->znear = 0.001f;
  p->zfar = 100.0f;
  p->ambient_weight = 0.8f;
  p->diffuse_weight = 0.5f;
}

int fpk_preprocess(const float* depth_raw, const uint8_t* mask, int width, int height,
                   fpk_intrinsics_t k, const fpk_params_t* p, float* depth_filtered, float* eroded,
                   float* xyz, int32_t* stats, void* stream) {
  if (validateParams(p) != 0) return 1;
  if (depth_raw == nullptr || depth_filtered == nullptr) return fail("fpk_preprocess: null depth");
  if (width <= 0 || height <= 0) return fail("fpk_preprocess: image dimensions must be positive");
  if (mask != nullptr && stats == nullptr) return fail("fpk_preprocess: stats buffer required");
  auto s = static_cast<cudaStream_t>(stream);
  if (mask != nullptr) {
    const cudaError_t e = cudaMemsetAsync(stats, 0, FPK_STATS_INTS * sizeof(int32_t), s);
    if (e != cudaSuccess) return fail(std::string("fpk_preprocess memset: ") + cudaGetErrorString(e));
  }
  const dim3 grid((width + kPreTileW - 1) / kPreTileW, (height + kPreTileH - 1) / kPreTileH);
  prof::countLaunch(prof::kPreprocess);
  prof::Scope scope(prof::kPreprocess, 20.0 * width * height, s);
  preprocessKernel<<<grid, dim3(32, 8), 0, s>>>(depth_raw, mask, width, height, k, *p,
                                                depth_filtered, eroded, xyz, stats);
  return checkLaunch("preprocessKernel");
}

int fpk_seed_poses(const int32_t* stats, const float* rotations, int n, fpk_intrinsics_t k,
                   const fpk_params_t* p, float* t0, float* poses, void* stream) {
  if (validateParams(p) != 0) return 1;
  if (stats == nullptr || (n > 0 && (rotations == nullptr || poses == nullptr))) {
    return fail("fpk_seed_poses: null buffer");
  }
  prof::countLaunch(prof::kPreprocess);
  seedPosesKernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(stats, rotations, n, k, *p,
                                                                     t0, poses);
  return checkLaunch("seedPosesKernel");
}

int fpk_crop_boxes(const float* poses, int n, fpk_intrinsics_t k, float diameter,
                   const fpk_params_t* p, float* boxes, void* stream) {
  if (validateParams(p) != 0) return 1;
  if (n <= 0) return fail("fpk_crop_boxes: n must be positive");
  prof::countLaunch(prof::kOther);
  prof::Scope scope(prof::kOther, 0.0, static_cast<cudaStream_t>(stream));
  cropBoxesKernel<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      poses, n, k, diameter, p->crop_ratio, reinterpret_cast<float4*>(boxes));
  return checkLaunch("cropBoxesKernel");
}

size_t fpk_render_workspace_bytes(int n, int n_vertices, const fpk_params_t* p) {
  if (p == nullptr || n <= 0 || n_vertices <= 0) return 0;
  return RenderWorkspace(n, n_vertices, p->input_width, p->input_height).total;
}

int fpk_render(const fpk_mesh_t* mesh, const float* poses, const float* boxes, int n,
               fpk_intrinsics_t k, const fpk_params_t* p, float* out_rgb, float* out_xyz,
               int32_t* tri_ids, void* workspace, size_t workspace_bytes, void* stream) {
  if (validateParams(p) != 0 || validateMesh(mesh) != 0) return 1;
  if (n <= 0) return fail("fpk_render: batch must be positive");
  if (poses == nullptr || boxes == nullptr || out_rgb == nullptr || out_xyz == nullptr) {
    return fail("fpk_render: null buffer");
  }
  RenderArgs a{};
  a.mesh = *mesh;
  a.poses = poses;
  a.boxes_in = boxes;
  a.n = n;
  a.k = k;
  a.p = *p;
  a.out_rgb = out_rgb;
  a.out_xyz = out_xyz;
  a.tri_ids = tri_ids;
  return launchRender<RenderOut::kNhwc>(a, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int fpk_pack(const uint8_t* rgb, const float* depth_filtered, int width, int height,
             fpk_intrinsics_t k, const fpk_params_t* p, const float* rend_rgb,
             const float* rend_xyz, const float* poses, const float* boxes, int n, float diameter,
             float invalid_depth_threshold, float* net_rendered, float* net_observed,
             void* stream) {
  if (validateParams(p) != 0) return 1;
  if (n <= 0 || width <= 0 || height <= 0) return fail("fpk_pack: bad sizes");
  RenderArgs a{};
  a.poses = poses;
  a.boxes_in = boxes;
  a.n = n;
  a.k = k;
  a.p = *p;
  a.diameter = diameter;
  a.frame_rgb = rgb;
  a.frame_depth = depth_filtered;
  a.img_w = width;
  a.img_h = height;
  a.invalid_threshold = invalid_depth_threshold;
  const long long total = static_cast<long long>(n) * p->input_width * p->input_height;
  prof::countLaunch(prof::kOther);
  packNchwKernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0,
                   static_cast<cudaStream_t>(stream)>>>(a, rend_rgb, rend_xyz, net_rendered,
                                                        net_observed);
  return checkLaunch("packNchwKernel");
}

int fpk_render_pack(const fpk_mesh_t* mesh, const float* poses, int n, const uint8_t* rgb,
                    const float* depth_filtered, int width, int height, fpk_intrinsics_t k,
                    const fpk_params_t* p, float diameter, float invalid_depth_threshold, int dtype,
                    void* net_input, long long plane_stride, float* boxes, void* workspace,
                    size_t workspace_bytes, void* stream) {
  if (validateParams(p) != 0 || validateMesh(mesh) != 0) return 1;
  if (n <= 0 || width <= 0 || height <= 0) return fail("fpk_render_pack: bad sizes");
  if ((p->input_width & 1) || (p->input_height & 1)) {
    return fail("fpk_render_pack: crop size must be even");
  }
  RenderArgs a{};
  a.mesh = *mesh;
  a.poses = poses;
  a.boxes_out = boxes;
  a.n = n;
  a.k = k;
  a.p = *p;
  a.diameter = diameter;
  a.frame_rgb = rgb;
  a.frame_depth = depth_filtered;
  a.img_w = width;
  a.img_h = height;
  a.invalid_threshold = invalid_depth_threshold;
  a.net = net_input;
  a.plane_stride = plane_stride;
  if (plane_stride % 16 != 0 || reinterpret_cast<uintptr_t>(net_input) % 16 != 0) {
    return fail("fpk_render_pack: net_input and plane_stride must be 16-byte aligned");
  }
  a.grid_w = (p->input_width + 7) / 2;
  a.grid_h = (p->input_height + 7) / 2;
  auto s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case FPK_DTYPE_F32:
      return launchRender<RenderOut::kS2dF32>(a, workspace, workspace_bytes, s);
    case FPK_DTYPE_F32_EXACT:
      return launchRender<RenderOut::kS2dF32Exact>(a, workspace, workspace_bytes, s);
    case FPK_DTYPE_F16:
      return launchRender<RenderOut::kS2dF16>(a, workspace, workspace_bytes, s);
    case FPK_DTYPE_BF16:
      return launchRender<RenderOut::kS2dBf16>(a, workspace, workspace_bytes, s);
    default:
      return fail("fpk_render_pack: unknown dtype");
  }
}

int fpk_apply_deltas(float* poses, const float* delta_t, const float* delta_r, int n,
                     float diameter, const fpk_params_t* p, void* stream) {
  if (validateParams(p) != 0) return 1;
  if (n <= 0) return fail("fpk_apply_deltas: n must be positive");
  prof::countLaunch(prof::kOther);
  prof::Scope scope(prof::kOther, 0.0, static_cast<cudaStream_t>(stream));
  applyDeltasKernel<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      poses, delta_t, delta_r, n, diameter, p->rotation_normalizer_rad);
  return checkLaunch("applyDeltasKernel");
}

int fpk_select_best(const float* poses, const float* scores, int n, const float* center3,
                    float* result, void* stream) {
  if (n <= 0 || center3 == nullptr) return fail("fpk_select_best: bad arguments");
  prof::countLaunch(prof::kOther);
  prof::Scope scope(prof::kOther, 0.0, static_cast<cudaStream_t>(stream));
  selectBestKernel<<<1, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      poses, scores, n, center3[0], center3[1], center3[2], result);
  return checkLaunch("selectBestKernel");
}

}  // extern "C"
