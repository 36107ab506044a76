// Device helpers shared by the pipeline kernels.
//
// Parity note: the rasterizer's triangle ids and the preprocess outputs must be
// bit-identical to the reference build. Every floating-point expression below is
// therefore written in the same operand order and grouping as the reference
// source it cites, so nvcc contracts it into the same FMAs; do not "simplify"
// these expressions (hoisting a reciprocal, reassociating a sum) without
// re-running the GPU parity tests against the reference kernels.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "fpk.h"

namespace fpb {

// reference src/cuda_pipeline.cu:30-32
__device__ __forceinline__ bool validDepth(float z, float dmin, float dmax) {
  return isfinite(z) && z >= dmin && z < dmax;
}

// reference src/cuda_pipeline.cu:329-368 (cropBoxesKernel body for one pose).
__device__ __forceinline__ float4 cropBox(const float* pose, fpk_intrinsics_t k, float diameter,
                                          float crop_ratio) {
  const float3 center = make_float3(pose[3], pose[7], pose[11]);
  const float radius = diameter * crop_ratio * 0.5f;
  const float3 offsets[5] = {make_float3(0.0f, 0.0f, 0.0f), make_float3(radius, 0.0f, 0.0f),
                             make_float3(-radius, 0.0f, 0.0f), make_float3(0.0f, radius, 0.0f),
                             make_float3(0.0f, -radius, 0.0f)};
  float center_u = 0.0f;
  float center_v = 0.0f;
  float radius_px = 1.0f;
#pragma unroll
  for (int j = 0; j < 5; ++j) {
    const float3 p = make_float3(center.x + offsets[j].x, center.y + offsets[j].y,
                                 center.z + offsets[j].z);
    const float inv_z = fabsf(p.z) > 1e-12f ? 1.0f / p.z : 0.0f;
    const float u = k.fx * p.x * inv_z + k.cx;
    const float v = k.fy * p.y * inv_z + k.cy;
    if (j == 0) {
      center_u = u;
      center_v = v;
    } else {
      radius_px = fmaxf(radius_px, fabsf(u - center_u));
      radius_px = fmaxf(radius_px, fabsf(v - center_v));
    }
  }
  return make_float4(roundf(center_u - radius_px), roundf(center_v - radius_px),
                     roundf(center_u + radius_px), roundf(center_v + radius_px));
}

// reference src/raster_kernels.cuh:324-330 normalize3 (+z fallback).
__device__ __forceinline__ float3 normalize3(float3 v) {
  const float n = sqrtf(fmaxf(v.x * v.x + v.y * v.y + v.z * v.z, 0.0f));
  if (n < 1e-12f) {
    return make_float3(0.0f, 0.0f, 1.0f);
  }
  return make_float3(v.x / n, v.y / n, v.z / n);
}

// Per-hypothesis render constants kept in shared memory.
struct HypState {
  float pose[12];
  float4 box;
};

// reference src/raster_kernels.cuh:358-360 (object -> camera).
__device__ __forceinline__ float3 camPosition(const float* pose, float3 p) {
  return make_float3(pose[0] * p.x + pose[1] * p.y + pose[2] * p.z + pose[3],
                     pose[4] * p.x + pose[5] * p.y + pose[6] * p.z + pose[7],
                     pose[8] * p.x + pose[9] * p.y + pose[10] * p.z + pose[11]);
}

// reference src/raster_kernels.cuh:361-364 (rotated, normalised normal).
__device__ __forceinline__ float3 camNormal(const float* pose, float3 n) {
  return normalize3(make_float3(pose[0] * n.x + pose[1] * n.y + pose[2] * n.z,
                                pose[4] * n.x + pose[5] * n.y + pose[6] * n.z,
                                pose[8] * n.x + pose[9] * n.y + pose[10] * n.z));
}

// reference src/raster_kernels.cuh:368-379 (camera -> crop-box clip space).
__device__ __forceinline__ float4 clipPosition(float3 cam, float4 box, fpk_intrinsics_t k,
                                               float znear, float zfar) {
  const float z = fmaxf(cam.z, znear);
  const float u = k.fx * cam.x / z + k.cx;
  const float v = k.fy * cam.y / z + k.cy;
  const float crop_w = fmaxf(box.z - box.x, 1.0f);
  const float crop_h = fmaxf(box.w - box.y, 1.0f);
  const float ndc_x = 2.0f * (u - box.x) / crop_w - 1.0f;
  const float ndc_y = 1.0f - 2.0f * (v - box.y) / crop_h;
  const float depth = zfar - znear;
  const float clip_z = ((zfar + znear) / depth) * z - (2.0f * zfar * znear / depth);
  return make_float4(ndc_x * z, ndc_y * z, clip_z, z);
}

__device__ __forceinline__ float3 loadF3(const float* a, int i) {
  return make_float3(__ldg(a + 3 * i), __ldg(a + 3 * i + 1), __ldg(a + 3 * i + 2));
}

// reference src/builtin_raster_renderer.cu:28-33 packDepthKey.
__device__ __forceinline__ unsigned long long packDepthKey(float zw, int tri_plus_one) {
  const float d01 = fminf(fmaxf(zw * 0.5f + 0.5f, 0.0f), 1.0f);
  const unsigned int depth_bits = __float_as_uint(d01);
  return (static_cast<unsigned long long>(depth_bits) << 32) |
         static_cast<unsigned int>(tri_plus_one);
}

}  // namespace fpb
