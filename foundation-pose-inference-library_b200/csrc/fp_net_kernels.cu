// Non-GEMM kernels of RefineNet / ScoreNet (the GEMMs live in fp_gemm.cu, the
// self-attention in fp_attention.cu). Planar activations: 16-byte records of
// 8 (fp16/bf16, "KP8") or 4 (fp32, "KP4") channels.
//
//  * layerNorm16Kernel per-row LayerNorm over 512 channels (planar -> planar),
//                      in registers for fp16/bf16; layerNormKernel (shared-memory
//                      tile) for fp32
//  * tokenMeanKernel   mean over the tokens of each sequence (planar -> fp32)
//  * linearF32Kernel / smallAttentionKernel  fp32 tail of ScoreNet (attention
//                      across hypotheses); linearFewKernel for the 512->3 /
//                      512->1 heads
//  * nchwToStemKernel  NCHW fp32 network inputs (the IInferenceRunner seam) to
//                      the stem's space-to-depth planar layout
//  * convertKernel     fp32 -> fp16/bf16 weight copies
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "fp_launch.hpp"
#include "fp_net_kernels.cuh"
#include "fpk.h"
#include "fp_profile.hpp"
#include "fp_tc.cuh"

namespace fpb {
namespace net {

template <typename T>
__device__ __forceinline__ float toF(T v);
template <>
__device__ __forceinline__ float toF<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float toF<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float toF<float>(float v) { return v; }

template <typename T>
__device__ __forceinline__ T cvt(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 cvt<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half cvt<__half>(float v) { return __float2half_rn(v); }
// fp32 network activations are TF32 tensor-core operands downstream: round
// to nearest TF32 where they are produced.
template <>
__device__ __forceinline__ float cvt<float>(float v) { return tc::tf32Round(v); }

// Conversion of a produced activation: kExact keeps fp32 values as computed
// (FPK_DTYPE_F32_EXACT, the strict-FP32 networks), else cvt<T>.
template <typename T, bool kExact>
__device__ __forceinline__ T cvtOut(float v) {
  if constexpr (kExact && sizeof(T) == 4) {
    return v;
  } else {
    return cvt<T>(v);
  }
}

// LayerNorm over 512 channels (eps inside the sqrt, biased variance, affine)
// for R rows per CTA, planar in/out: 16-byte records of 8 (fp16/bf16) or 4
// (fp32) channels.
template <typename T, int R, bool kExact = false>
__global__ void __launch_bounds__(256) layerNormKernel(LnArgs a) {
  tc::pdlTrigger();
  tc::pdlWait();
  constexpr int kPR = 16 / static_cast<int>(sizeof(T));
  constexpr int kPlanes = 512 / kPR;
  constexpr int kLd = 512 + kPR;  // padded row, keeps 16-byte records aligned
  __shared__ __align__(16) T tile[R][kLd];
  const long long r0 = static_cast<long long>(blockIdx.x) * R;
  for (int c = threadIdx.x; c < R * kPlanes; c += 256) {
    const int plane = c / R;
    const int row = c % R;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r0 + row < a.rows) {
      v = *reinterpret_cast<const uint4*>(a.in + static_cast<long long>(plane) * a.in_plane_stride +
                                          (r0 + row) * 16);
    }
    *reinterpret_cast<uint4*>(&tile[row][plane * kPR]) = v;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int rr = 0; rr < R / 8; ++rr) {
    const int row = warp * (R / 8) + rr;
    float v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = toF<T>(tile[row][lane * 16 + i]);
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) s += v[i];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    const float mean = s * (1.0f / 512.0f);
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float d = v[i] - mean;
      q += d * d;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) q += __shfl_xor_sync(0xffffffffu, q, off);
    const float rstd = rsqrtf(q * (1.0f / 512.0f) + a.eps);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int ch = lane * 16 + i;
      tile[row][ch] = cvtOut<T, kExact>((v[i] - mean) * rstd * a.gamma[ch] + a.beta[ch]);
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < R * kPlanes; c += 256) {
    const int plane = c / R;
    const int row = c % R;
    if (r0 + row < a.rows) {
      *reinterpret_cast<uint4*>(a.out + static_cast<long long>(plane) * a.out_plane_stride +
                                (r0 + row) * 16) = *reinterpret_cast<const uint4*>(&tile[row][plane * kPR]);
    }
  }
}

template <typename T>
__device__ __forceinline__ float2 toF2(uint32_t w);
template <>
__device__ __forceinline__ float2 toF2<__half>(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}
template <>
__device__ __forceinline__ float2 toF2<__nv_bfloat16>(uint32_t w) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
}
template <typename T>
__device__ __forceinline__ uint32_t fromF2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t fromF2<__half>(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t fromF2<__nv_bfloat16>(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// LayerNorm over 512 channels of 16-bit planar activations, in registers: a
// warp normalises 4 rows; lane l holds channel planes g, g+8, ..., g+56
// (g = l / 4) of row l % 4, so every warp-wide load or store moves 8 planes x
// 4 consecutive rows (64 contiguous bytes per plane), and all 8 loads of a
// lane are in flight together. Row statistics: per-lane partial sums, then a
// butterfly over the 8 lanes of the row.
template <typename T>
__global__ void __launch_bounds__(256, 2) layerNorm16Kernel(LnArgs a) {
  tc::pdlTrigger();
  __shared__ float gamma[512], beta[512];
  for (int i = threadIdx.x; i < 512; i += 256) {
    gamma[i] = a.gamma[i];
    beta[i] = a.beta[i];
  }
  __syncthreads();
  tc::pdlWait();  // weights above; activations from here on
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2;
  const long long row = (static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5)) * 4 + (lane & 3);
  const bool valid = row < a.rows;
  uint4 rec[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    rec[k] = valid ? *reinterpret_cast<const uint4*>(a.in + static_cast<long long>(g + 8 * k) * a.in_plane_stride +
                                                     row * 16)
                   : make_uint4(0, 0, 0, 0);
  }
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t w[4] = {rec[k].x, rec[k].y, rec[k].z, rec[k].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = toF2<T>(w[j]);
      s += f.x + f.y;
    }
  }
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  const float mean = s * (1.0f / 512.0f);
  float q = 0.0f;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t w[4] = {rec[k].x, rec[k].y, rec[k].z, rec[k].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = toF2<T>(w[j]);
      const float d0 = f.x - mean;
      const float d1 = f.y - mean;
      q += d0 * d0 + d1 * d1;
    }
  }
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) q += __shfl_xor_sync(0xffffffffu, q, off);
  const float rstd = rsqrtf(q * (1.0f / 512.0f) + a.eps);
  if (!valid) return;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int ch = (g + 8 * k) * 8;
    const uint32_t w[4] = {rec[k].x, rec[k].y, rec[k].z, rec[k].w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = toF2<T>(w[j]);
      const int c = ch + 2 * j;
      o[j] = fromF2<T>((f.x - mean) * rstd * gamma[c] + beta[c], (f.y - mean) * rstd * gamma[c + 1] + beta[c + 1]);
    }
    *reinterpret_cast<uint4*>(a.out + static_cast<long long>(g + 8 * k) * a.out_plane_stride + row * 16) =
        make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Mean over the seq_len rows of each sequence, 512 channels, fp32 out.
// Grid (sequences, plane groups of 8): warp w of a block owns channel plane
// 8 * blockIdx.y + w; lane l adds rows l, l + 32, ... (four rows' records in
// flight per lane, 512 contiguous bytes per warp-wide load), then a butterfly
// over the 32 lanes. A sequence's mean no longer waits on one CTA's serial
// walk over its 400 rows (the one-hypothesis passes of tracking).
template <typename T>
__global__ void __launch_bounds__(256) tokenMeanKernel(const unsigned char* __restrict__ in,
                                                       long long plane_stride, int seq_len,
                                                       float* __restrict__ out) {
  tc::pdlTrigger();
  tc::pdlWait();
  constexpr int kPR = 16 / static_cast<int>(sizeof(T));
  const int lane = threadIdx.x & 31;
  const int plane = blockIdx.y * 8 + (threadIdx.x >> 5);
  const long long base = static_cast<long long>(blockIdx.x) * seq_len;
  const unsigned char* src = in + static_cast<long long>(plane) * plane_stride + base * 16;
  float acc[kPR] = {};
  int r = lane;
  for (; r + 96 < seq_len; r += 128) {
    alignas(16) T rec[4][kPR];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      *reinterpret_cast<uint4*>(rec[u]) = *reinterpret_cast<const uint4*>(src + static_cast<long long>(r + 32 * u) * 16);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
#pragma unroll
      for (int e = 0; e < kPR; ++e) acc[e] += toF<T>(rec[u][e]);
    }
  }
  for (; r < seq_len; r += 32) {
    alignas(16) T rec[kPR];
    *reinterpret_cast<uint4*>(rec) = *reinterpret_cast<const uint4*>(src + static_cast<long long>(r) * 16);
#pragma unroll
    for (int e = 0; e < kPR; ++e) acc[e] += toF<T>(rec[e]);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
    for (int e = 0; e < kPR; ++e) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], off);
  }
  if (lane < kPR) {
    float v = acc[0];
#pragma unroll
    for (int e = 1; e < kPR; ++e) v = lane == e ? acc[e] : v;
    out[blockIdx.x * 512 + plane * kPR + lane] = v / seq_len;
  }
}

// y[m][n] = sum_k x[m][k] * w[n][k] + b[n] (+ relu) for n <= 8 outputs (the
// 512 -> 3 pose heads and the 512 -> 1 score head): one block per row, thread
// t takes k = t, t + 256, ... (coalesced row reads, every load of a thread
// issued before its products), then a butterfly per warp and the 8 warps'
// sums added in warp order.
__global__ void __launch_bounds__(256) linearFewKernel(const float* __restrict__ x, const float* __restrict__ w,
                                                       const float* __restrict__ b, float* __restrict__ y, int m,
                                                       int n, int k, int relu) {
  tc::pdlTrigger();
  tc::pdlWait();
  __shared__ float part[8][8];
  const int row = blockIdx.x;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  float acc[8] = {};
  const float* xr = x + static_cast<long long>(row) * k;
#pragma unroll 4
  for (int kk = threadIdx.x; kk < k; kk += 256) {
    const float xv = xr[kk];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j < n) acc[j] = fmaf(xv, __ldg(w + static_cast<long long>(j) * k + kk), acc[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], off);
  }
  if (lane == 0) {
#pragma unroll
    for (int j = 0; j < 8; ++j) part[warp][j] = acc[j];
  }
  __syncthreads();
  if (threadIdx.x < n) {
    float v = part[0][threadIdx.x];
#pragma unroll
    for (int q = 1; q < 8; ++q) v += part[q][threadIdx.x];
    v += b != nullptr ? b[threadIdx.x] : 0.0f;
    y[static_cast<long long>(row) * n + threadIdx.x] = relu ? fmaxf(v, 0.0f) : v;
  }
}

// y[m][n] = sum_k x[m][k] * w[n][k] + b[n] (+ relu), fp32, 32x32 output tiles.
__global__ void __launch_bounds__(256) linearF32Kernel(const float* __restrict__ x,
                                                       const float* __restrict__ w,
                                                       const float* __restrict__ b, float* __restrict__ y,
                                                       int m, int n, int k, int relu) {
  tc::pdlTrigger();
  tc::pdlWait();
  __shared__ float xs[32][33];
  __shared__ float ws[32][33];
  const int tx = threadIdx.x & 31;
  const int ty = threadIdx.x >> 5;  // 0..7, each thread 4 rows
  const int m0 = blockIdx.y * 32;
  const int n0 = blockIdx.x * 32;
  float acc[4] = {0, 0, 0, 0};
  for (int k0 = 0; k0 < k; k0 += 32) {
    for (int i = ty; i < 32; i += 8) {
      xs[i][tx] = (m0 + i < m && k0 + tx < k) ? x[(m0 + i) * k + k0 + tx] : 0.0f;
      ws[i][tx] = (n0 + i < n && k0 + tx < k) ? w[(n0 + i) * k + k0 + tx] : 0.0f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < 32; ++kk) {
      const float wv = ws[tx][kk];
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[r] += xs[ty * 4 + r][kk] * wv;
    }
    __syncthreads();
  }
  for (int r = 0; r < 4; ++r) {
    const int mm = m0 + ty * 4 + r;
    const int nn = n0 + tx;
    if (mm < m && nn < n) {
      float v = acc[r] + (b != nullptr ? b[nn] : 0.0f);
      y[mm * n + nn] = relu ? fmaxf(v, 0.0f) : v;
    }
  }
}

// Attention across one short fp32 sequence (ScoreNet's cross-hypothesis layer):
// qkv [len][3*512], 4 heads of 128; one CTA per (query, head).
__global__ void __launch_bounds__(128) smallAttentionKernel(const float* __restrict__ qkv, int len,
                                                            float* __restrict__ out) {
  tc::pdlTrigger();
  tc::pdlWait();
  extern __shared__ float sc[];
  __shared__ float red[4];
  const int i = blockIdx.x;
  const int h = blockIdx.y;
  const int t = threadIdx.x;
  const float* q = qkv + static_cast<long long>(i) * 1536 + h * 128;
  const float scale = rsqrtf(128.0f);
  for (int j = t; j < len; j += 128) {
    const float* kr = qkv + static_cast<long long>(j) * 1536 + 512 + h * 128;
    float s = 0.0f;
    for (int d = 0; d < 128; ++d) s += q[d] * kr[d];
    sc[j] = s * scale;
  }
  __syncthreads();
  float mx = -INFINITY;
  for (int j = t; j < len; j += 128) mx = fmaxf(mx, sc[j]);
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if ((t & 31) == 0) red[t >> 5] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  __syncthreads();
  float sum = 0.0f;
  for (int j = t; j < len; j += 128) {
    const float e = expf(sc[j] - mx);
    sc[j] = e;
    sum += e;
  }
  for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  if ((t & 31) == 0) red[t >> 5] = sum;
  __syncthreads();
  sum = red[0] + red[1] + red[2] + red[3];
  float acc = 0.0f;
  for (int j = 0; j < len; ++j) acc += sc[j] * qkv[static_cast<long long>(j) * 1536 + 1024 + h * 128 + t];
  out[static_cast<long long>(i) * 512 + h * 128 + t] = acc / sum;
}

// NCHW fp32 [n][6][H][W] (rendered, observed) -> stem space-to-depth KP8.
template <typename T, bool kExact = false>
__global__ void nchwToStemKernel(const float* __restrict__ rendered, const float* __restrict__ observed,
                                 int n, int H, int W, unsigned char* __restrict__ dst,
                                 long long plane_stride) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = 2LL * n * H * W;
  if (idx >= total) return;
  const int x = static_cast<int>(idx % W);
  const int y = static_cast<int>((idx / W) % H);
  const int img = static_cast<int>(idx / (static_cast<long long>(W) * H));
  const float* src = img < n ? rendered : observed;
  const int s = img < n ? img : img - n;
  const long long plane = static_cast<long long>(H) * W;
  alignas(16) T v[8];
#pragma unroll
  for (int c = 0; c < 6; ++c) {
    v[c] = cvtOut<T, kExact>(src[(static_cast<long long>(s) * 6 + c) * plane + static_cast<long long>(y) * W + x]);
  }
  v[6] = cvt<T>(0.0f);
  v[7] = cvt<T>(0.0f);
  const int gw = (W + 7) / 2;
  const int gh = (H + 7) / 2;
  const int gy = (y + 3) >> 1;
  const int gx = (x + 3) >> 1;
  const int sub = ((y + 3) & 1) * 2 + ((x + 3) & 1);
  const long long row = ((static_cast<long long>(img) * gh + gy) * gw + gx) * 16;
  // 8 channels per sub-pixel: one record (16-bit) or two planes of 4 (fp32).
  constexpr int kRecs = static_cast<int>(sizeof(T)) / 2;
#pragma unroll
  for (int q = 0; q < kRecs; ++q) {
    *reinterpret_cast<uint4*>(dst + (sub * kRecs + q) * plane_stride + row) =
        reinterpret_cast<const uint4*>(v)[q];
  }
}

// Strict-FP32 operand split of a KP4 planar activation: hi = x rounded to
// nearest TF32, lo = (x - hi) rounded to nearest TF32, over every row of the
// window [-pre, rows + post) of every plane (rows outside the activation's
// range are copied as they are, so the guard rows read by shifted
// convolution windows stay as the source has them). Three TF32 products
// hi*W_hi + hi*W_lo + lo*W_hi recover an fp32-accurate product (the dropped
// lo*W_lo term and the roundings are below fp32 rounding of the sum).
__global__ void splitTf32Kernel(const float4* __restrict__ src, long long src_stride, float4* __restrict__ hi,
                                float4* __restrict__ lo, long long dst_stride, long long rows, int planes, int pre,
                                int post) {
  const long long span = rows + pre + post;
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= span * planes) return;
  const int p = static_cast<int>(i / span);
  const long long r = i - static_cast<long long>(p) * span - pre;
  const float4 x = src[p * (src_stride / 16) + r];
  const float4 h = make_float4(tc::tf32Round(x.x), tc::tf32Round(x.y), tc::tf32Round(x.z), tc::tf32Round(x.w));
  hi[p * (dst_stride / 16) + r] = h;
  lo[p * (dst_stride / 16) + r] = make_float4(tc::tf32Round(x.x - h.x), tc::tf32Round(x.y - h.y),
                                              tc::tf32Round(x.z - h.z), tc::tf32Round(x.w - h.w));
}

// fp32 -> half-precision copy (weights).
template <typename T>
__global__ void convertKernel(const float* __restrict__ in, T* __restrict__ out, long long n) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) out[i] = cvt<T>(in[i]);
}

// ---------------------------------------------------------------------------
// Launchers.
// ---------------------------------------------------------------------------

cudaError_t launchLayerNorm(const LnArgs& a, int dtype, cudaStream_t s) {
  prof::countLaunch(prof::kOther);
  prof::Scope scope(prof::kOther, 0.0, s);
  switch (dtype) {
    case FPK_DTYPE_BF16:
      return launchPdl(layerNorm16Kernel<__nv_bfloat16>, dim3(static_cast<unsigned>((a.rows + 31) / 32)), dim3(256), 0, s, a);
    case FPK_DTYPE_F32:
      return launchPdl(layerNormKernel<float, 16>, dim3(static_cast<unsigned>((a.rows + 15) / 16)), dim3(256), 0, s, a);
    case FPK_DTYPE_F32_EXACT:
      return launchPdl(layerNormKernel<float, 16, true>, dim3(static_cast<unsigned>((a.rows + 15) / 16)), dim3(256), 0,
                       s, a);
    default:
      return launchPdl(layerNorm16Kernel<__half>, dim3(static_cast<unsigned>((a.rows + 31) / 32)), dim3(256), 0, s, a);
  }
}

cudaError_t launchTokenMean(const unsigned char* in, long long plane_stride, int seq_len, int n_seq,
                            float* out, int dtype, cudaStream_t s) {
  prof::countLaunch(prof::kOther);
  prof::Scope scope(prof::kOther, 0.0, s);
  switch (dtype) {
    case FPK_DTYPE_BF16:
      return launchPdl(tokenMeanKernel<__nv_bfloat16>, dim3(n_seq, 64 / 8), dim3(256), 0, s, in, plane_stride, seq_len, out);
    case FPK_DTYPE_F32:
    case FPK_DTYPE_F32_EXACT:
      return launchPdl(tokenMeanKernel<float>, dim3(n_seq, 128 / 8), dim3(256), 0, s, in, plane_stride, seq_len, out);
    default:
      return launchPdl(tokenMeanKernel<__half>, dim3(n_seq, 64 / 8), dim3(256), 0, s, in, plane_stride, seq_len, out);
  }
}

cudaError_t launchLinearF32(const float* x, const float* w, const float* b, float* y, int m, int n,
                            int k, bool relu, cudaStream_t s) {
  prof::countLaunch(prof::kOther);
  prof::Scope scope(prof::kOther, 0.0, s);
  if (n <= 8) {
    return launchPdl(linearFewKernel, dim3(m), dim3(256), 0, s, x, w, b, y, m, n, k, relu ? 1 : 0);
  }
  const dim3 grid((n + 31) / 32, (m + 31) / 32);
  return launchPdl(linearF32Kernel, grid, dim3(256), 0, s, x, w, b, y, m, n, k, relu ? 1 : 0);
}

cudaError_t launchSmallAttention(const float* qkv, int len, float* out, cudaStream_t s) {
  prof::countLaunch(prof::kOther);
  prof::Scope scope(prof::kOther, 0.0, s);
  return launchPdl(smallAttentionKernel, dim3(len, 4), dim3(128), static_cast<size_t>(len) * sizeof(float), s, qkv, len,
                   out);
}

cudaError_t launchNchwToStem(const float* rendered, const float* observed, int n, int H, int W,
                             void* dst, long long plane_stride, int dtype, cudaStream_t s) {
  prof::countLaunch(prof::kOther);
  prof::Scope scope(prof::kOther, 0.0, s);
  const long long total = 2LL * n * H * W;
  const unsigned grid = static_cast<unsigned>((total + 255) / 256);
  auto* d = static_cast<unsigned char*>(dst);
  switch (dtype) {
    case FPK_DTYPE_BF16:
      nchwToStemKernel<__nv_bfloat16><<<grid, 256, 0, s>>>(rendered, observed, n, H, W, d, plane_stride);
      break;
    case FPK_DTYPE_F32:
      nchwToStemKernel<float><<<grid, 256, 0, s>>>(rendered, observed, n, H, W, d, plane_stride);
      break;
    case FPK_DTYPE_F32_EXACT:
      nchwToStemKernel<float, true><<<grid, 256, 0, s>>>(rendered, observed, n, H, W, d, plane_stride);
      break;
    default:
      nchwToStemKernel<__half><<<grid, 256, 0, s>>>(rendered, observed, n, H, W, d, plane_stride);
  }
  return cudaGetLastError();
}

cudaError_t launchSplitTf32(const unsigned char* src, long long src_stride, unsigned char* hi, unsigned char* lo,
                            long long dst_stride, long long rows, int planes, int pre, int post, cudaStream_t s) {
  prof::countLaunch(prof::kOther);
  const long long total = (rows + pre + post) * planes;
  splitTf32Kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, s>>>(
      reinterpret_cast<const float4*>(src), src_stride, reinterpret_cast<float4*>(hi),
      reinterpret_cast<float4*>(lo), dst_stride, rows, planes, pre, post);
  return cudaGetLastError();
}

cudaError_t launchConvert(const float* in, void* out, long long n, bool bf16, cudaStream_t s) {
  prof::countLaunch(prof::kOther);
  const unsigned grid = static_cast<unsigned>((n + 255) / 256);
  if (bf16) {
    convertKernel<__nv_bfloat16><<<grid, 256, 0, s>>>(in, static_cast<__nv_bfloat16*>(out), n);
  } else {
    convertKernel<__half><<<grid, 256, 0, s>>>(in, static_cast<__half*>(out), n);
  }
  return cudaGetLastError();
}

}  // namespace net
}  // namespace fpb
