// Non-GEMM kernels of RefineNet / ScoreNet (the GEMMs live in fp_gemm.cu).
//
//  * attentionKernel   fused softmax(Q K^T / sqrt(d)) V over one sequence per
//                      (query block, layer*head, sequence); online softmax,
//                      bf16/fp16 tensor-core mma.sync tiles, KP8 in and out
//  * layerNormKernel   per-row LayerNorm over 512 channels (KP8 -> KP8)
//  * tokenMeanKernel   mean over the tokens of each sequence (KP8 -> fp32)
//  * linearF32Kernel / smallAttentionKernel  fp32 tail of ScoreNet (attention
//                      across hypotheses) and the 512->3 / 512->1 heads
//  * nchwToStemKernel  NCHW fp32 network inputs (the IInferenceRunner seam) to
//                      the stem's space-to-depth KP8 layout
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "fp_net_kernels.cuh"
#include "fp_profile.hpp"

namespace fpb {
namespace net {

template <typename T>
struct MmaTraits;

template <>
struct MmaTraits<__nv_bfloat16> {
  __device__ static __forceinline__ void mma(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ static __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ static __forceinline__ float2 unpack(uint32_t v) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v));
  }
};

template <>
struct MmaTraits<__half> {
  __device__ static __forceinline__ void mma(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ static __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ static __forceinline__ float2 unpack(uint32_t v) {
    return __half22float2(*reinterpret_cast<const __half2*>(&v));
  }
};

__device__ __forceinline__ void ldsm4(uint32_t* r, const void* p) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

__device__ __forceinline__ void ldsm4t(uint32_t* r, const void* p) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

constexpr int kHeadDim = 128;
constexpr int kQBlock = 64;
constexpr int kKBlock = 64;
constexpr int kLd = kHeadDim + 8;  // padded smem row (elements): conflict-free ldmatrix

// Copies a [64 rows x 128 channels] tile (16 KP8 planes) into padded smem rows;
// rows >= valid are zero-filled.
template <typename T>
__device__ __forceinline__ void loadTile(T* sm, const unsigned char* base, long long plane_stride,
                                         int plane0, long long row0, int valid) {
  for (int c = threadIdx.x; c < 64 * 16; c += 128) {
    const int plane = c >> 6;
    const int row = c & 63;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row < valid) {
      v = *reinterpret_cast<const uint4*>(base + static_cast<long long>(plane0 + plane) * plane_stride +
                                          (row0 + row) * 16);
    }
    *reinterpret_cast<uint4*>(sm + row * kLd + plane * 8) = v;
  }
}

template <typename T>
__global__ void __launch_bounds__(128) attentionKernel(AttnArgs a) {
  using Tr = MmaTraits<T>;
  extern __shared__ __align__(16) unsigned char smem[];
  T* qs = reinterpret_cast<T*>(smem);
  T* ks = qs + kQBlock * kLd;
  T* vs = ks + kKBlock * kLd;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2;
  const int tq = lane & 3;
  const int q0 = blockIdx.x * kQBlock;
  const int layer = blockIdx.y / a.heads;
  const int head = blockIdx.y - layer * a.heads;
  const long long row_base = static_cast<long long>(blockIdx.z) * a.seq_len;
  const int qp = layer * a.qkv_layer_planes + a.q_plane + head * 16;
  const int kp = layer * a.qkv_layer_planes + a.k_plane + head * 16;
  const int vp = layer * a.qkv_layer_planes + a.v_plane + head * 16;

  loadTile(qs, a.qkv, a.qkv_plane_stride, qp, row_base + q0, a.seq_len - q0);
  __syncthreads();
  uint32_t qa[8][4];
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    ldsm4(qa[kk], qs + (warp * 16 + (lane & 15)) * kLd + kk * 16 + (lane >> 4) * 8);
  }
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;

  const int nkb = (a.seq_len + kKBlock - 1) / kKBlock;
  for (int kb = 0; kb < nkb; ++kb) {
    const int k0 = kb * kKBlock;
    __syncthreads();
    loadTile(ks, a.qkv, a.qkv_plane_stride, kp, row_base + k0, a.seq_len - k0);
    loadTile(vs, a.qkv, a.qkv_plane_stride, vp, row_base + k0, a.seq_len - k0);
    __syncthreads();
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b[4];
        ldsm4(b, ks + (np * 16 + (lane & 7) + (lane >> 4) * 8) * kLd + kk * 16 + ((lane >> 3) & 1) * 8);
        Tr::mma(s[2 * np], qa[kk], b[0], b[1]);
        Tr::mma(s[2 * np + 1], qa[kk], b[2], b[3]);
      }
    }
    // Scale into the log2 domain and mask keys past the sequence end.
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int key = k0 + j * 8 + 2 * tq;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const bool valid = key + (e & 1) < a.seq_len;
        s[j][e] = valid ? s[j][e] * a.scale_log2 : -INFINITY;
      }
      mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
      mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float alpha0 = exp2f(m0 - mx0);
    const float alpha1 = exp2f(m1 - mx1);
    m0 = mx0;
    m1 = mx1;
    float sum0 = 0.0f, sum1 = 0.0f;
    uint32_t pa[4][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float p0 = exp2f(s[j][0] - m0);
      const float p1 = exp2f(s[j][1] - m0);
      const float p2 = exp2f(s[j][2] - m1);
      const float p3 = exp2f(s[j][3] - m1);
      sum0 += p0 + p1;
      sum1 += p2 + p3;
      pa[j >> 1][(j & 1) * 2 + 0] = Tr::pack(p0, p1);
      pa[j >> 1][(j & 1) * 2 + 1] = Tr::pack(p2, p3);
    }
    l0 = l0 * alpha0 + sum0;
    l1 = l1 * alpha1 + sum1;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= alpha0;
      o[j][1] *= alpha0;
      o[j][2] *= alpha1;
      o[j][3] *= alpha1;
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        uint32_t b[4];
        ldsm4t(b, vs + (kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * kLd + dp * 16 + (lane >> 4) * 8);
        Tr::mma(o[2 * dp], pa[kk], b[0], b[1]);
        Tr::mma(o[2 * dp + 1], pa[kk], b[2], b[3]);
      }
    }
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = 1.0f / l0;
  const float inv1 = 1.0f / l1;
  __syncthreads();
  // Stage O (normalised) in the Q tile, then store 16-byte records per plane.
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int col = j * 8 + 2 * tq;
    *reinterpret_cast<uint32_t*>(qs + (warp * 16 + g) * kLd + col) = Tr::pack(o[j][0] * inv0, o[j][1] * inv0);
    *reinterpret_cast<uint32_t*>(qs + (warp * 16 + g + 8) * kLd + col) = Tr::pack(o[j][2] * inv1, o[j][3] * inv1);
  }
  __syncthreads();
  const int op = layer * a.out_layer_planes + head * 16;
  for (int c = threadIdx.x; c < 64 * 16; c += 128) {
    const int plane = c >> 6;
    const int row = c & 63;
    if (q0 + row < a.seq_len) {
      *reinterpret_cast<uint4*>(a.out + static_cast<long long>(op + plane) * a.out_plane_stride +
                                (row_base + q0 + row) * 16) =
          *reinterpret_cast<const uint4*>(qs + row * kLd + plane * 8);
    }
  }
}

// LayerNorm over 512 channels for 32 rows per CTA (eps inside the sqrt, biased
// variance, affine), KP8 in/out.
template <typename T>
__global__ void __launch_bounds__(256) layerNormKernel(LnArgs a) {
  using Tr = MmaTraits<T>;
  __shared__ __align__(16) T tile[32][512 + 8];
  const long long r0 = static_cast<long long>(blockIdx.x) * 32;
  for (int c = threadIdx.x; c < 32 * 64; c += 256) {
    const int plane = c >> 5;
    const int row = c & 31;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r0 + row < a.rows) {
      v = *reinterpret_cast<const uint4*>(a.in + static_cast<long long>(plane) * a.in_plane_stride +
                                          (r0 + row) * 16);
    }
    *reinterpret_cast<uint4*>(&tile[row][plane * 8]) = v;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int rr = 0; rr < 4; ++rr) {
    const int row = warp * 4 + rr;
    float v[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float2 f = Tr::unpack(*reinterpret_cast<const uint32_t*>(&tile[row][lane * 16 + 2 * i]));
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
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
    for (int i = 0; i < 8; ++i) {
      const int ch = lane * 16 + 2 * i;
      const float y0 = (v[2 * i] - mean) * rstd * a.gamma[ch] + a.beta[ch];
      const float y1 = (v[2 * i + 1] - mean) * rstd * a.gamma[ch + 1] + a.beta[ch + 1];
      *reinterpret_cast<uint32_t*>(&tile[row][ch]) = Tr::pack(y0, y1);
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < 32 * 64; c += 256) {
    const int plane = c >> 5;
    const int row = c & 31;
    if (r0 + row < a.rows) {
      *reinterpret_cast<uint4*>(a.out + static_cast<long long>(plane) * a.out_plane_stride +
                                (r0 + row) * 16) = *reinterpret_cast<const uint4*>(&tile[row][plane * 8]);
    }
  }
}

// Mean over the seq_len rows of each sequence, 512 channels, fp32 out.
template <typename T>
__global__ void __launch_bounds__(256) tokenMeanKernel(const unsigned char* __restrict__ in,
                                                       long long plane_stride, int seq_len,
                                                       float* __restrict__ out) {
  using Tr = MmaTraits<T>;
  __shared__ float part[4][512];
  const int plane = threadIdx.x >> 2;
  const int sub = threadIdx.x & 3;
  const long long base = static_cast<long long>(blockIdx.x) * seq_len;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int r = sub; r < seq_len; r += 4) {
    const uint4 u = *reinterpret_cast<const uint4*>(in + static_cast<long long>(plane) * plane_stride +
                                                    (base + r) * 16);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = Tr::unpack(w[i]);
      acc[2 * i] += f.x;
      acc[2 * i + 1] += f.y;
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) part[sub][plane * 8 + e] = acc[e];
  __syncthreads();
  for (int c = threadIdx.x; c < 512; c += 256) {
    out[blockIdx.x * 512 + c] = (((part[0][c] + part[1][c]) + part[2][c]) + part[3][c]) / seq_len;
  }
}

// y[m][n] = sum_k x[m][k] * w[n][k] + b[n] (+ relu), fp32, 32x32 output tiles.
__global__ void __launch_bounds__(256) linearF32Kernel(const float* __restrict__ x,
                                                       const float* __restrict__ w,
                                                       const float* __restrict__ b, float* __restrict__ y,
                                                       int m, int n, int k, int relu) {
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

template <typename T>
__device__ __forceinline__ T cvt(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 cvt<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half cvt<__half>(float v) { return __float2half_rn(v); }

// NCHW fp32 [n][6][H][W] (rendered, observed) -> stem space-to-depth KP8.
template <typename T>
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
  for (int c = 0; c < 6; ++c) v[c] = cvt<T>(src[(static_cast<long long>(s) * 6 + c) * plane + static_cast<long long>(y) * W + x]);
  v[6] = cvt<T>(0.0f);
  v[7] = cvt<T>(0.0f);
  const int gw = (W + 7) / 2;
  const int gh = (H + 7) / 2;
  const int gy = (y + 3) >> 1;
  const int gx = (x + 3) >> 1;
  const int sub = ((y + 3) & 1) * 2 + ((x + 3) & 1);
  *reinterpret_cast<uint4*>(dst + sub * plane_stride + ((static_cast<long long>(img) * gh + gy) * gw + gx) * 16) =
      *reinterpret_cast<const uint4*>(v);
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

cudaError_t launchAttention(const AttnArgs& a, int layers, int n_seq, bool bf16, cudaStream_t s) {
  const size_t smem = 3 * kQBlock * kLd * 2;
  const dim3 grid((a.seq_len + kQBlock - 1) / kQBlock, layers * a.heads, n_seq);
  prof::countLaunch(prof::kAttention);
  static int attr_mask = 0;  // one bit per device: dynamic smem opt-in done
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 31 && !(attr_mask & (1 << dev))) {
    cudaFuncSetAttribute(attentionKernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
    cudaFuncSetAttribute(attentionKernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
    attr_mask |= 1 << dev;
  }
  if (bf16) {
    attentionKernel<__nv_bfloat16><<<grid, 128, smem, s>>>(a);
  } else {
    attentionKernel<__half><<<grid, 128, smem, s>>>(a);
  }
  return cudaGetLastError();
}

cudaError_t launchLayerNorm(const LnArgs& a, bool bf16, cudaStream_t s) {
  prof::countLaunch(prof::kOther);
  const int grid = static_cast<int>((a.rows + 31) / 32);
  if (bf16) {
    layerNormKernel<__nv_bfloat16><<<grid, 256, 0, s>>>(a);
  } else {
    layerNormKernel<__half><<<grid, 256, 0, s>>>(a);
  }
  return cudaGetLastError();
}

cudaError_t launchTokenMean(const unsigned char* in, long long plane_stride, int seq_len, int n_seq,
                            float* out, bool bf16, cudaStream_t s) {
  prof::countLaunch(prof::kOther);
  if (bf16) {
    tokenMeanKernel<__nv_bfloat16><<<n_seq, 256, 0, s>>>(in, plane_stride, seq_len, out);
  } else {
    tokenMeanKernel<__half><<<n_seq, 256, 0, s>>>(in, plane_stride, seq_len, out);
  }
  return cudaGetLastError();
}

cudaError_t launchLinearF32(const float* x, const float* w, const float* b, float* y, int m, int n,
                            int k, bool relu, cudaStream_t s) {
  prof::countLaunch(prof::kOther);
  const dim3 grid((n + 31) / 32, (m + 31) / 32);
  linearF32Kernel<<<grid, 256, 0, s>>>(x, w, b, y, m, n, k, relu ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t launchSmallAttention(const float* qkv, int len, float* out, cudaStream_t s) {
  prof::countLaunch(prof::kOther);
  smallAttentionKernel<<<dim3(len, 4), 128, static_cast<size_t>(len) * sizeof(float), s>>>(qkv, len, out);
  return cudaGetLastError();
}

cudaError_t launchNchwToStem(const float* rendered, const float* observed, int n, int H, int W,
                             void* dst, long long plane_stride, bool bf16, cudaStream_t s) {
  prof::countLaunch(prof::kOther);
  const long long total = 2LL * n * H * W;
  const unsigned grid = static_cast<unsigned>((total + 255) / 256);
  if (bf16) {
    nchwToStemKernel<__nv_bfloat16><<<grid, 256, 0, s>>>(rendered, observed, n, H, W,
                                                         static_cast<unsigned char*>(dst), plane_stride);
  } else {
    nchwToStemKernel<__half><<<grid, 256, 0, s>>>(rendered, observed, n, H, W,
                                                  static_cast<unsigned char*>(dst), plane_stride);
  }
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
