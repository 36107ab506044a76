// Self-attention in exact fp32 (FMA pipes, no tensor cores) for the
// strict-FP32 networks (FPK_DTYPE_F32_EXACT). The reference's FP32 engines
// disable TF32 (src/tensorrt_runner.cu:65-80), so the FP32 option here keeps
// every attention product in fp32 as well; the tensor-core kernel
// (fp_attention.cu) serves FP16 / BF16 / TF32.
//
// One CTA of 256 threads per (64-query block, layer x head, sequence):
// Q^T, K^T and V of the head (128 channels, 32 KP4 planes) are staged in
// shared memory one 64-key block at a time; each thread owns a 4 x 4 tile of
// the 64 x 64 scores and a 4-row x 8-channel tile of the output, with the
// running row maximum and sum of the online softmax kept per row and shared
// across the 16 threads of a row through shuffles.
#include <cuda_runtime.h>

#include <cmath>

#include "fp_launch.hpp"
#include "fp_net_kernels.cuh"
#include "fp_profile.hpp"
#include "fp_tc.cuh"
#include "fpk.h"

namespace fpb {
namespace attn_exact {

constexpr int kQ = 64;      // queries per CTA
constexpr int kK = 64;      // keys per block
constexpr int kD = 128;     // head dim
constexpr int kPlanes = 32;  // KP4 planes per head
constexpr int kThreads = 256;
constexpr size_t kSmem = (static_cast<size_t>(kD) * kQ + kD * kK + kK * kD + kK * kQ) * sizeof(float);

__global__ void __launch_bounds__(kThreads) attentionExactKernel(net::AttnArgs a) {
  tc::pdlTrigger();
  tc::pdlWait();
  extern __shared__ __align__(16) float sm[];
  float* qt = sm;               // [kD][kQ]  Q transposed
  float* kt = qt + kD * kQ;     // [kD][kK]  K transposed
  float* vs = kt + kD * kK;     // [kK][kD]
  float* pt = vs + kK * kD;     // [kK][kQ]  P transposed
  const int tid = threadIdx.x;
  const int ty = tid >> 4;  // score / output row group (4 rows)
  const int tx = tid & 15;  // score column group (4 keys) / output channel group (8 channels)
  const int q0 = blockIdx.x * kQ;
  const int layer = blockIdx.y / a.heads;
  const int head = blockIdx.y - layer * a.heads;
  const long long row_base = static_cast<long long>(blockIdx.z) * a.seq_len;
  const int qp = layer * a.qkv_layer_planes + a.q_plane + head * kPlanes;
  const int kp = layer * a.qkv_layer_planes + a.k_plane + head * kPlanes;
  const int vp = layer * a.qkv_layer_planes + a.v_plane + head * kPlanes;
  auto rec = [&](int plane, long long row) {
    return *reinterpret_cast<const float4*>(a.qkv + plane * a.qkv_plane_stride + row * 16);
  };
  for (int i = tid; i < kPlanes * kQ; i += kThreads) {
    const int p = i / kQ;
    const int r = i - p * kQ;
    const float4 v = q0 + r < a.seq_len ? rec(qp + p, row_base + q0 + r) : make_float4(0.f, 0.f, 0.f, 0.f);
    qt[(4 * p + 0) * kQ + r] = v.x;
    qt[(4 * p + 1) * kQ + r] = v.y;
    qt[(4 * p + 2) * kQ + r] = v.z;
    qt[(4 * p + 3) * kQ + r] = v.w;
  }
  const float scale = 1.0f / sqrtf(static_cast<float>(kD));
  float m[4], l[4], o[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) o[i][j] = 0.0f;
  }
  for (int k0 = 0; k0 < a.seq_len; k0 += kK) {
    __syncthreads();  // the previous block's K, V and P are consumed
    for (int i = tid; i < kPlanes * kK; i += kThreads) {
      const int p = i / kK;
      const int r = i - p * kK;
      const bool in = k0 + r < a.seq_len;
      const float4 kv = in ? rec(kp + p, row_base + k0 + r) : make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 vv = in ? rec(vp + p, row_base + k0 + r) : make_float4(0.f, 0.f, 0.f, 0.f);
      kt[(4 * p + 0) * kK + r] = kv.x;
      kt[(4 * p + 1) * kK + r] = kv.y;
      kt[(4 * p + 2) * kK + r] = kv.z;
      kt[(4 * p + 3) * kK + r] = kv.w;
      *reinterpret_cast<float4*>(vs + r * kD + 4 * p) = vv;
    }
    __syncthreads();
    // Scores of rows 4ty..4ty+3 against keys 4tx..4tx+3.
    float sc[4][4] = {};
#pragma unroll 4
    for (int d = 0; d < kD; ++d) {
      const float4 qa = *reinterpret_cast<const float4*>(qt + d * kQ + 4 * ty);
      const float4 kb = *reinterpret_cast<const float4*>(kt + d * kK + 4 * tx);
      const float qv[4] = {qa.x, qa.y, qa.z, qa.w};
      const float kv[4] = {kb.x, kb.y, kb.z, kb.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) sc[i][j] = fmaf(qv[i], kv[j], sc[i][j]);
    }
    // Online softmax per row: the row's 64 scores live in 16 threads.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        sc[i][j] = k0 + 4 * tx + j < a.seq_len ? sc[i][j] * scale : -INFINITY;
        mx = fmaxf(mx, sc[i][j]);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_new = fmaxf(m[i], mx);
      const float alpha = expf(m[i] - m_new);  // 0 on the first block (m = -inf)
      float rs = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float pv = expf(sc[i][j] - m_new);
        pt[(4 * tx + j) * kQ + 4 * ty + i] = pv;
        rs += pv;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
      l[i] = l[i] * alpha + rs;
      m[i] = m_new;
#pragma unroll
      for (int c = 0; c < 8; ++c) o[i][c] *= alpha;
    }
    __syncthreads();
    // O rows 4ty..4ty+3, channels 8tx..8tx+7 += P V.
#pragma unroll 4
    for (int j = 0; j < kK; ++j) {
      const float4 pa = *reinterpret_cast<const float4*>(pt + j * kQ + 4 * ty);
      const float4 v0 = *reinterpret_cast<const float4*>(vs + j * kD + 8 * tx);
      const float4 v1 = *reinterpret_cast<const float4*>(vs + j * kD + 8 * tx + 4);
      const float pv[4] = {pa.x, pa.y, pa.z, pa.w};
      const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < 8; ++c) o[i][c] = fmaf(pv[i], vv[c], o[i][c]);
    }
  }
  const int op = layer * a.out_layer_planes + head * kPlanes + 2 * tx;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = q0 + 4 * ty + i;
    if (r >= a.seq_len) continue;
    const float inv = 1.0f / l[i];
    unsigned char* dst = a.out + op * a.out_plane_stride + (row_base + r) * 16;
    *reinterpret_cast<float4*>(dst) = make_float4(o[i][0] * inv, o[i][1] * inv, o[i][2] * inv, o[i][3] * inv);
    *reinterpret_cast<float4*>(dst + a.out_plane_stride) =
        make_float4(o[i][4] * inv, o[i][5] * inv, o[i][6] * inv, o[i][7] * inv);
  }
}

}  // namespace attn_exact

namespace net {

cudaError_t launchAttentionExact(const AttnArgs& a, int layers, int n_seq, cudaStream_t s) {
  using namespace attn_exact;
  if (a.seq_len <= 0) return cudaErrorInvalidValue;
  static DeviceOnce smem_attr;
  const cudaError_t e = smem_attr.run([] {
    return cudaFuncSetAttribute(attentionExactKernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(kSmem));
  });
  if (e != cudaSuccess) return e;
  prof::countLaunch(prof::kAttention);
  return launchPdl(attentionExactKernel, dim3((a.seq_len + kQ - 1) / kQ, layers * a.heads, n_seq), dim3(kThreads),
                   kSmem, s, a);
}

}  // namespace net
}  // namespace fpb
