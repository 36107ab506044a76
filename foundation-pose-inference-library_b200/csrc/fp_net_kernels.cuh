// Launchers of the non-GEMM network kernels (fp_net_kernels.cu).
#pragma once

#include <cuda_runtime.h>

#include <cuda.h>

namespace fpb {

// 2-D TMA map over a planar activation with the rows of a plane as one
// contiguous run of 8-byte elements: dims {2 * rows, planes}, one box =
// box_rows (<= 128) rows x box_planes planes, landing as [plane][row][16 B].
// Coordinates are (2 * first row, first plane); rows outside [0, rows) read
// as zeros. Long contiguous inner runs move far faster through the TMA unit
// than boxes whose innermost dimension is one 16-byte record. Returns 0, or
// non-zero with the error recorded (fpk_last_error).
int makePlanarRowsMap(const void* base, long long rows, int planes, long long plane_stride, int box_rows,
                      int box_planes, CUtensorMap* map, const char* who);

namespace net {

// Self-attention over KP8 q/k/v planes. For layer z and head h the query /
// key / value channels are planes z*qkv_layer_planes + {q,k,v}_plane + 16h;
// the output goes to planes z*out_layer_planes + 16h. Head dim 128.
struct AttnArgs {
  const unsigned char* qkv;
  long long qkv_plane_stride;
  int qkv_layer_planes;
  int q_plane, k_plane, v_plane;
  unsigned char* out;
  long long out_plane_stride;
  int out_layer_planes;
  int seq_len;
  int heads;
  float scale_log2;  // log2(e) / sqrt(head_dim)
  int* error_flag;   // device flag set by the tensor-core kernel on a timed-out wait
};

struct LnArgs {
  const unsigned char* in;
  long long in_plane_stride;
  unsigned char* out;
  long long out_plane_stride;
  long long rows;
  const float* gamma;
  const float* beta;
  float eps;
};

// tcgen05 / TMEM attention (fp_attention.cu); dtype FPK_DTYPE_*, needs error_flag.
cudaError_t launchAttentionTc(const AttnArgs& a, int layers, int n_seq, int dtype, cudaStream_t s);
cudaError_t launchLayerNorm(const LnArgs& a, int dtype, cudaStream_t s);
cudaError_t launchTokenMean(const unsigned char* in, long long plane_stride, int seq_len, int n_seq,
                            float* out, int dtype, cudaStream_t s);
cudaError_t launchLinearF32(const float* x, const float* w, const float* b, float* y, int m, int n,
                            int k, bool relu, cudaStream_t s);
cudaError_t launchSmallAttention(const float* qkv, int len, float* out, cudaStream_t s);
cudaError_t launchNchwToStem(const float* rendered, const float* observed, int n, int H, int W,
                             void* dst, long long plane_stride, int dtype, cudaStream_t s);
cudaError_t launchConvert(const float* in, void* out, long long n, bool bf16, cudaStream_t s);
// Strict-FP32 operand split (fp_net_kernels.cu splitTf32Kernel): src, hi, lo
// point at row 0 of plane 0 of KP4 planar buffers; rows [-pre, rows + post).
cudaError_t launchSplitTf32(const unsigned char* src, long long src_stride, unsigned char* hi, unsigned char* lo,
                            long long dst_stride, long long rows, int planes, int pre, int post, cudaStream_t s);
// fp32 FMA self-attention (fp_attention_exact.cu) for FPK_DTYPE_F32_EXACT, same
// arguments and layout as launchAttentionTc with KP4 records.
cudaError_t launchAttentionExact(const AttnArgs& a, int layers, int n_seq, cudaStream_t s);

}  // namespace net
}  // namespace fpb
