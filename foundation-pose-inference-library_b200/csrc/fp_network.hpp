// RefineNet / ScoreNet on the B200 kernels (internal header).
#pragma once

#include <cuda_runtime.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

#include "fpk.h"

namespace fpb {

// Guard rows around every plane of a planar activation buffer: convolution
// windows may start up to kGuardPre rows before row 0 and end kGuardPost rows
// after the last row (both zero, never written).
constexpr long long kGuardPre = 256;
constexpr long long kGuardPost = 512;

// Device buffer in the channel-group planar layout (include/fpk.h).
struct Planar {
  void* mem = nullptr;
  unsigned char* base = nullptr;  // row 0 of plane 0
  long long plane_stride = 0;
  long long rows = 0;
  int planes = 0;
  size_t bytes = 0;
};

struct DeviceAlloc;  // owns cudaMalloc'd memory

// Flat fp32 weight pack (.fpw), see python/fp_b200/weights.py for the format.
struct WeightPack {
  int arch = -1;  // 0 refine, 1 score
  std::map<std::string, std::vector<float>> tensors;
  std::map<std::string, std::vector<int>> shapes;
  static WeightPack load(const std::string& path);
  const std::vector<float>& at(const std::string& name) const;
};

enum class NetPrecision { kFP32 = 0, kTF32 = 1, kFP16 = 2, kBF16 = 3 };

struct ConvLayer {
  void* w = nullptr;       // [cout][K'] in the activation type, chunk-major
  void* w_lo = nullptr;    // strict FP32: the weights' TF32 remainder (w - w rounded), same layout
  float* bias = nullptr;   // [cout]
  int cin = 0, cout = 0, taps = 0;
  int tap_off[FPK_GEMM_MAX_TAPS] = {};
  double flops_per_row = 0.0;  // algorithmic FLOPs per valid output row (un-padded op)
};

class Network;

// Owns both networks, their shared activation workspace and the stem input
// buffer that the fused render+pack kernel writes.
class NetworkRunner {
 public:
  NetworkRunner(const std::string& refine_path, const std::string& score_path,
                NetPrecision precision, int max_batch, int crop_w, int crop_h);
  ~NetworkRunner();
  NetworkRunner(const NetworkRunner&) = delete;
  NetworkRunner& operator=(const NetworkRunner&) = delete;

  // Stem input for `n` hypotheses (images 0..n-1 rendered, n..2n-1 observed,
  // grouped per micro-batch chunk: see stemImage()).
  const Planar& stem() const { return stem_; }
  int dtype() const;      // FPK_DTYPE_F16 / FPK_DTYPE_BF16 / FPK_DTYPE_F32 (FP32 and TF32)
  int perRecord() const;  // channels per 16-byte activation record: 8, or 4 for fp32
  NetPrecision precision() const { return precision_; }
  int maxBatch() const { return max_batch_; }

  // RefineNet on images [2*first, 2*(first+count)) of the stem buffer laid out
  // as chunks of `count` (rendered block then observed block).
  void refine(int count, int first_chunk, float* delta_t, float* delta_r, cudaStream_t s);
  // ScoreNet over all n hypotheses (stem laid out as one chunk of n).
  void score(int n, float* scores, cudaStream_t s);
  // ScoreNet split at its one cross-hypothesis step, for sharded registers:
  // the per-hypothesis part (encoder, token self-attention, token mean) writes
  // 512 fp32 features per hypothesis; the head attends across all n of them
  // (features gathered from every shard) and writes n scores.
  void scoreFeatures(int n, float* features, cudaStream_t s);
  void scoreHead(int n, const float* features, float* scores, cudaStream_t s);
  static constexpr int kFeatureDim = 512;
  // NCHW fp32 inputs (IInferenceRunner seam) -> stem buffer, one chunk of n.
  void loadNchw(const float* rendered, const float* observed, int n, cudaStream_t s);
  // Device error flag of the pipelined kernels (0 = ok).
  int* errorFlag() const { return err_; }
  // After a pipeline timeout has been reported: zero the error flag.
  void clearError(cudaStream_t s);
  // Algorithmic FLOPs of one forward per hypothesis (for rooflines).
  double refineFlopsPerHyp() const;
  double scoreFlopsPerHyp() const;

 private:
  struct Act;
  void encoder(const Network& net, int n, long long stem_row0, cudaStream_t s);
  void gemm(const ConvLayer& L, const Planar& a, long long a_row0, long long rows, const Planar& dst,
            int mode, int img_rows, int grid_w, int valid_h, int valid_w, bool relu,
            const Planar* residual, int dst_img_rows, int dst_grid_w, int img_mod, int ch_step,
            const float* pos, cudaStream_t s, long long dst_row0 = 0, int a_plane0 = 0);

  NetPrecision precision_;
  int max_batch_;
  int crop_w_, crop_h_;
  std::unique_ptr<Network> refine_;
  std::unique_ptr<Network> score_;
  std::vector<void*> allocations_;
  Planar stem_;
  std::unique_ptr<Act> act_;
  int* err_ = nullptr;
  // Split-K scratch for one-hypothesis passes (track): layers of a single
  // image pair fill a few SMs per tile row, so their K range is split across
  // CTAs (see fpk_gemm_desc_t). Batched passes never split, which keeps every
  // hypothesis's result independent of the batch it runs in.
  void* splitk_ = nullptr;
  long long splitk_bytes_ = 0;
  bool split_k_ = false;
  // Strict FP32 (precision kFP32): each layer runs as three TF32 GEMMs of
  // split operands, hi*W_hi + hi*W_lo + lo*W_hi; the split activation and the
  // two partial sums live here (bytes each; 0 for the other precisions).
  void* split_hi_ = nullptr;
  void* split_lo_ = nullptr;
  void* partial_[2] = {nullptr, nullptr};
  size_t split_bytes_ = 0, partial_bytes_ = 0;
  void exactGemm(const fpk_gemm_desc_t& d, const ConvLayer& L, cudaStream_t s);
};

}  // namespace fpb
