// TEST / BENCHMARK INFRASTRUCTURE ONLY (not product code).
//
// Stand-in for the reference's TensorRtRunner (declared in the reference's own
// include/foundation_pose_nvidia/tensorrt_runner.hpp, implemented there in
// src/tensorrt_runner.cu on TensorRT 10, which is not installed here). It lets
// oracle/Makefile link the reference's unmodified estimator, C ABI, pipeline
// kernels and rasterizer (src/foundation_pose.cpp, c_api.cpp, cuda_pipeline.cu,
// builtin_raster_renderer.cu, ...) into oracle/_ref/libfpref_full.so, so the
// reference's whole fp_register_frame / fp_track_frame -- its sequencing, its
// kernels, its synchronisation points -- can be timed on the same B200 as this
// build. Only the network engines differ: each enqueue calls a callback that
// the host program registers (bench.py runs RefineNet / ScoreNet as torch/cuDNN
// networks on the same weight pack, on the stream passed in).
//
// Behaviour kept from the reference runner (src/tensorrt_runner.cu:445-532):
//  - the micro-batch is min(batch_size, max_batch) and must divide max_batch;
//  - RefineNet runs in chunks of that micro-batch with a host synchronisation
//    of the stream between chunks;
//  - ScoreNet always runs the whole batch.
#include <algorithm>
#include <cstddef>
#include <string>

#include "foundation_pose_nvidia/exception.hpp"
#include "foundation_pose_nvidia/tensorrt_runner.hpp"

extern "C" {
typedef int (*refnet_refine_fn)(const float* rendered, const float* observed, float* delta_t,
                                float* delta_r, int batch, void* stream);
typedef int (*refnet_score_fn)(const float* rendered, const float* observed, float* scores, int batch,
                               void* stream);
}

namespace {
refnet_refine_fn g_refine = nullptr;
refnet_score_fn g_score = nullptr;
}  // namespace

extern "C" void refnet_set_callbacks(refnet_refine_fn refine, refnet_score_fn score) {
  g_refine = refine;
  g_score = score;
}

namespace foundation_pose_nvidia {

class TensorRtRunner::Engine {};

TensorRtRunner::TensorRtRunner(RuntimeOptions options, Config config, int max_batch)
    : options_(std::move(options)), config_(config), max_batch_(max_batch) {
  const int requested = config.batch_size > 0 ? config.batch_size : max_batch;
  engine_batch_ = std::min(max_batch, requested);
  if (engine_batch_ > 0 && max_batch % engine_batch_ != 0) {
    throw FoundationPoseError("max_batch (" + std::to_string(max_batch) + ") must be divisible by effective_bs (" +
                              std::to_string(engine_batch_) + ")");
  }
  if (max_batch_ <= 0 || engine_batch_ <= 0) {
    throw FoundationPoseError("TensorRT runner requires a positive batch size");
  }
  checkCuda(cudaSetDevice(options_.device_id), "cudaSetDevice");
}

TensorRtRunner::~TensorRtRunner() = default;

void TensorRtRunner::prepareForBatch(int batch_size) {
  if (batch_size <= 0 || batch_size > max_batch_) {
    throw FoundationPoseError("TensorRT prepare batch size exceeds configured maximum");
  }
  if (g_refine == nullptr || g_score == nullptr) {
    throw FoundationPoseError("network stand-in: refnet_set_callbacks was not called");
  }
}

void TensorRtRunner::enqueueRefine(const float* rendered, const float* observed, float* delta_translation,
                                   float* delta_rotation, int batch_size, cudaStream_t stream) {
  if (batch_size <= 0 || batch_size > max_batch_) {
    throw FoundationPoseError("TensorRT refine batch size exceeds configured maximum");
  }
  if (g_refine == nullptr) throw FoundationPoseError("network stand-in: no RefineNet callback");
  const std::size_t stride =
      static_cast<std::size_t>(config_.n_channels) * config_.input_height * config_.input_width;
  for (int off = 0; off < batch_size; off += engine_batch_) {
    const int chunk = std::min(engine_batch_, batch_size - off);
    if (g_refine(rendered + off * stride, observed + off * stride, delta_translation + 3 * off,
                 delta_rotation + 3 * off, chunk, stream) != 0) {
      throw FoundationPoseError("network stand-in: RefineNet callback failed");
    }
    if (off + chunk < batch_size) {
      checkCuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize TensorRT refine chunk");
    }
  }
}

void TensorRtRunner::enqueueScore(const float* rendered, const float* observed, float* scores, int batch_size,
                                  cudaStream_t stream) {
  if (batch_size <= 0 || batch_size > max_batch_) {
    throw FoundationPoseError("TensorRT score batch size exceeds configured maximum");
  }
  if (g_score == nullptr) throw FoundationPoseError("network stand-in: no ScoreNet callback");
  if (g_score(rendered, observed, scores, batch_size, stream) != 0) {
    throw FoundationPoseError("network stand-in: ScoreNet callback failed");
  }
}

}  // namespace foundation_pose_nvidia
