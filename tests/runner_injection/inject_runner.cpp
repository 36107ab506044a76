// Test program (built by tests/test_runner_injection.py): drives the C++ seam
// of libfoundation_pose_nvidia.so the way an application that brings its own
// inference backend does (reference include/foundation_pose_nvidia/
// foundation_pose.hpp:27-31). A caller-defined IInferenceRunner -- here one
// that counts its calls and forwards them to the library's TensorRtRunner --
// and the library's BuiltinRasterRenderer are injected through
// FoundationPose(PreprocessedMesh, RuntimeOptions, unique_ptr<IInferenceRunner>,
// unique_ptr<IRenderer>, Config); the same frame is also registered on an
// estimator built with createFromCadFile (built-in backends, fused path).
// Prints one JSON line.
//
// usage: inject_runner <obj> <refine.fpw> <score.fpw> <frame.bin> <n_hyp> <n_refine> <precision>
// frame.bin: int32 width, height; float32 K[9]; rgb u8[h*w*3]; depth f32[h*w]; mask u8[h*w]
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <memory>
#include <string>
#include <vector>

#include "foundation_pose_nvidia/builtin_raster_renderer.hpp"
#include "foundation_pose_nvidia/exception.hpp"
#include "foundation_pose_nvidia/foundation_pose.hpp"
#include "foundation_pose_nvidia/mesh.hpp"
#include "foundation_pose_nvidia/tensorrt_runner.hpp"

using namespace foundation_pose_nvidia;

namespace {

class CountingRunner final : public IInferenceRunner {
 public:
  explicit CountingRunner(std::unique_ptr<IInferenceRunner> inner) : inner_(std::move(inner)) {}
  void prepareForBatch(int batch_size) override {
    ++prepares;
    inner_->prepareForBatch(batch_size);
  }
  void enqueueRefine(const float* rendered, const float* observed, float* dt, float* dr, int batch,
                     cudaStream_t stream) override {
    ++refines;
    refine_items += batch;
    inner_->enqueueRefine(rendered, observed, dt, dr, batch, stream);
  }
  void enqueueScore(const float* rendered, const float* observed, float* scores, int batch,
                    cudaStream_t stream) override {
    ++scores_calls;
    score_items += batch;
    inner_->enqueueScore(rendered, observed, scores, batch, stream);
  }
  int prepares = 0, refines = 0, refine_items = 0, scores_calls = 0, score_items = 0;

 private:
  std::unique_ptr<IInferenceRunner> inner_;
};

void printPose(const char* key, const PoseEstimate& e) {
  std::printf("\"%s\": [", key);
  for (int i = 0; i < 16; ++i) std::printf("%s%.9g", i ? ", " : "", e.pose.values[static_cast<std::size_t>(i)]);
  std::printf("], \"%s_score\": %.9g", key, e.score);
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 8) {
    std::fprintf(stderr, "usage: inject_runner obj refine score frame n_hyp n_refine precision\n");
    return 2;
  }
  try {
    std::ifstream in(argv[4], std::ios::binary);
    int wh[2];
    float k[9];
    in.read(reinterpret_cast<char*>(wh), sizeof(wh));
    in.read(reinterpret_cast<char*>(k), sizeof(k));
    const std::size_t px = static_cast<std::size_t>(wh[0]) * wh[1];
    std::vector<std::uint8_t> rgb(px * 3), mask(px);
    std::vector<float> depth(px);
    in.read(reinterpret_cast<char*>(rgb.data()), static_cast<std::streamsize>(rgb.size()));
    in.read(reinterpret_cast<char*>(depth.data()), static_cast<std::streamsize>(depth.size() * 4));
    in.read(reinterpret_cast<char*>(mask.data()), static_cast<std::streamsize>(mask.size()));
    if (!in) throw FoundationPoseError("short frame file");

    Config cfg;
    cfg.n_hypotheses = std::atoi(argv[5]);
    cfg.batch_size = cfg.n_hypotheses;
    cfg.tensorrt_precision = static_cast<TensorrtPrecision>(std::atoi(argv[7]));
    cfg.max_image_width = wh[0];
    cfg.max_image_height = wh[1];
    RuntimeOptions opts;
    opts.refine_model_path = argv[2];
    opts.score_model_path = argv[3];
    const int n_refine = std::atoi(argv[6]);
    const CameraIntrinsics K = CameraIntrinsics::fromRowMajor(k);

    auto runner = std::make_unique<CountingRunner>(std::make_unique<TensorRtRunner>(opts, cfg, cfg.n_hypotheses));
    CountingRunner* counts = runner.get();
    FoundationPose injected(preprocessMesh(loadMesh(argv[1]), cfg), opts, std::move(runner),
                            std::make_unique<BuiltinRasterRenderer>(cfg, opts.device_id, cfg.n_hypotheses), cfg);
    injected.prepareForBatch(cfg.n_hypotheses);
    const PoseEstimate a = injected.registerFrame(rgb.data(), depth.data(), mask.data(), wh[0], wh[1], K, n_refine);
    const PoseEstimate at = injected.trackFrame(rgb.data(), depth.data(), wh[0], wh[1], K, 2);

    FoundationPose builtin = FoundationPose::createFromCadFile(argv[1], opts, cfg);
    const PoseEstimate b = builtin.registerFrame(rgb.data(), depth.data(), mask.data(), wh[0], wh[1], K, n_refine);
    const PoseEstimate bt = builtin.trackFrame(rgb.data(), depth.data(), wh[0], wh[1], K, 2);

    std::printf("{");
    printPose("injected", a);
    std::printf(", ");
    printPose("injected_track", at);
    std::printf(", ");
    printPose("builtin", b);
    std::printf(", ");
    printPose("builtin_track", bt);
    std::printf(", \"prepares\": %d, \"refines\": %d, \"refine_items\": %d, \"scores\": %d, \"score_items\": %d}\n",
                counts->prepares, counts->refines, counts->refine_items, counts->scores_calls, counts->score_items);
    return 0;
  } catch (const FoundationPoseError& e) {
    std::printf("{\"error\": \"FoundationPoseError: %s\"}\n", e.what());
    return 1;
  } catch (const std::exception& e) {
    std::printf("{\"error\": \"%s\"}\n", e.what());
    return 1;
  }
}
