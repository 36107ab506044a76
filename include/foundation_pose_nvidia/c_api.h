/*
 * FoundationPose B200 runtime -- stable C ABI (drop-in for the reference's
 * include/foundation_pose_nvidia/c_api.h; SOVERSION 1).
 *
 * Every symbol, struct and field below has the same name, order, type and
 * meaning as the reference header so existing C/C++/ctypes callers keep
 * working unchanged; struct layouts are pinned with static_asserts in
 * csrc/fp_c_api.cpp. The implementation behind it is this project's own
 * sm_100a CUDA pipeline (fused preprocess, tile-resident rasterizer, fused
 * crop-warp/pack, tcgen05 RefineNet/ScoreNet) -- no TensorRT.
 *
 * Conventions (unchanged from the reference):
 *  - RGB HWC uint8, depth HW float32 metres, mask HW uint8 (non-zero = object).
 *  - K is 3x3 row-major float32, host memory.
 *  - Frame pointers may be host or CUDA device/managed memory (resolved through
 *    unified virtual addressing); they are borrowed for the call only.
 *  - Results: 4x4 row-major object-to-camera pose + score (track: score = 1).
 *  - Errors: NULL / non-zero return plus a NUL-terminated, truncated message
 *    in the caller's buffer ("" on success). No C++ exception crosses the ABI.
 *  - One handle = one CUDA stream + one workspace; a handle is not thread-safe.
 */
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifdef _WIN32
#ifdef FOUNDATION_POSE_NVIDIA_EXPORTS
#define FP_API __declspec(dllexport)
#else
#define FP_API __declspec(dllimport)
#endif
#else
#define FP_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

/** Opaque estimator handle (reference c_api.h:165). */
typedef struct fp_handle fp_handle_t;

/** Construction options (reference c_api.h:174-188). The model paths name this
 *  runtime's weight packs (see fp_weights.py); the tensor-name fields are kept
 *  for layout compatibility and validated against the pack's I/O names. */
typedef struct fp_create_options {
  const char* cad_path;
  int device_id;
  float mesh_unit_scale;
  const char* refine_model_path;
  const char* score_model_path;
  const char* engine_cache_dir;
  const char* refine_model_name;
  const char* score_model_name;
  const char* rendered_input_name;
  const char* observed_input_name;
  const char* refine_translation_output_name;
  const char* refine_rotation_output_name;
  const char* score_output_name;
} fp_create_options_t;

/** Network precision (reference c_api.h:200-205). FP32 = strict IEEE FP32 SIMT
 *  kernels; TF32/FP16/BF16 = tcgen05 tensor-core kernels. */
typedef enum fp_precision {
  FP_PRECISION_FP32 = 0,
  FP_PRECISION_TF32 = 1,
  FP_PRECISION_FP16 = 2,
  FP_PRECISION_BF16 = 3
} fp_precision_t;

/** Runtime configuration, append-only (reference c_api.h:211-226). */
typedef struct fp_config {
  int n_hypotheses;
  int n_refine_iters;
  int n_track_iters;
  float crop_ratio;
  int input_width;
  int input_height;
  int max_image_width;
  int max_image_height;
  int capture_cuda_graph;
  int model_free_sample_stride;
  int model_free_max_vertices;
  float model_free_depth_edge_threshold;
  int tensorrt_precision; /* name kept for ABI compatibility: the network precision */
  int batch_size;
} fp_config_t;

/** One RGB-D frame (reference c_api.h:238-245). */
typedef struct fp_image_view {
  int width;
  int height;
  const uint8_t* rgb_u8;
  const float* depth_m;
  const uint8_t* mask_u8;
  const float* k_row_major;
} fp_image_view_t;

/** One model-free reference view, host memory only (reference c_api.h:253-261). */
typedef struct fp_reference_image_view {
  int width;
  int height;
  const uint8_t* rgb_u8;
  const float* depth_m;
  const uint8_t* mask_u8;
  const float* k_row_major;
  const float* camera_to_world_row_major;
} fp_reference_image_view_t;

/** Pose + score (reference c_api.h:266-269). */
typedef struct fp_pose_result {
  float pose_row_major[16];
  float score;
} fp_pose_result_t;

/** Fill defaults (reference c_api.h:275). */
FP_API void fp_default_config(fp_config_t* config);

/** Model-based estimator from an OBJ/PLY mesh (reference c_api.h:285-288). */
FP_API fp_handle_t* fp_create(const fp_create_options_t* options,
                              const fp_config_t* config,
                              char* error_buffer,
                              size_t error_buffer_size);

/** Model-free estimator from reference views (reference c_api.h:300-305). */
FP_API fp_handle_t* fp_create_model_free(const fp_reference_image_view_t* references,
                                         size_t reference_count,
                                         const fp_create_options_t* options,
                                         const fp_config_t* config,
                                         char* error_buffer,
                                         size_t error_buffer_size);

/** Pre-build network state for a batch size (reference c_api.h:320-323). */
FP_API int fp_prepare(fp_handle_t* handle,
                      int batch_size,
                      char* error_buffer,
                      size_t error_buffer_size);

/** Release a handle; NULL is a no-op (reference c_api.h:329). */
FP_API void fp_destroy(fp_handle_t* handle);

/** Register: hypothesis search + refinement + scoring (reference c_api.h:347-353). */
FP_API int fp_register_frame(fp_handle_t* handle,
                             const fp_image_view_t* image,
                             int n_refine,
                             int n_hypotheses,
                             fp_pose_result_t* result,
                             char* error_buffer,
                             size_t error_buffer_size);

/** Track from the previous pose (reference c_api.h:369-374). */
FP_API int fp_track_frame(fp_handle_t* handle,
                          const fp_image_view_t* image,
                          int n_refine,
                          fp_pose_result_t* result,
                          char* error_buffer,
                          size_t error_buffer_size);

/** Sharded register, phase 1 (no counterpart in the reference: the
 * multi-GPU extension of fp_register_frame). One handle per GPU, all created
 * from the same mesh and config. Each shard refines hypotheses
 * [shard_begin, shard_begin + shard_count) of the n_hypotheses seeded for
 * `image` and writes, into device memory on its handle's GPU, their ScoreNet
 * features (shard_count x FP_SCORE_FEATURE_DIM floats) and refined
 * object-centred poses (shard_count x 16 floats). Returns when they are
 * complete. Requires the built-in renderer and networks. */
#define FP_SCORE_FEATURE_DIM 512
FP_API int fp_register_shard_begin(fp_handle_t* handle,
                                   const fp_image_view_t* image,
                                   int n_refine,
                                   int n_hypotheses,
                                   int shard_begin,
                                   int shard_count,
                                   float* features,
                                   float* poses,
                                   char* error_buffer,
                                   size_t error_buffer_size);

/** Sharded register, phase 2: the caller gathers every shard's features and
 * poses (e.g. an NCCL all-gather) into device memory on this handle's GPU, in
 * hypothesis order; this runs ScoreNet's cross-hypothesis head and the
 * arg-max over all n_hypotheses and returns what fp_register_frame would. The
 * handle can then track. */
FP_API int fp_register_shard_finish(fp_handle_t* handle,
                                    const float* features,
                                    const float* poses,
                                    int n_hypotheses,
                                    fp_pose_result_t* result,
                                    char* error_buffer,
                                    size_t error_buffer_size);

/** Opaque multi-object group (reference c_api.h:398). */
typedef struct fp_group fp_group_t;

#define FP_OBJECT_OK 0
#define FP_OBJECT_FAILED 1
#define FP_OBJECT_SKIPPED 2

/** reference c_api.h:420-424 */
FP_API fp_group_t* fp_group_create(const fp_create_options_t* objects,
                                   size_t object_count,
                                   const fp_config_t* config,
                                   char* error_buffer,
                                   size_t error_buffer_size);
/** reference c_api.h:427 */
FP_API size_t fp_group_size(const fp_group_t* group);
/** reference c_api.h:439 */
FP_API fp_handle_t* fp_group_handle(fp_group_t* group, size_t index);
/** reference c_api.h:449-452 */
FP_API int fp_group_prepare(fp_group_t* group,
                            int batch_size,
                            char* error_buffer,
                            size_t error_buffer_size);
/** reference c_api.h:474-482 */
FP_API int fp_group_register_frame(fp_group_t* group,
                                   const fp_image_view_t* image,
                                   const uint8_t* const* masks,
                                   int n_refine,
                                   int n_hypotheses,
                                   fp_pose_result_t* results,
                                   int* statuses,
                                   char* error_buffer,
                                   size_t error_buffer_size);
/** reference c_api.h:501-508 */
FP_API int fp_group_track_frame(fp_group_t* group,
                                const fp_image_view_t* image,
                                const int* active,
                                int n_refine,
                                fp_pose_result_t* results,
                                int* statuses,
                                char* error_buffer,
                                size_t error_buffer_size);
/** reference c_api.h:515 */
FP_API void fp_group_destroy(fp_group_t* group);

/** cudaDeviceSynchronize on the calling thread's device (reference c_api.h:525). */
FP_API int fp_synchronize_device(char* error_buffer, size_t error_buffer_size);

/** Static build string (reference c_api.h:531). */
FP_API const char* fp_build_info(void);

#ifdef __cplusplus
}
#endif
