/*
 * fpk: kernel-level C ABI of the FoundationPose B200 runtime.
 *
 * These are the sm_100a kernels behind libfoundation_pose_nvidia.so, exported
 * with plain pointers and sizes (no C++ or torch types) so tests, benchmarks
 * and FFI callers can drive each hot-path stage on their own device buffers.
 * All array pointers are DEVICE pointers unless marked (host). `stream` is a
 * cudaStream_t (NULL = legacy default stream). Every call is asynchronous on
 * `stream`; it returns 0 on success or a non-zero code and records a message
 * readable through fpk_last_error() (thread-local).
 *
 * Each entry point names the reference interface it replaces
 * (paths inside nvidia-isaac/foundation-pose-inference-library).
 */
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "foundation_pose_nvidia/c_api.h" /* FP_API */

#ifdef __cplusplus
extern "C" {
#endif

/* Hot-path fields of the reference Config (include/foundation_pose_nvidia/config.hpp:20-67). */
typedef struct fpk_params {
  float depth_min, depth_max;
  int erosion_radius, bilateral_radius;
  float depth_diff_threshold, erosion_ratio_threshold, bilateral_sigma_d, bilateral_sigma_r;
  float crop_ratio;
  int input_width, input_height;
  float rotation_normalizer_rad, znear, zfar, ambient_weight, diffuse_weight;
} fpk_params_t;

/* Camera intrinsics fx, fy, cx, cy (reference types.hpp:174-192). */
typedef struct fpk_intrinsics {
  float fx, fy, cx, cy;
} fpk_intrinsics_t;

/* Device mesh in the centred object frame (reference cuda_pipeline.hpp:21-35).
 * colors are float RGB in [0,1]; uvs/texture optional (NULL / 0). */
typedef struct fpk_mesh {
  const float* vertices;  /* [n_vertices*3] */
  const float* normals;   /* [n_vertices*3] */
  const float* colors;    /* [n_vertices*3] */
  const float* uvs;       /* [n_vertices*2] or NULL */
  const float* texture;   /* [texture_height*texture_width*3] or NULL */
  const int32_t* faces;   /* [n_faces*3] */
  int n_vertices;
  int n_faces;
  int texture_width;
  int texture_height;
} fpk_mesh_t;

/* Network-input element types for fpk_render_pack. */
#define FPK_DTYPE_F32 0
#define FPK_DTYPE_F16 1
#define FPK_DTYPE_BF16 2
/* fp32 kept exact: values are stored without rounding to TF32. fpk_gemm still
 * multiplies on the tensor cores as TF32 (it is the building block of the
 * exact-FP32 layers, which sum three TF32 products of split operands);
 * fpk_attention runs fp32 FMA arithmetic; fpk_render_pack stores plain fp32. */
#define FPK_DTYPE_F32_EXACT 3

/* Size in int32 of the translation-statistics scratch (bbox, count, 65,536-bin histogram). */
#define FPK_STATS_INTS (8 + 65536)

FP_API const char* fpk_last_error(void);
FP_API void fpk_default_params(fpk_params_t* p);

/* Fused depth erode -> bilateral -> (xyz) -> mask statistics, one pass over the frame.
 * Replaces runDepthPreprocess + runDepthToXyz + the statistics half of
 * runInitialTranslation (reference src/cuda_pipeline.cu:743-796).
 * mask may be NULL (track: no statistics). stats must hold FPK_STATS_INTS
 * int32 and is zeroed by this call when mask != NULL. eroded and xyz are
 * optional outputs (NULL to skip). */
FP_API int fpk_preprocess(const float* depth_raw, const uint8_t* mask, int width, int height,
                          fpk_intrinsics_t k, const fpk_params_t* p, float* depth_filtered,
                          float* eroded, float* xyz, int32_t* stats, void* stream);

/* Median-depth translation + pose seeding. Replaces finalizeTranslationKernel +
 * seedPosesKernel (reference src/cuda_pipeline.cu:239-278, 301-327, 797-812).
 * rotations [n*9] row-major; writes t0 [3] and poses [n*16]; re-zeroes nothing. */
FP_API int fpk_seed_poses(const int32_t* stats, const float* rotations, int n, fpk_intrinsics_t k,
                          const fpk_params_t* p, float* t0, float* poses, void* stream);

/* Square crop boxes (l, t, r, b) per pose. Replaces computeCropBoxesOnDevice
 * (reference src/cuda_pipeline.cu:814-826). */
FP_API int fpk_crop_boxes(const float* poses, int n, fpk_intrinsics_t k, float diameter,
                          const fpk_params_t* p, float* boxes, void* stream);

/* Device workspace (bytes, 256-byte aligned) of one fpk_render /
 * fpk_render_pack call over n hypotheses of a mesh with n_vertices vertices:
 * per (hypothesis, vertex) clip and pixel positions, the z-buffer of 64-bit
 * (depth, triangle) keys per crop pixel and the queue of large triangles.
 * Passing workspace = NULL to those calls allocates it stream-ordered per call. */
FP_API size_t fpk_render_workspace_bytes(int n, int n_vertices, const fpk_params_t* p);

/* Rasterize + shade every hypothesis into its crop: NHWC float3 RGB and camera
 * XYZ, rows top-down. Replaces IRenderer::render / BuiltinRasterRenderer::render
 * (reference src/builtin_raster_renderer.cu:218-281, raster_kernels.cuh:336-495).
 * boxes are read (compute them with fpk_crop_boxes). tri_ids (optional,
 * [n*H*W] int32, rows bottom-up like the reference rast buffer) receives
 * triangle_index+1, 0 = background. Four launches: vertex transform,
 * per-triangle raster into an L2-resident z-buffer, warp-per-triangle raster
 * of large triangles, pixel-parallel resolve + shading. */
FP_API int fpk_render(const fpk_mesh_t* mesh, const float* poses, const float* boxes, int n,
                      fpk_intrinsics_t k, const fpk_params_t* p, float* out_rgb, float* out_xyz,
                      int32_t* tri_ids, void* workspace, size_t workspace_bytes, void* stream);

/* Crop-warp + normalisation into the two NCHW [n,6,H,W] fp32 network inputs.
 * Replaces prepareNetworkInputsOnDevice (reference src/cuda_pipeline.cu:434-511, 828-845).
 * Observed XYZ is back-projected from depth_filtered on the fly. */
FP_API int fpk_pack(const uint8_t* rgb, const float* depth_filtered, int width, int height,
                    fpk_intrinsics_t k, const fpk_params_t* p, const float* rend_rgb,
                    const float* rend_xyz, const float* poses, const float* boxes, int n,
                    float diameter, float invalid_depth_threshold, float* net_rendered,
                    float* net_observed, void* stream);

/* Crop boxes + rasterize + shade + crop-warp + pack (vertex transform,
 * per-triangle raster, pixel-parallel resolve + shading + packing), writing both
 * network inputs straight into the stem's space-to-depth KP8 layout: crop pixel
 * (y, x) of image i (rendered i = 0..n-1, observed n+i) goes to plane
 * ((y+3)%2)*2 + (x+3)%2, row i*gh*gw + ((y+3)/2)*gw + (x+3)/2 with
 * gh = (H+7)/2, gw = (W+7)/2 (83 x 83 for 160 x 160 crops): 16 bytes = 6 values
 * + 2 zeros of `dtype` (fp32 values rounded to nearest TF32, the precision the
 * tensor cores read them at; two records per pixel for fp32). net_input points at row 0 of plane 0; planes are
 * plane_stride bytes apart. Rows never written (the zero border of the grid)
 * must be zero before first use. Replaces the computeCropBoxes ->
 * IRenderer::render -> prepareNetworkInputs sequence (reference
 * src/foundation_pose.cpp:429-443). boxes (optional) receives the crop boxes. */
FP_API int fpk_render_pack(const fpk_mesh_t* mesh, const float* poses, int n,
                           const uint8_t* rgb, const float* depth_filtered, int width, int height,
                           fpk_intrinsics_t k, const fpk_params_t* p, float diameter,
                           float invalid_depth_threshold, int dtype, void* net_input,
                           long long plane_stride, float* boxes, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Host-only mesh ingest: load an OBJ/PLY, scale by mesh_unit_scale, compute
 * normals when missing, centre on the bounding-box centre and measure the
 * diameter. Replaces loadMesh + preprocessMesh (reference src/mesh.cpp:577-680)
 * as used by FoundationPose::createFromCadFile (src/foundation_pose.cpp:281-294).
 * Call once with NULL arrays to get the counts, then again with arrays of
 * n_vertices*3 floats (vertices, normals), n_vertices*3 bytes (colours) and
 * n_faces*3 int32 (faces). center3 [3] and diameter receive the centring. */
FP_API int fpk_load_mesh(const char* path, float mesh_unit_scale, int* n_vertices, int* n_faces,
                         float* vertices, float* normals, uint8_t* colors, int32_t* faces,
                         float* center3, float* diameter);

/* Model-free object mesh from reference RGB-D views (host buffers), built on
 * the current GPU. Replaces the reconstruction behind fp_create_model_free
 * (reference src/foundation_pose.cpp:91-182): masked, valid depth samples on a
 * stride lattice back-projected into the world frame, grid triangles with
 * depth-continuous corners, area-weighted vertex normals; the mesh before
 * centring. config supplies the model-free fields and the depth range (NULL =
 * defaults). Call once with NULL arrays for the counts, then with arrays of
 * n_vertices*3 floats (vertices, normals), n_vertices*3 bytes (colours) and
 * n_faces*3 int32 (faces). */
FP_API int fpk_model_free_mesh(const fp_reference_image_view_t* views, size_t count, const fp_config_t* config,
                               int* n_vertices, int* n_faces, float* vertices, uint8_t* colors, float* normals,
                               int32_t* faces);

/* R <- exp(tanh(dr)*norm)^T R; t += dt*diameter/2. Replaces applyPoseDeltasOnDevice
 * (reference src/cuda_pipeline.cu:513-547, 847-858). In place. */
FP_API int fpk_apply_deltas(float* poses, const float* delta_t, const float* delta_r, int n,
                            float diameter, const fpk_params_t* p, void* stream);

/* Arg-max of scores (first maximum wins) + un-centre by the mesh centre (host
 * center3). result = {pose[16], score, index-as-int32}. Replaces
 * selectBestPoseOnDevice (reference src/cuda_pipeline.cu:549-582, 860-868). */
FP_API int fpk_select_best(const float* poses, const float* scores, int n, const float* center3,
                           float* result, void* stream);

/* ---------------------------------------------------------------------------
 * Tensor-core GEMM / implicit convolution (tcgen05 + TMEM, sm_100a).
 *
 * Activations use the channel-group planar layout: plane p holds one 16-byte
 * record per row, channels 8p..8p+7 for fp16/bf16 ("KP8") or 4p..4p+3 for
 * fp32 ("KP4"), so row r of plane p is at base + p*plane_stride + r*16 bytes.
 * Every plane carries zeroed guard rows before row 0 and after the last row,
 * so shifted convolution windows may start at negative rows. fp32 operands run
 * on the tensor cores as TF32 (tcgen05 kind::tf32), fp32 accumulation.
 *
 * out[r, n] = epilogue( sum_t sum_c A[r + tap_off[t], c] * W[n, t, c] + bias[n] )
 * over rows r of a padded spatial grid (img_rows = grid rows per image,
 * grid_w = grid width; rows whose (gy, gx) falls outside valid_h x valid_w are
 * computed but not stored). W is [cout][K'] with K' = (cin/cw)*taps*cw in
 * chunk-major order: k' = chunk*(taps*cw) + tap*cw + c, cw = min(cin, 64) for
 * 16-bit types and min(cin, 32) for fp32 (one chunk = 128 bytes of a row).
 * dst_mode selects where row r / channel n lands:
 *   SAME   (r, n)
 *   S2D    space-to-depth for a following stride-2 conv: cell ((gy+1)/2, (gx+1)/2)
 *          of a dst grid (dst_img_rows, dst_grid_w), channel ((gy+1)%2*2+(gx+1)%2)*cout + n
 *   CONCAT image i -> image i % img_mod, channel (i / img_mod)*ch_step + n
 *   TOKENS dense rows img*valid_h*valid_w + gy*valid_w + gx, adding pos[(gy*valid_w+gx)*cout + n]
 * Replaces the TensorRT engines' convolution / matmul layers behind
 * IInferenceRunner::enqueueRefine / enqueueScore (reference
 * src/tensorrt_runner.cu:367-407). */
#define FPK_DST_SAME 0
#define FPK_DST_S2D 1
#define FPK_DST_CONCAT 2
#define FPK_DST_TOKENS 3
#define FPK_GEMM_MAX_TAPS 16

typedef struct fpk_gemm_desc {
  const void* a;
  long long a_plane_stride;
  int rows;
  int cin;
  int taps;
  int tap_off[FPK_GEMM_MAX_TAPS];
  const void* w;
  int cout;
  const float* bias;
  const void* residual; /* same layout/grid as A (cout channels), or NULL */
  long long res_plane_stride;
  int relu;
  void* dst;
  long long dst_plane_stride;
  int dst_mode;
  int img_rows, grid_w, valid_h, valid_w;
  int dst_img_rows, dst_grid_w, img_mod, ch_step;
  const float* pos;
  int dtype;       /* FPK_DTYPE_F16, FPK_DTYPE_BF16 or FPK_DTYPE_F32 (TF32 math) */
  int* error_flag; /* device int32; set non-zero if a pipeline wait times out */
  /* Optional split-K scratch (device, or NULL). When given, a layer whose
   * output tiles fill less than half of the GPU splits its K range over up to
   * 8 CTAs per tile, which write fp32 partial sums here; a second launch adds
   * the partials of each output in split order and applies the epilogue, so
   * results are deterministic for a given layer and row count (they differ
   * from the unsplit sum in the last bits). Nothing in it needs initialising. */
  void* splitk_ws;
  long long splitk_ws_bytes;
} fpk_gemm_desc_t;

FP_API int fpk_gemm(const fpk_gemm_desc_t* desc, void* stream);

/* Layers with 256-channel output tiles (cout a multiple of 256) run as CTA
 * pairs (clusters of two CTAs issuing tcgen05 cta_group::2 MMAs on 256-row
 * tiles) when their rows fill every SM; enable = 0 keeps every layer on
 * single-CTA tiles. Process-wide;
 * returns the previous setting. No reference counterpart (a tuning switch). */
FP_API int fpk_gemm_set_cta_pairs(int enable);

/* Tuning switch (no reference counterpart): with enable != 0 (the default),
 * dense 16-bit layers on CTA pairs (SAME destination, every row valid, 256-
 * channel tiles: the transformer linears) stage each 32-column chunk of the
 * output in shared memory and write it with one bulk tensor store per warp;
 * enable = 0 keeps per-thread 16-byte stores. Results are bit-identical either
 * way. Process-wide; returns the previous setting. */
FP_API int fpk_gemm_set_tma_store(int enable);

/* Failure-injection test switch (no reference counterpart). With enable != 0
 * every following fpk_gemm runs on single-CTA tiles whose producer issues no
 * loads, so the MMA warp's bounded wait for its first operand tile runs out
 * (~2 s): the kernel records a non-zero code in desc->error_flag, every role
 * exits without leaving a copy or an MMA in flight, and the context stays
 * usable. The output is not written. Process-wide; returns the previous
 * setting. Used by the tests of the bounded-wait error path only. */
FP_API int fpk_gemm_test_withhold_loads(int enable);

/* Fused multi-head self-attention on tcgen05/TMEM (head dim 128):
 * out = softmax(Q K^T / sqrt(128)) V for every (layer, head, sequence), over
 * planar activations of `dtype` (fp16/bf16 KP8, or fp32 KP4 run as TF32).
 * Sequence s occupies rows [s*seq_len, (s+1)*seq_len). For layer z and head
 * h, Q / K / V are the 128 channels starting at channel
 * z*qkv_layer_channels + {q,k,v}_channel + 128h of `qkv`, and the output goes
 * to channels z*out_layer_channels + 128h of `out`. Replaces the attention
 * inside the TensorRT engines behind IInferenceRunner::enqueueRefine /
 * enqueueScore (reference src/tensorrt_runner.cu:367-407). */
FP_API int fpk_attention(const void* qkv, long long qkv_plane_stride, int qkv_layer_channels,
                         int q_channel, int k_channel, int v_channel, void* out,
                         long long out_plane_stride, int out_layer_channels, int layers, int heads,
                         int seq_len, int n_seq, int dtype, int* error_flag, void* stream);

/* ---------------------------------------------------------------------------
 * RefineNet / ScoreNet as a unit: the built-in inference backend behind
 * IInferenceRunner (reference include/foundation_pose_nvidia/inference_runner.hpp:12-30,
 * src/tensorrt_runner.cu:498-532). Weight packs (.fpw) replace the ONNX files;
 * precision is any FP_PRECISION_* (FP32 and TF32 both run as TF32 on the tensor cores).
 * Inputs are NCHW [n,6,160,160] fp32 device tensors (rendered = inputA,
 * observed = inputB); outputs are device fp32 trans/rot [n,3] and score [n].
 * A handle owns its device memory for max_batch hypotheses on the current device. */
typedef struct fpk_net fpk_net_t;
FP_API fpk_net_t* fpk_net_create(const char* refine_pack, const char* score_pack, int precision,
                                 int max_batch);
FP_API void fpk_net_destroy(fpk_net_t* net);
FP_API int fpk_net_refine(fpk_net_t* net, const float* rendered, const float* observed, int n,
                          float* trans, float* rot, void* stream);
FP_API int fpk_net_score(fpk_net_t* net, const float* rendered, const float* observed, int n,
                         float* scores, void* stream);
/* Device error flag of the pipelined kernels: 0 = ok (non-zero after a wait timed out). */
FP_API int fpk_net_error(fpk_net_t* net, int* host_flag);

/* Allocation-free initial translation. No counterpart in the reference: it is
 * the same chain as fpk_preprocess + fpk_seed_poses (the reference's
 * runDepthPreprocess + runInitialTranslation) for callers that may not allocate
 * device memory -- real-time loops and safety-reviewed deployments that freeze
 * their memory at start-up, and plugin hosts that own every buffer. The caller
 * passes the raw depth and mask (device) and receives t0 [3] (device); the
 * filtered depth and the depth histogram live in fixed device arrays built
 * into the library (about 3.8 MiB on every GPU that loads it, until exit).
 * Frames larger than FPK_NOALLOC_MAX_PIXELS (1280x720) are rejected with an
 * error. The first call on a device looks up the arrays' device addresses;
 * under CUDA's default lazy module loading that is also when the driver sets
 * the arrays' memory aside on that device, so make one warm-up call per device
 * at start-up, before the memory footprint is frozen and before any stream
 * capture (CUDA_MODULE_LOADING=EAGER reserves them at library load instead).
 * All calls share the arrays: calls that overlap on the GPU race and must be
 * serialised by the caller. */
#define FPK_NOALLOC_MAX_PIXELS (1280 * 720)
FP_API int fpk_initial_translation_noalloc(const float* depth_raw, const uint8_t* mask, int width,
                                           int height, fpk_intrinsics_t k, const fpk_params_t* p,
                                           float* t0, void* stream);

/* ---------------------------------------------------------------------------
 * Benchmark instrumentation (no counterpart in the reference, which has no
 * tracing). Stages: 0 tensor-core GEMM, 1 fused render+pack / render,
 * 2 attention, 3 other network kernels, 4 frame preprocess.
 * fpk_profile_enable(1) makes every stage record a CUDA event pair on its own
 * stream plus its algorithmic work (GEMM: FLOPs of the un-padded convolution or
 * matmul; render: bytes of mesh + frame read and network input written).
 * Launch counts are always kept. fpk_profile_read fills arrays of 5 per stage
 * (any may be NULL) and returns 5. */
FP_API void fpk_profile_enable(int enable);
FP_API void fpk_profile_reset(void);
FP_API int fpk_profile_read(double* ms, double* work, long long* timed, long long* launches);

#ifdef __cplusplus
}
#endif
