/*
 * TEST INFRASTRUCTURE ONLY. CPU restatement (plain C) of the reference
 * FoundationPose render-and-compare hot path, used as the parity checker for
 * the CUDA product kernels. Only tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg may load it; the product library never links or calls it.
 *
 * Parity pins: the reference's own CPU functions (src/pipeline_utils.cpp,
 * src/mesh.cpp) compiled into oracle/_ref/libfpref_cpu.so, and the reference's
 * own CUDA kernels (src/cuda_pipeline.cu, src/builtin_raster_renderer.cu)
 * compiled into oracle/_ref/libfpref_gpu.so and run on the GPU box; golden
 * vectors produced from both live under tests/golden/.
 *
 * Functions follow the reference's GPU semantics (the shipped path). Where the
 * reference's CPU twin differs (erosion border handling, exact vs histogram
 * median), a *_cpu variant restates the CPU behaviour so it can be pinned too.
 */
#ifndef FP_ORACLE_H
#define FP_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Fields of the reference Config (include/foundation_pose_nvidia/config.hpp:20-67)
 * read on the hot path. */
typedef struct fpo_config {
  float depth_min, depth_max;
  int erosion_radius, bilateral_radius;
  float depth_diff_threshold, erosion_ratio_threshold, bilateral_sigma_d, bilateral_sigma_r;
  float crop_ratio;
  int input_width, input_height;
  float rotation_normalizer_rad, znear, zfar, ambient_weight, diffuse_weight;
} fpo_config;

void fpo_default_config(fpo_config* c);

/* K1 erode / K2 bilateral / K3 depth->xyz (GPU semantics). */
void fpo_erode(const float* in, float* out, int w, int h, const fpo_config* c);
void fpo_bilateral(const float* in, float* out, int w, int h, const fpo_config* c);
void fpo_depth_to_xyz(const float* depth, float* xyz, int w, int h, const float* k4,
                      const fpo_config* c);
/* CPU twin: pipeline_utils.cpp:250 preprocessDepth (clamp, border-as-bad erosion, bilateral). */
void fpo_preprocess_cpu(const float* depth, float* out, int w, int h, const fpo_config* c);

/* K4-K6 initial translation (GPU semantics: histogram median). */
void fpo_initial_translation(const float* depth, const uint8_t* mask, int w, int h,
                             const float* k4, const fpo_config* c, float* t3);
/* CPU twin: pipeline_utils.cpp:288 guessTranslation (exact median). */
void fpo_guess_translation_cpu(const float* depth, const uint8_t* mask, int w, int h,
                               const float* k4, const fpo_config* c, float* t3);

/* a5: rotation grid (pipeline_utils.cpp:215-246); returns count, writes up to max. */
int fpo_rotation_grid(float* out9, int max_count);
/* K7 seed poses. */
void fpo_seed_poses(const float* rot9, const float* t3, int n, float* poses16);
/* K8 crop boxes. */
void fpo_crop_boxes(const float* poses16, int n, const float* k4, float diameter,
                    const fpo_config* c, float* boxes4);

/* K9-K13 render: rgb/xyz NHWC [B,H,W,3] top-down; rast [B,H,W,4] bottom-up
 * (b0, b1, zw, tri+1). colors are float [0,1] per vertex. rast may be NULL. */
void fpo_render(const float* verts, const float* normals, const float* colors, int n_verts,
                const int32_t* faces, int n_faces, const float* poses16, const float* boxes4,
                int batch, const float* k4, const fpo_config* c, float* out_rgb, float* out_xyz,
                float* out_rast);

/* K14 pack: network inputs NCHW [B,6,H,W] for rendered and observed. */
void fpo_pack(const uint8_t* rgb, const float* xyz_map, int img_w, int img_h,
              const float* rend_rgb, const float* rend_xyz, const float* poses16,
              const float* boxes4, int batch, int crop_w, int crop_h, float diameter,
              float invalid_threshold, float* net_rendered, float* net_observed);

/* K15 pose deltas (GPU semantics) in place. */
void fpo_apply_deltas(float* poses16, const float* dt, const float* dr, int batch, float diameter,
                      const fpo_config* c);
/* K16 arg-max + un-centre. Returns the index. */
int fpo_select_best(const float* poses16, const float* scores, int batch, const float* center3,
                    float* out_pose16, float* out_score);

/* a14 mesh: computeVertexNormals (mesh.cpp:589-610), preprocessMesh centre/diameter
 * (mesh.cpp:612-660). centered may alias verts. */
void fpo_vertex_normals(const float* verts, int n_verts, const int32_t* faces, int n_faces,
                        float* normals);
void fpo_mesh_center_diameter(const float* verts, int n_verts, int sample_points,
                              float* center3, float* diameter, float* centered);

#ifdef __cplusplus
}
#endif
#endif
