// TEST INFRASTRUCTURE ONLY (not product code).
//
// Compiles the reference's estimator source (src/foundation_pose.cpp,
// unmodified) into this translation unit so the test oracle can also call its
// model-free reconstruction, which the reference keeps in an anonymous
// namespace (reconstructReferenceMesh, foundation_pose.cpp:91-182). Linked into
// oracle/_ref/libfpref_full.so in place of a separate foundation_pose.cpp
// object; the library's fp_* entry points are unaffected. The reconstruction
// runs on the host only, so tests can call it without a GPU.
#include "foundation_pose.cpp"

extern "C" {

// Views: count reference views of width x height (host arrays per view), K
// row-major 3x3 per view, camera_to_world row-major 4x4 per view. Returns 0 and
// the counts; fills at most cap_v vertices / cap_f faces of the arrays given.
int refmf_reconstruct(int count, int width, int height, const float* const* depth, const std::uint8_t* const* rgb,
                      const std::uint8_t* const* mask, const float* k9, const float* c2w16, int sample_stride,
                      int max_vertices, float edge_threshold, float depth_min, float depth_max, int* n_vertices,
                      int* n_faces, float* vertices, std::uint8_t* colors, float* normals, std::int32_t* faces,
                      int cap_v, int cap_f, char* err, int err_size) {
  using namespace foundation_pose_nvidia;
  try {
    std::vector<ModelFreeReferenceView> views(static_cast<std::size_t>(count));
    for (int i = 0; i < count; ++i) {
      ModelFreeReferenceView& v = views[static_cast<std::size_t>(i)];
      v.width = width;
      v.height = height;
      v.rgb_u8 = rgb[i];
      v.depth_m = depth[i];
      v.mask_u8 = mask[i];
      v.intrinsics = CameraIntrinsics::fromRowMajor(k9 + 9 * i);
      for (int k = 0; k < 16; ++k) v.camera_to_world.values[static_cast<std::size_t>(k)] = c2w16[16 * i + k];
    }
    Config cfg;
    cfg.model_free_sample_stride = sample_stride;
    cfg.model_free_max_vertices = max_vertices;
    cfg.model_free_depth_edge_threshold = edge_threshold;
    cfg.depth_min = depth_min;
    cfg.depth_max = depth_max;
    const Mesh m = reconstructReferenceMesh(views, cfg);
    *n_vertices = static_cast<int>(m.vertices.size());
    *n_faces = static_cast<int>(m.faces.size());
    for (int i = 0; i < *n_vertices && i < cap_v; ++i) {
      vertices[3 * i] = m.vertices[i].x;
      vertices[3 * i + 1] = m.vertices[i].y;
      vertices[3 * i + 2] = m.vertices[i].z;
      colors[3 * i] = m.vertex_colors[i].r;
      colors[3 * i + 1] = m.vertex_colors[i].g;
      colors[3 * i + 2] = m.vertex_colors[i].b;
      normals[3 * i] = m.normals[i].x;
      normals[3 * i + 1] = m.normals[i].y;
      normals[3 * i + 2] = m.normals[i].z;
    }
    for (int i = 0; i < *n_faces && i < cap_f; ++i)
      for (int k = 0; k < 3; ++k) faces[3 * i + k] = static_cast<std::int32_t>(m.faces[i][k]);
    return 0;
  } catch (const std::exception& e) {
    std::snprintf(err, static_cast<std::size_t>(err_size), "%s", e.what());
    return 1;
  }
}

}  // extern "C"
