// Test-oracle shim (not product code): exposes the reference's own CPU
// functions through a flat C ABI so tests/golden/make_golden.py can drive them
// with ctypes. Linked against the unmodified reference sources
// src/pipeline_utils.cpp and src/mesh.cpp (built by oracle/Makefile into
// oracle/_ref/libfpref_cpu.so). Only tests and the fixture generator load it.
#include <cstdint>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

#include "foundation_pose_nvidia/config.hpp"
#include "foundation_pose_nvidia/mesh.hpp"
#include "foundation_pose_nvidia/types.hpp"
#include "pipeline_utils.hpp"

namespace fpn = foundation_pose_nvidia;

namespace {
fpn::Config defaults() { return fpn::Config{}; }
fpn::CameraIntrinsics intr(const float* k4) { return fpn::CameraIntrinsics{k4[0], k4[1], k4[2], k4[3]}; }
}  // namespace

extern "C" {

// reference: src/pipeline_utils.cpp:352 makeRotationGrid -> rotations (row-major 3x3)
int refcpu_rotation_grid(float* out, int max_count) {
  const auto rots = fpn::detail::makeRotationGrid(defaults());
  const int n = static_cast<int>(rots.size());
  for (int i = 0; i < n && i < max_count; ++i) {
    std::memcpy(out + 9 * i, rots[i].values.data(), 9 * sizeof(float));
  }
  return n;
}

// reference: src/pipeline_utils.cpp:250 preprocessDepth (erode + bilateral, CPU semantics)
int refcpu_preprocess_depth(const float* depth, int w, int h, float* out) {
  try {
    fpn::DepthImage img;
    img.width = w;
    img.height = h;
    img.meters.assign(depth, depth + static_cast<std::size_t>(w) * h);
    const auto r = fpn::detail::preprocessDepth(img, defaults());
    std::memcpy(out, r.data(), r.size() * sizeof(float));
    return 0;
  } catch (const std::exception&) {
    return 1;
  }
}

// reference: src/pipeline_utils.cpp:265 depthToXyz
void refcpu_depth_to_xyz(const float* depth, int w, int h, const float* k4, float* xyz) {
  std::vector<float> d(depth, depth + static_cast<std::size_t>(w) * h);
  const auto r = fpn::detail::depthToXyz(d, w, h, intr(k4), defaults());
  for (std::size_t i = 0; i < r.size(); ++i) {
    xyz[3 * i + 0] = r[i].x;
    xyz[3 * i + 1] = r[i].y;
    xyz[3 * i + 2] = r[i].z;
  }
}

// reference: src/pipeline_utils.cpp:288 guessTranslation (exact median, CPU semantics)
void refcpu_guess_translation(const float* depth, const std::uint8_t* mask, int w, int h,
                              const float* k4, float* t3) {
  std::vector<float> d(depth, depth + static_cast<std::size_t>(w) * h);
  fpn::MaskImage m;
  m.width = w;
  m.height = h;
  m.values.assign(mask, mask + static_cast<std::size_t>(w) * h);
  const auto t = fpn::detail::guessTranslation(d, m, intr(k4), defaults());
  t3[0] = t.x;
  t3[1] = t.y;
  t3[2] = t.z;
}

// reference: src/pipeline_utils.cpp:356 computeCropBoxes
void refcpu_crop_boxes(const float* poses, int n, const float* k4, float diameter, float* boxes) {
  std::vector<fpn::Mat4f> p(static_cast<std::size_t>(n));
  for (int i = 0; i < n; ++i) {
    std::memcpy(p[i].values.data(), poses + 16 * i, 16 * sizeof(float));
  }
  const auto b = fpn::detail::computeCropBoxes(p, intr(k4), diameter, defaults());
  for (int i = 0; i < n; ++i) {
    boxes[4 * i + 0] = b[i].left;
    boxes[4 * i + 1] = b[i].top;
    boxes[4 * i + 2] = b[i].right;
    boxes[4 * i + 3] = b[i].bottom;
  }
}

// reference: src/pipeline_utils.cpp:398 applyDelta
void refcpu_apply_delta(const float* pose, const float* dt, const float* dr, float diameter,
                        float* out) {
  fpn::Mat4f p;
  std::memcpy(p.values.data(), pose, 16 * sizeof(float));
  const auto r = fpn::detail::applyDelta(p, fpn::Vec3f{dt[0], dt[1], dt[2]},
                                         fpn::Vec3f{dr[0], dr[1], dr[2]}, diameter, defaults());
  std::memcpy(out, r.values.data(), 16 * sizeof(float));
}

// reference: src/mesh.cpp:577 loadMesh + :612 preprocessMesh. Returns vertex and
// face counts; a second call with non-NULL buffers copies the centred mesh out.
int refcpu_load_mesh(const char* path, int* n_verts, int* n_faces, float* centered_verts,
                     float* normals, std::uint8_t* colors, std::uint32_t* faces, float* center3,
                     float* diameter, char* err, int err_len) {
  try {
    const fpn::Mesh mesh = fpn::loadMesh(path);
    const fpn::PreprocessedMesh pm = fpn::preprocessMesh(mesh, defaults());
    *n_verts = static_cast<int>(pm.centered_mesh.vertices.size());
    *n_faces = static_cast<int>(pm.centered_mesh.faces.size());
    if (centered_verts != nullptr) {
      const auto& m = pm.centered_mesh;
      for (std::size_t i = 0; i < m.vertices.size(); ++i) {
        centered_verts[3 * i + 0] = m.vertices[i].x;
        centered_verts[3 * i + 1] = m.vertices[i].y;
        centered_verts[3 * i + 2] = m.vertices[i].z;
        normals[3 * i + 0] = m.normals[i].x;
        normals[3 * i + 1] = m.normals[i].y;
        normals[3 * i + 2] = m.normals[i].z;
        const fpn::Vec3u8 c = i < m.vertex_colors.size() ? m.vertex_colors[i] : fpn::Vec3u8{};
        colors[3 * i + 0] = c.r;
        colors[3 * i + 1] = c.g;
        colors[3 * i + 2] = c.b;
      }
      for (std::size_t i = 0; i < m.faces.size(); ++i) {
        faces[3 * i + 0] = m.faces[i][0];
        faces[3 * i + 1] = m.faces[i][1];
        faces[3 * i + 2] = m.faces[i][2];
      }
    }
    center3[0] = pm.center.x;
    center3[1] = pm.center.y;
    center3[2] = pm.center.z;
    *diameter = pm.diameter;
    return 0;
  } catch (const std::exception& e) {
    if (err != nullptr && err_len > 0) {
      std::strncpy(err, e.what(), static_cast<std::size_t>(err_len - 1));
      err[err_len - 1] = '\0';
    }
    return 1;
  }
}

}  // extern "C"
