// Plain data types of the C++ seam (reference include/foundation_pose_nvidia/types.hpp:11-283).
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

#pragma GCC visibility push(default)
namespace foundation_pose_nvidia {

struct Vec2f {
  float x = 0.0f;
  float y = 0.0f;
};

struct Vec3f {
  float x = 0.0f;
  float y = 0.0f;
  float z = 0.0f;
  friend Vec3f operator+(Vec3f a, Vec3f b) { return {a.x + b.x, a.y + b.y, a.z + b.z}; }
  friend Vec3f operator-(Vec3f a, Vec3f b) { return {a.x - b.x, a.y - b.y, a.z - b.z}; }
  friend Vec3f operator*(Vec3f a, float s) { return {a.x * s, a.y * s, a.z * s}; }
  friend Vec3f operator/(Vec3f a, float s) { return {a.x / s, a.y / s, a.z / s}; }
};

struct Vec3u8 {
  std::uint8_t r = 128;
  std::uint8_t g = 128;
  std::uint8_t b = 128;
};

struct Mat3f {
  std::array<float, 9> values{};
  static Mat3f identity() {
    Mat3f m;
    m.values[0] = m.values[4] = m.values[8] = 1.0f;
    return m;
  }
  float& operator()(std::size_t r, std::size_t c) { return values[r * 3 + c]; }
  float operator()(std::size_t r, std::size_t c) const { return values[r * 3 + c]; }
};

struct Mat4f {
  std::array<float, 16> values{};
  static Mat4f identity() {
    Mat4f m;
    m.values[0] = m.values[5] = m.values[10] = m.values[15] = 1.0f;
    return m;
  }
  float& operator()(std::size_t r, std::size_t c) { return values[r * 4 + c]; }
  float operator()(std::size_t r, std::size_t c) const { return values[r * 4 + c]; }
};

struct CameraIntrinsics {
  float fx = 0.0f;
  float fy = 0.0f;
  float cx = 0.0f;
  float cy = 0.0f;
  static CameraIntrinsics fromRowMajor(const float* k) { return {k[0], k[4], k[2], k[5]}; }
};

struct ModelFreeReferenceView {
  int width = 0;
  int height = 0;
  const std::uint8_t* rgb_u8 = nullptr;
  const float* depth_m = nullptr;
  const std::uint8_t* mask_u8 = nullptr;
  CameraIntrinsics intrinsics{};
  Mat4f camera_to_world = Mat4f::identity();
};

struct Mesh {
  std::vector<Vec3f> vertices;
  std::vector<std::array<std::uint32_t, 3>> faces;
  std::vector<Vec3f> normals;
  std::vector<Vec2f> uvs;
  std::vector<Vec3u8> vertex_colors;
  int texture_width = 0;
  int texture_height = 0;
  std::vector<Vec3u8> texture_rgb;
  std::string source_path;
  bool hasTexture() const { return texture_width > 0 && texture_height > 0 && !texture_rgb.empty(); }
};

struct PreprocessedMesh {
  Mesh centered_mesh;
  float diameter = 0.0f;
  Vec3f center{};
  std::vector<Vec3f> downsampled_points;
};

struct PoseEstimate {
  Mat4f pose = Mat4f::identity();  // object-to-camera, original mesh frame
  float score = 0.0f;
};

}  // namespace foundation_pose_nvidia
#pragma GCC visibility pop
