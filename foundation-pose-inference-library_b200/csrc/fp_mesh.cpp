// Mesh ingest and host-side geometry: OBJ/PLY loading, vertex normals, mesh
// centring and diameter (reference src/mesh.cpp:139-680), the pose-hypothesis
// rotation grid (reference src/pipeline_utils.cpp:141-246) and model-free mesh
// reconstruction from reference views (reference src/foundation_pose.cpp:91-182).
// All of this runs once per estimator at construction time.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <limits>
#include <map>
#include <numbers>
#include <span>
#include <sstream>
#include <string>
#include <utility>
#include <vector>

#include "foundation_pose_nvidia/config.hpp"
#include "foundation_pose_nvidia/device_buffer.hpp"
#include "foundation_pose_nvidia/foundation_pose.hpp"
#include "foundation_pose_nvidia/types.hpp"
#include "fp_host.hpp"
#include "fpk.h"

namespace foundation_pose_nvidia {

namespace {

float dot(Vec3f a, Vec3f b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
Vec3f cross(Vec3f a, Vec3f b) {
  return {a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x};
}
float norm(Vec3f a) { return std::sqrt(std::max(dot(a, a), 0.0f)); }
Vec3f normalizeOrZero(Vec3f a) {
  const float n = norm(a);
  return n < 1e-12f ? Vec3f{} : a / n;
}

std::string lowerExt(const std::filesystem::path& p) {
  std::string e = p.extension().string();
  for (char& c : e) c = static_cast<char>(std::tolower(static_cast<unsigned char>(c)));
  return e;
}

void stripCr(std::string& s) {
  if (!s.empty() && s.back() == '\r') s.pop_back();
}

std::uint32_t objIndex(const std::string& token, std::size_t count) {
  const int idx = std::stoi(token.substr(0, token.find('/')));
  if (idx > 0) return static_cast<std::uint32_t>(idx - 1);
  if (idx < 0) return static_cast<std::uint32_t>(static_cast<int>(count) + idx);
  throw FoundationPoseError("OBJ indices are 1-based; got index 0");
}

// OBJ: "v x y z [r g b]" (colours in [0,1] are scaled to [0,255], then
// clamped and truncated to 8 bits; default grey 128), "vt u v", polygon faces
// fanned into triangles. Normals are recomputed from the faces.
Mesh loadObj(const std::filesystem::path& path) {
  std::ifstream in(path);
  if (!in) throw FoundationPoseError("Failed to open OBJ mesh: " + path.string());
  Mesh mesh;
  mesh.source_path = path.string();
  std::string line;
  while (std::getline(in, line)) {
    if (line.empty() || line[0] == '#') continue;
    std::istringstream iss(line);
    std::string tag;
    iss >> tag;
    if (tag == "v") {
      Vec3f p{};
      iss >> p.x >> p.y >> p.z;
      mesh.vertices.push_back(p);
      float r = 128.0f, g = 128.0f, b = 128.0f;
      if ((iss >> r >> g >> b) && r <= 1.0f && g <= 1.0f && b <= 1.0f) {
        r *= 255.0f;
        g *= 255.0f;
        b *= 255.0f;
      }
      mesh.vertex_colors.push_back({static_cast<std::uint8_t>(std::clamp(r, 0.0f, 255.0f)),
                                    static_cast<std::uint8_t>(std::clamp(g, 0.0f, 255.0f)),
                                    static_cast<std::uint8_t>(std::clamp(b, 0.0f, 255.0f))});
    } else if (tag == "vt") {
      Vec2f uv{};
      iss >> uv.x >> uv.y;
      mesh.uvs.push_back(uv);
    } else if (tag == "f") {
      std::vector<std::uint32_t> idx;
      std::string tok;
      while (iss >> tok) idx.push_back(objIndex(tok, mesh.vertices.size()));
      for (std::size_t i = 1; i + 1 < idx.size(); ++i) mesh.faces.push_back({idx[0], idx[i], idx[i + 1]});
    }
  }
  if (mesh.vertices.empty() || mesh.faces.empty()) {
    throw FoundationPoseError("OBJ mesh has no usable vertices/faces: " + path.string());
  }
  computeVertexNormals(mesh);
  return mesh;
}

// ---- PLY (ascii / binary_little_endian) ----

struct PlyProp {
  bool list = false;
  std::string type, count_type, item_type, name;
};
struct PlyElem {
  std::string name;
  std::size_t count = 0;
  std::vector<PlyProp> props;
};

class PlySource {
 public:
  PlySource(std::istream& in, bool binary) : in_(in), binary_(binary) {}
  void beginRecord() {
    if (!binary_) {
      std::string line;
      std::getline(in_, line);
      stripCr(line);
      line_.clear();
      line_.str(line);
    }
  }
  double scalar(const std::string& type) {
    if (!binary_) {
      double v = 0.0;
      line_ >> v;
      if (!line_) throw FoundationPoseError("Malformed ASCII PLY scalar");
      return v;
    }
    if (type == "char" || type == "int8") return read<std::int8_t>();
    if (type == "uchar" || type == "uint8") return read<std::uint8_t>();
    if (type == "short" || type == "int16") return read<std::int16_t>();
    if (type == "ushort" || type == "uint16") return read<std::uint16_t>();
    if (type == "int" || type == "int32") return read<std::int32_t>();
    if (type == "uint" || type == "uint32") return read<std::uint32_t>();
    if (type == "float" || type == "float32") return read<float>();
    if (type == "double" || type == "float64") return read<double>();
    throw FoundationPoseError("Unsupported PLY scalar type: " + type);
  }
  std::uint32_t count(const std::string& type) {
    const double v = scalar(type);
    if (v < 0.0) throw FoundationPoseError("Negative PLY list count");
    return static_cast<std::uint32_t>(v);
  }

 private:
  template <class T>
  double read() {
    T v{};
    in_.read(reinterpret_cast<char*>(&v), sizeof(T));
    if (!in_) throw FoundationPoseError("Unexpected EOF while reading binary PLY");
    return static_cast<double>(v);
  }
  std::istream& in_;
  bool binary_;
  std::istringstream line_;
};

Mesh loadPly(const std::filesystem::path& path) {
  std::ifstream in(path, std::ios::binary);
  if (!in) throw FoundationPoseError("Failed to open PLY mesh: " + path.string());
  std::string line;
  std::getline(in, line);
  stripCr(line);
  if (line != "ply") throw FoundationPoseError("Not a PLY file: " + path.string());
  bool binary = false;
  std::vector<PlyElem> elems;
  while (std::getline(in, line)) {
    stripCr(line);
    if (line == "end_header") break;
    std::istringstream iss(line);
    std::string tag;
    iss >> tag;
    if (tag == "format") {
      std::string fmt;
      iss >> fmt;
      if (fmt == "binary_little_endian") {
        binary = true;
      } else if (fmt != "ascii") {
        throw FoundationPoseError("Unsupported PLY format: " + fmt);
      }
    } else if (tag == "element") {
      PlyElem e;
      iss >> e.name >> e.count;
      elems.push_back(e);
    } else if (tag == "property" && !elems.empty()) {
      PlyProp p;
      std::string kind;
      iss >> kind;
      if (kind == "list") {
        p.list = true;
        iss >> p.count_type >> p.item_type >> p.name;
      } else {
        p.type = kind;
        iss >> p.name;
      }
      elems.back().props.push_back(p);
    }
  }
  Mesh mesh;
  mesh.source_path = path.string();
  PlySource src(in, binary);
  for (const PlyElem& e : elems) {
    if (e.name == "vertex") {
      mesh.vertices.resize(e.count);
      mesh.vertex_colors.assign(e.count, Vec3u8{128, 128, 128});
      mesh.normals.resize(e.count);
      for (std::size_t i = 0; i < e.count; ++i) {
        src.beginRecord();
        Vec3f n{};
        bool has_n = false, has_uv = false;
        float u = 0.0f, v = 0.0f;
        for (const PlyProp& p : e.props) {
          if (p.list) {
            const std::uint32_t c = src.count(p.count_type);
            for (std::uint32_t j = 0; j < c; ++j) (void)src.scalar(p.item_type);
            continue;
          }
          const double val = src.scalar(p.type);
          Vec3f& vx = mesh.vertices[i];
          auto u8 = [](double x) { return static_cast<std::uint8_t>(std::clamp(x, 0.0, 255.0)); };
          if (p.name == "x") vx.x = static_cast<float>(val);
          else if (p.name == "y") vx.y = static_cast<float>(val);
          else if (p.name == "z") vx.z = static_cast<float>(val);
          else if (p.name == "nx") { n.x = static_cast<float>(val); has_n = true; }
          else if (p.name == "ny") { n.y = static_cast<float>(val); has_n = true; }
          else if (p.name == "nz") { n.z = static_cast<float>(val); has_n = true; }
          else if (p.name == "red" || p.name == "diffuse_red") mesh.vertex_colors[i].r = u8(val);
          else if (p.name == "green" || p.name == "diffuse_green") mesh.vertex_colors[i].g = u8(val);
          else if (p.name == "blue" || p.name == "diffuse_blue") mesh.vertex_colors[i].b = u8(val);
          else if (p.name == "texture_u") { u = static_cast<float>(val); has_uv = true; }
          else if (p.name == "texture_v") { v = static_cast<float>(val); has_uv = true; }
        }
        if (has_uv) {
          if (mesh.uvs.size() != mesh.vertices.size()) mesh.uvs.resize(mesh.vertices.size());
          mesh.uvs[i] = {u, v};
        }
        if (has_n) mesh.normals[i] = normalizeOrZero(n);
      }
    } else if (e.name == "face") {
      for (std::size_t i = 0; i < e.count; ++i) {
        src.beginRecord();
        std::vector<std::uint32_t> idx;
        for (const PlyProp& p : e.props) {
          if (p.list) {
            const std::uint32_t c = src.count(p.count_type);
            std::vector<std::uint32_t> vals(c);
            for (std::uint32_t j = 0; j < c; ++j) vals[j] = static_cast<std::uint32_t>(src.scalar(p.item_type));
            if (p.name == "vertex_indices" || p.name == "vertex_index") idx = std::move(vals);
          } else {
            (void)src.scalar(p.type);
          }
        }
        for (std::size_t j = 1; j + 1 < idx.size(); ++j) mesh.faces.push_back({idx[0], idx[j], idx[j + 1]});
      }
    } else {
      for (std::size_t i = 0; i < e.count; ++i) {
        src.beginRecord();
        if (!binary) continue;
        for (const PlyProp& p : e.props) {
          if (p.list) {
            const std::uint32_t c = src.count(p.count_type);
            for (std::uint32_t j = 0; j < c; ++j) (void)src.scalar(p.item_type);
          } else {
            (void)src.scalar(p.type);
          }
        }
      }
    }
  }
  if (mesh.vertices.empty() || mesh.faces.empty()) {
    throw FoundationPoseError("PLY mesh has no usable vertices/faces: " + path.string());
  }
  const bool normals_ok = mesh.normals.size() == mesh.vertices.size() &&
                          std::any_of(mesh.normals.begin(), mesh.normals.end(),
                                      [](Vec3f n) { return norm(n) > 0.5f; });
  if (!normals_ok) computeVertexNormals(mesh);
  // Textures (PNG) are not decoded by this build: textured PLYs render with
  // their vertex colours (grey if none).
  return mesh;
}

}  // namespace

Mesh loadMesh(const std::filesystem::path& path) {
  const std::string ext = lowerExt(path);
  if (ext == ".obj") return loadObj(path);
  if (ext == ".ply") return loadPly(path);
  throw FoundationPoseError("Unsupported mesh extension '" + ext + "'. Expected .obj or .ply");
}

void computeVertexNormals(Mesh& mesh) {
  mesh.normals.assign(mesh.vertices.size(), Vec3f{});
  const std::size_t nv = mesh.vertices.size();
  for (const auto& f : mesh.faces) {
    if (f[0] >= nv || f[1] >= nv || f[2] >= nv) continue;
    const Vec3f a = mesh.vertices[f[0]], b = mesh.vertices[f[1]], c = mesh.vertices[f[2]];
    const Vec3f n = cross(b - a, c - a);
    for (int k = 0; k < 3; ++k) mesh.normals[f[k]] = mesh.normals[f[k]] + n;
  }
  for (Vec3f& n : mesh.normals) {
    n = normalizeOrZero(n);
    if (norm(n) < 1e-6f) n = {0.0f, 0.0f, 1.0f};
  }
}

PreprocessedMesh preprocessMesh(const Mesh& mesh, const Config& config) {
  if (mesh.vertices.size() < 4 || mesh.faces.empty()) {
    throw FoundationPoseError("Mesh must contain at least four vertices and one face");
  }
  Vec3f lo{std::numeric_limits<float>::max(), std::numeric_limits<float>::max(),
           std::numeric_limits<float>::max()};
  Vec3f hi{std::numeric_limits<float>::lowest(), std::numeric_limits<float>::lowest(),
           std::numeric_limits<float>::lowest()};
  for (Vec3f v : mesh.vertices) {
    lo = {std::min(lo.x, v.x), std::min(lo.y, v.y), std::min(lo.z, v.z)};
    hi = {std::max(hi.x, v.x), std::max(hi.y, v.y), std::max(hi.z, v.z)};
  }
  PreprocessedMesh out;
  out.center = (lo + hi) * 0.5f;
  out.centered_mesh = mesh;
  for (Vec3f& v : out.centered_mesh.vertices) v = v - out.center;
  const auto& cv = out.centered_mesh.vertices;
  const std::size_t samples = std::min<std::size_t>(static_cast<std::size_t>(config.mesh_sample_points), cv.size());
  const std::size_t stride = std::max<std::size_t>(1, cv.size() / std::max<std::size_t>(samples, 1));
  std::vector<Vec3f> s;
  for (std::size_t i = 0; i < cv.size() && s.size() < samples; i += stride) s.push_back(cv[i]);
  // Diameter: the largest pairwise distance of the strided samples.
  float d = 0.0f;
  for (std::size_t i = 0; i < s.size(); ++i)
    for (std::size_t j = i + 1; j < s.size(); ++j) d = std::max(d, norm(s[i] - s[j]));
  if (d <= 0.0f) d = norm(hi - lo);
  out.diameter = std::max(d, 1e-6f);
  return out;
}

namespace fpb_host {

namespace {

using M3 = std::array<float, 9>;

M3 mul3(const M3& a, const M3& b) {
  M3 o{};
  for (int r = 0; r < 3; ++r)
    for (int c = 0; c < 3; ++c) {
      float v = 0.0f;
      for (int k = 0; k < 3; ++k) v += a[r * 3 + k] * b[k * 3 + c];
      o[r * 3 + c] = v;
    }
  return o;
}

M3 transpose3(const M3& m) {
  M3 o{};
  for (int r = 0; r < 3; ++r)
    for (int c = 0; c < 3; ++c) o[r * 3 + c] = m[c * 3 + r];
  return o;
}

// Icosahedron subdivided (edge midpoints pushed to the unit sphere) until it
// has at least min_vertices vertices.
std::vector<Vec3f> icosphereVertices(int min_vertices) {
  const float t = (1.0f + std::sqrt(5.0f)) * 0.5f;
  std::vector<Vec3f> v = {{-1, t, 0}, {1, t, 0}, {-1, -t, 0}, {1, -t, 0}, {0, -1, t}, {0, 1, t},
                          {0, -1, -t}, {0, 1, -t}, {t, 0, -1}, {t, 0, 1}, {-t, 0, -1}, {-t, 0, 1}};
  for (Vec3f& p : v) p = normalizeOrZero(p);
  std::vector<std::array<int, 3>> f = {{0, 11, 5}, {0, 5, 1},  {0, 1, 7},   {0, 7, 10}, {0, 10, 11},
                                       {1, 5, 9},  {5, 11, 4}, {11, 10, 2}, {10, 7, 6}, {7, 1, 8},
                                       {3, 9, 4},  {3, 4, 2},  {3, 2, 6},   {3, 6, 8},  {3, 8, 9},
                                       {4, 9, 5},  {2, 4, 11}, {6, 2, 10},  {8, 6, 7},  {9, 8, 1}};
  while (static_cast<int>(v.size()) < min_vertices) {
    std::map<std::pair<int, int>, int> mids;
    auto mid = [&](int a, int b) {
      const auto key = std::minmax(a, b);
      auto it = mids.find(key);
      if (it != mids.end()) return it->second;
      const int idx = static_cast<int>(v.size());
      v.push_back(normalizeOrZero((v[a] + v[b]) * 0.5f));
      mids.emplace(key, idx);
      return idx;
    };
    std::vector<std::array<int, 3>> next;
    next.reserve(f.size() * 4);
    for (const auto& tri : f) {
      const int ab = mid(tri[0], tri[1]), bc = mid(tri[1], tri[2]), ca = mid(tri[2], tri[0]);
      next.push_back({tri[0], ab, ca});
      next.push_back({tri[1], bc, ab});
      next.push_back({tri[2], ca, bc});
      next.push_back({ab, bc, ca});
    }
    f = std::move(next);
  }
  return v;
}

}  // namespace

// Object-in-camera rotations for every icosphere viewpoint and in-plane step:
// the camera sits on the unit sphere looking at the origin (z towards the
// object, x = up x z, y = z x x), rotated in-plane by j*step about its z, and
// the hypothesis is the inverse (transpose) of that camera rotation. Rotations
// closer than cluster_threshold_deg to an earlier one are dropped.
std::vector<Mat3f> makeRotationGrid(const Config& config) {
  const float pi = std::numbers::pi_v<float>;
  const std::vector<Vec3f> views = icosphereVertices(config.min_n_views);
  const int n_inplane = std::max(1, static_cast<int>(std::round(360.0f / config.inplane_step_deg)));
  const float step = config.inplane_step_deg * pi / 180.0f;
  std::vector<M3> rots;
  for (Vec3f view : views) {
    const Vec3f z = normalizeOrZero(view * -1.0f);
    Vec3f x = cross({0.0f, 0.0f, 1.0f}, z);
    if (norm(x) < 0.001f) x = {1.0f, 0.0f, 0.0f};
    x = normalizeOrZero(x);
    const Vec3f y = normalizeOrZero(cross(z, x));
    const M3 base = {x.x, y.x, z.x, x.y, y.y, z.y, x.z, y.z, z.z};
    for (int j = 0; j < n_inplane; ++j) {
      const float th = static_cast<float>(j) * step;
      const float c = std::cos(th), s = std::sin(th);
      const M3 rz = {c, -s, 0.0f, s, c, 0.0f, 0.0f, 0.0f, 1.0f};
      rots.push_back(transpose3(mul3(base, rz)));
    }
  }
  const float threshold = config.cluster_threshold_deg * pi / 180.0f;
  std::vector<M3> kept;
  for (const M3& cand : rots) {
    bool fresh = true;
    for (const M3& k : kept) {
      const M3 rel = mul3(cand, transpose3(k));
      const float cos_t = std::clamp((rel[0] + rel[4] + rel[8] - 1.0f) * 0.5f, -1.0f, 1.0f);
      if (std::acos(cos_t) < threshold) {
        fresh = false;
        break;
      }
    }
    if (fresh) kept.push_back(cand);
  }
  std::vector<Mat3f> out(kept.size());
  for (std::size_t i = 0; i < kept.size(); ++i) std::copy(kept[i].begin(), kept[i].end(), out[i].values.begin());
  return out;
}

}  // namespace fpb_host
}  // namespace foundation_pose_nvidia

namespace fpb {
int fail(const std::string& msg);
}

extern "C" int fpk_load_mesh(const char* path, float mesh_unit_scale, int* n_vertices, int* n_faces,
                             float* vertices, float* normals, uint8_t* colors, int32_t* faces,
                             float* center3, float* diameter) {
  using namespace foundation_pose_nvidia;
  try {
    if (path == nullptr || n_vertices == nullptr || n_faces == nullptr) {
      return fpb::fail("fpk_load_mesh: path and count outputs are required");
    }
    Mesh mesh = loadMesh(path);
    if (mesh_unit_scale > 0.0f && mesh_unit_scale != 1.0f) {
      for (Vec3f& v : mesh.vertices) v = v * mesh_unit_scale;
    }
    const PreprocessedMesh pm = preprocessMesh(mesh, Config{});
    const Mesh& m = pm.centered_mesh;
    *n_vertices = static_cast<int>(m.vertices.size());
    *n_faces = static_cast<int>(m.faces.size());
    if (vertices != nullptr) {
      for (std::size_t i = 0; i < m.vertices.size(); ++i) {
        vertices[3 * i] = m.vertices[i].x;
        vertices[3 * i + 1] = m.vertices[i].y;
        vertices[3 * i + 2] = m.vertices[i].z;
        const Vec3f n = i < m.normals.size() ? m.normals[i] : Vec3f{0.0f, 0.0f, 1.0f};
        if (normals != nullptr) {
          normals[3 * i] = n.x;
          normals[3 * i + 1] = n.y;
          normals[3 * i + 2] = n.z;
        }
        const Vec3u8 c = i < m.vertex_colors.size() ? m.vertex_colors[i] : Vec3u8{};
        if (colors != nullptr) {
          colors[3 * i] = c.r;
          colors[3 * i + 1] = c.g;
          colors[3 * i + 2] = c.b;
        }
      }
    }
    if (faces != nullptr) {
      for (std::size_t i = 0; i < m.faces.size(); ++i)
        for (int k = 0; k < 3; ++k) faces[3 * i + k] = static_cast<int32_t>(m.faces[i][k]);
    }
    if (center3 != nullptr) {
      center3[0] = pm.center.x;
      center3[1] = pm.center.y;
      center3[2] = pm.center.z;
    }
    if (diameter != nullptr) *diameter = pm.diameter;
    return 0;
  } catch (const std::exception& e) {
    return fpb::fail(e.what());
  }
}
