// Mesh ingest (reference include/foundation_pose_nvidia/mesh.hpp): OBJ / PLY
// loading, area-weighted vertex normals, and the preprocessing an estimator
// applies (bounding-box centring, diameter).
#pragma once

#include <filesystem>

#include "foundation_pose_nvidia/config.hpp"
#include "foundation_pose_nvidia/types.hpp"

#pragma GCC visibility push(default)
namespace foundation_pose_nvidia {

Mesh loadMesh(const std::filesystem::path& path);
void computeVertexNormals(Mesh& mesh);
PreprocessedMesh preprocessMesh(const Mesh& mesh, const Config& config);

}  // namespace foundation_pose_nvidia
#pragma GCC visibility pop
