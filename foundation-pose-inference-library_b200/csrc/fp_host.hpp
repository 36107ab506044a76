// Host-side helpers shared by the runtime translation units (internal).
#pragma once

#include <span>
#include <vector>

#include "foundation_pose_nvidia/config.hpp"
#include "foundation_pose_nvidia/types.hpp"

namespace foundation_pose_nvidia {
namespace fpb_host {

std::vector<Mat3f> makeRotationGrid(const Config& config);
Mesh reconstructReferenceMesh(std::span<const ModelFreeReferenceView> refs, const Config& config);

}  // namespace fpb_host
}  // namespace foundation_pose_nvidia
