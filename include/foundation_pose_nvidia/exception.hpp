// FoundationPoseError (reference include/foundation_pose_nvidia/exception.hpp:18-21):
// the one exception type the runtime throws; a std::runtime_error.
#pragma once

#include <stdexcept>

#pragma GCC visibility push(default)
namespace foundation_pose_nvidia {

class FoundationPoseError : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};

}  // namespace foundation_pose_nvidia
#pragma GCC visibility pop
