"""ctypes bindings to the fp_* C ABI (include/foundation_pose_nvidia/c_api.h)."""
from foundation_pose_nvidia.bindings._ctypes_types import (
    Config,
    CreateOptions,
    ImageView,
    PoseResult,
    ReferenceImageView,
)
from foundation_pose_nvidia.bindings._library import FPLibrary, load_library
from foundation_pose_nvidia.bindings._loader import candidate_libraries, repo_root

__all__ = ["Config", "CreateOptions", "FPLibrary", "ImageView", "PoseResult",
           "ReferenceImageView", "candidate_libraries", "load_library", "repo_root"]
