"""Python bindings for the FoundationPose B200 runtime's C ABI.

Same public surface as the reference package of the same name
(python/src/foundation_pose_nvidia/__init__.py): the high-level estimator API in
:mod:`foundation_pose_nvidia.core` and the ctypes layer in
:mod:`foundation_pose_nvidia.bindings`.
"""
from foundation_pose_nvidia._version import __version__
from foundation_pose_nvidia.bindings import FPLibrary, load_library
from foundation_pose_nvidia.core import (
    Estimator,
    EstimatorOptions,
    MultiObjectEstimator,
    MultiObjectPoseEstimate,
    ObjectSpec,
    PoseEstimate,
    Precision,
    RegisterOptions,
    RgbdFrame,
    RuntimeConfig,
    register_sharded,
    shard_range,
)
from foundation_pose_nvidia.exceptions import FoundationPoseError, LibraryNotFoundError

__all__ = [
    "Estimator", "EstimatorOptions", "FPLibrary", "FoundationPoseError", "LibraryNotFoundError",
    "MultiObjectEstimator", "MultiObjectPoseEstimate", "ObjectSpec", "PoseEstimate", "Precision",
    "RegisterOptions", "RgbdFrame", "RuntimeConfig", "__version__", "load_library", "register_sharded",
    "shard_range",
]
