"""High-level estimator API."""
from foundation_pose_nvidia.core.config import Precision, RuntimeConfig
from foundation_pose_nvidia.core.estimator import Estimator
from foundation_pose_nvidia.core.frame import RgbdFrame
from foundation_pose_nvidia.core.multi_object import (MultiObjectEstimator, MultiObjectPoseEstimate,
                                                     ObjectSpec, RegisterOptions)
from foundation_pose_nvidia.core.options import EstimatorOptions
from foundation_pose_nvidia.core.sharded import gather_shards, register_sharded, shard_range
from foundation_pose_nvidia.core.types import PoseEstimate

__all__ = ["Estimator", "EstimatorOptions", "MultiObjectEstimator", "MultiObjectPoseEstimate",
           "ObjectSpec", "PoseEstimate", "Precision", "RegisterOptions", "RgbdFrame",
           "RuntimeConfig", "gather_shards", "register_sharded", "shard_range"]
