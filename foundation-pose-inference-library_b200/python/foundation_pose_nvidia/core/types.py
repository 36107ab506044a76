from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class PoseEstimate:
    """Pose from register/track: 4x4 row-major object-to-camera (metres)."""

    pose: np.ndarray
    score: float
    elapsed_s: float

    @classmethod
    def from_ctypes(cls, pose_row_major, score: float, elapsed_s: float) -> PoseEstimate:
        return cls(pose=np.asarray(pose_row_major, np.float32).reshape(4, 4).copy(),
                   score=float(score), elapsed_s=float(elapsed_s))
