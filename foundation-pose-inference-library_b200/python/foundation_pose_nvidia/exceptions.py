class FoundationPoseError(RuntimeError):
    """Error reported by the runtime (non-zero status / NULL handle)."""


class LibraryNotFoundError(FoundationPoseError):
    """libfoundation_pose_nvidia.so could not be located."""
