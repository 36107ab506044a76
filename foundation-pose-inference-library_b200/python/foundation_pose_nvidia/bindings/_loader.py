"""Locate libfoundation_pose_nvidia.so: explicit path, $FP_LIBRARY, or the
in-tree build (foundation-pose-inference-library_b200/lib)."""
from __future__ import annotations

import os
from pathlib import Path

from foundation_pose_nvidia.exceptions import LibraryNotFoundError

_NAME = "libfoundation_pose_nvidia.so"


def repo_root() -> Path:
    return Path(__file__).resolve().parents[3]


def candidate_libraries(root: Path | None = None) -> list[Path]:
    root = root or repo_root()
    return [root / "lib" / _NAME, root / "build" / _NAME, root.parent / "build" / _NAME]


def resolve_library_path(path: Path | str | None = None) -> Path:
    if path is not None:
        selected = Path(path).expanduser().resolve()
    elif os.environ.get("FP_LIBRARY"):
        selected = Path(os.environ["FP_LIBRARY"]).expanduser().resolve()
    else:
        selected = next((p for p in candidate_libraries() if p.exists()), None)
    if selected is None or not selected.is_file():
        searched = "\n  ".join(str(p) for p in candidate_libraries())
        raise LibraryNotFoundError(f"Could not find {_NAME}. Searched:\n  {searched}")
    return selected
