"""RuntimeConfig: Python view of fp_config_t (reference python/.../core/config.py:16-68)."""
from __future__ import annotations

from dataclasses import dataclass
from enum import IntEnum
from typing import TYPE_CHECKING

from foundation_pose_nvidia.bindings._ctypes_types import Config

if TYPE_CHECKING:
    from foundation_pose_nvidia.bindings._library import FPLibrary


class Precision(IntEnum):
    """Network precision (fp_precision_t)."""

    FP32 = 0
    TF32 = 1
    FP16 = 2
    BF16 = 3


@dataclass
class RuntimeConfig:
    """Fields left as None keep the library defaults (fp_default_config)."""

    n_hypotheses: int | None = None
    n_refine_iters: int | None = None
    n_track_iters: int | None = None
    crop_ratio: float | None = None
    input_width: int | None = None
    input_height: int | None = None
    max_image_width: int | None = None
    max_image_height: int | None = None
    capture_cuda_graph: bool | None = None
    tensorrt_precision: Precision | int | None = None
    batch_size: int | None = None  # appended last, like fp_config_t

    def to_ctypes(self, library: FPLibrary) -> Config:
        cfg = library.default_config()
        for name, value in self.__dict__.items():
            if value is None:
                continue
            setattr(cfg, name, int(value) if name in ("capture_cuda_graph", "tensorrt_precision") else value)
        return cfg

    @classmethod
    def from_ctypes(cls, cfg: Config) -> RuntimeConfig:
        return cls(n_hypotheses=cfg.n_hypotheses, n_refine_iters=cfg.n_refine_iters,
                   n_track_iters=cfg.n_track_iters, crop_ratio=cfg.crop_ratio,
                   input_width=cfg.input_width, input_height=cfg.input_height,
                   max_image_width=cfg.max_image_width, max_image_height=cfg.max_image_height,
                   capture_cuda_graph=bool(cfg.capture_cuda_graph),
                   tensorrt_precision=Precision(cfg.tensorrt_precision), batch_size=cfg.batch_size)
