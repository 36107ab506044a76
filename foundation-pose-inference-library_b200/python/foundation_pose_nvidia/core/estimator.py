"""Estimator: context-managed fp_create / fp_register_frame / fp_track_frame
(reference core/estimator.py:21-223). Timing brackets each call with a device
synchronize and time.perf_counter, as the reference wrapper does."""
from __future__ import annotations

import ctypes as C
import time
from typing import Any

import numpy as np

from foundation_pose_nvidia.bindings import Config, CreateOptions, FPLibrary, PoseResult, load_library
from foundation_pose_nvidia.core.config import RuntimeConfig
from foundation_pose_nvidia.core.frame import RgbdFrame
from foundation_pose_nvidia.core.options import EstimatorOptions
from foundation_pose_nvidia.core.types import PoseEstimate
from foundation_pose_nvidia.exceptions import FoundationPoseError


class Estimator:
    def __init__(self, options: EstimatorOptions, config: RuntimeConfig | Config, *,
                 library: FPLibrary | None = None, obj_id: int = 0,
                 prepare_batch: int | None = None, prepare_track_batch: bool = False):
        self.handle = None
        self.library = library or load_library(print_build_info=True)
        self.lib = self.library.cdll
        self.obj_id = int(obj_id)
        self.setup_timings: list[dict[str, Any]] = []
        self._strings = options.encoded_strings()
        self._config = config.to_ctypes(self.library) if isinstance(config, RuntimeConfig) else config
        s = self._strings
        create = CreateOptions(C.c_char_p(s[0]), int(options.device_id), C.c_float(options.mesh_unit_scale),
                               *[C.c_char_p(v) for v in s[1:]])
        err = C.create_string_buffer(4096)
        t0 = time.perf_counter()
        self.handle = self.lib.fp_create(C.byref(create), C.byref(self._config), err, len(err))
        self.setup_timings.append({"obj_id": self.obj_id, "type": "create_estimator",
                                   "time_s": time.perf_counter() - t0, "cad_path": str(options.cad_path)})
        if not self.handle:
            raise FoundationPoseError(err.value.decode("utf-8"))
        try:
            if options.prepare and prepare_batch is not None:
                self._prepare(int(prepare_batch))
            elif prepare_track_batch:
                self._prepare(1)
        except BaseException:
            self.close()
            raise

    @property
    def config(self) -> Config:
        return self._config

    def _prepare(self, batch_size: int) -> None:
        err = C.create_string_buffer(4096)
        t0 = time.perf_counter()
        status = self.lib.fp_prepare(self.handle, batch_size, err, len(err))
        self.library.synchronize()
        self.setup_timings.append({"obj_id": self.obj_id, "type": "prepare_estimator",
                                   "time_s": time.perf_counter() - t0, "batch_size": batch_size})
        if status != 0:
            raise FoundationPoseError(err.value.decode("utf-8"))

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.fp_destroy(self.handle)
            self.handle = None

    __del__ = close

    def __enter__(self) -> Estimator:
        return self

    def __exit__(self, *_: object) -> None:
        self.close()

    def register(self, frame, *, n_refine: int = -1, n_hypotheses: int = -1) -> PoseEstimate:
        if isinstance(frame, RgbdFrame):
            if frame.mask is None:
                raise ValueError("register requires a mask")
            return self._register_arrays(frame.rgb, frame.depth_m, frame.mask, frame.intrinsics,
                                         n_refine, n_hypotheses)
        rgb, depth_m, mask, k = frame
        return self._register_arrays(rgb, depth_m, mask, k, n_refine, n_hypotheses)

    def track(self, frame, *, n_refine: int = -1) -> PoseEstimate:
        if isinstance(frame, RgbdFrame):
            view = frame.to_image_view(with_mask=False)
        else:
            rgb, depth_m, k = frame
            view = RgbdFrame(rgb, depth_m, k).to_image_view(with_mask=False)
        return self._track_view(view, n_refine)

    def register_arrays(self, rgb, depth_m, mask, intrinsics, n_refine: int, n_hypotheses: int):
        r = self._register_arrays(rgb, depth_m, mask, intrinsics, n_refine, n_hypotheses)
        return (r.pose, r.score), r.elapsed_s

    def track_arrays(self, rgb, depth_m, intrinsics, n_refine: int):
        r = self.track((rgb, depth_m, intrinsics), n_refine=n_refine)
        return r.pose, r.elapsed_s

    def _register_arrays(self, rgb, depth_m, mask, intrinsics, n_refine, n_hypotheses) -> PoseEstimate:
        view = RgbdFrame(rgb, depth_m, intrinsics, mask).to_image_view(with_mask=True)
        result = PoseResult()
        err = C.create_string_buffer(4096)
        self.library.synchronize()
        t0 = time.perf_counter()
        status = self.lib.fp_register_frame(self.handle, C.byref(view), n_refine, n_hypotheses,
                                            C.byref(result), err, len(err))
        self.library.synchronize()
        elapsed = time.perf_counter() - t0
        if status != 0:
            raise FoundationPoseError(err.value.decode("utf-8"))
        return PoseEstimate.from_ctypes(result.pose_row_major, result.score, elapsed)

    def _track_view(self, view, n_refine: int) -> PoseEstimate:
        result = PoseResult()
        err = C.create_string_buffer(4096)
        self.library.synchronize()
        t0 = time.perf_counter()
        status = self.lib.fp_track_frame(self.handle, C.byref(view), n_refine, C.byref(result), err,
                                         len(err))
        self.library.synchronize()
        elapsed = time.perf_counter() - t0
        if status != 0:
            raise FoundationPoseError(err.value.decode("utf-8"))
        return PoseEstimate.from_ctypes(result.pose_row_major, result.score, elapsed)
