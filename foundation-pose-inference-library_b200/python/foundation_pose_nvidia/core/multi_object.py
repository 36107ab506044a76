"""MultiObjectEstimator over the fp_group_* API (reference core/multi_object.py:14-279)."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import numpy as np

from foundation_pose_nvidia.bindings import CreateOptions, PoseResult, load_library
from foundation_pose_nvidia.core.frame import RgbdFrame

STATUS_NAMES = {0: "OK", 1: "FAILED", 2: "SKIPPED"}


@dataclass
class ObjectSpec:
    name: str
    cad_path: Path
    mesh_unit_scale: float = 1.0


@dataclass(frozen=True)
class MultiObjectPoseEstimate:
    object_spec: ObjectSpec
    pose: np.ndarray
    score: float
    status: int
    status_name: str


@dataclass
class RegisterOptions:
    library_path: Path | None
    refine_model_path: Path
    score_model_path: Path
    engine_cache_dir: Path
    device_id: int = 0
    n_hypotheses: int = 64
    n_refine: int = 3
    capture_cuda_graph: bool = False
    prepare: bool = True
    refine_translation_output_name: str = "trans"
    refine_rotation_output_name: str = "rot"
    score_output_name: str = "score"
    tensorrt_precision: int | None = None


def _b(v) -> bytes | None:
    return None if v is None else str(v).encode("utf-8")


class MultiObjectEstimator:
    def __init__(self, options: RegisterOptions):
        self.options = options
        Path(options.engine_cache_dir).mkdir(parents=True, exist_ok=True)
        self.library = self.lib = self.group = self.config = None
        self.objects: list[ObjectSpec] = []
        self._strings: list[bytes | None] = []

    def close(self) -> None:
        if getattr(self, "group", None) and getattr(self, "lib", None):
            self.lib.fp_group_destroy(self.group)
        self.group = self.lib = self.library = self.config = None
        self.objects, self._strings = [], []

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self) -> MultiObjectEstimator:
        return self

    def __exit__(self, *_: object) -> None:
        self.close()

    def _create_group(self, frame: Any, objects: list[ObjectSpec]) -> None:
        if self.group:
            if [o.name for o in objects] != [o.name for o in self.objects]:
                raise ValueError("Cannot reuse a multi-object group with different objects")
            return
        o = self.options
        self.library = load_library(o.library_path, print_build_info=False)
        self.library.bind_group_api(len(objects))
        self.lib = self.library.cdll
        cfg = self.library.default_config()
        cfg.max_image_width, cfg.max_image_height = int(frame.rgb.shape[1]), int(frame.rgb.shape[0])
        if o.n_hypotheses > 0:
            cfg.n_hypotheses = o.n_hypotheses
        if o.n_refine >= 0:
            cfg.n_refine_iters = o.n_refine
        cfg.capture_cuda_graph = 1 if o.capture_cuda_graph else 0
        if o.tensorrt_precision is not None:
            cfg.tensorrt_precision = int(o.tensorrt_precision)
        self.config = cfg
        self.objects = list(objects)
        opts = (CreateOptions * len(objects))()
        for i, obj in enumerate(objects):
            strs = [_b(obj.cad_path), _b(o.refine_model_path), _b(o.score_model_path),
                    _b(o.engine_cache_dir), _b(o.refine_translation_output_name),
                    _b(o.refine_rotation_output_name), _b(o.score_output_name)]
            self._strings.extend(strs)
            opts[i].cad_path, opts[i].device_id = strs[0], o.device_id
            opts[i].mesh_unit_scale = obj.mesh_unit_scale
            opts[i].refine_model_path, opts[i].score_model_path, opts[i].engine_cache_dir = strs[1:4]
            opts[i].rendered_input_name, opts[i].observed_input_name = b"inputA", b"inputB"
            (opts[i].refine_translation_output_name, opts[i].refine_rotation_output_name,
             opts[i].score_output_name) = strs[4:7]
        err = C.create_string_buffer(4096)
        self.group = self.lib.fp_group_create(opts, len(objects), C.byref(cfg), err, len(err))
        if not self.group:
            raise RuntimeError(f"fp_group_create failed: {err.value.decode(errors='replace')}")
        if self.lib.fp_group_size(self.group) != len(objects):
            raise RuntimeError("fp_group_size does not match the object count")
        if o.prepare:
            batch = cfg.n_hypotheses if o.n_hypotheses <= 0 else o.n_hypotheses
            rc = self.lib.fp_group_prepare(self.group, batch, err, len(err))
            if rc != 0:
                raise RuntimeError(f"fp_group_prepare failed for {rc} object(s): "
                                   f"{err.value.decode(errors='replace')}")

    def _estimates(self, results, statuses) -> list[MultiObjectPoseEstimate]:
        out = []
        for i, obj in enumerate(self.objects):
            st = int(statuses[i])
            out.append(MultiObjectPoseEstimate(
                object_spec=obj, pose=np.asarray(results[i].pose_row_major, np.float32).reshape(4, 4).copy(),
                score=float(results[i].score), status=st, status_name=STATUS_NAMES.get(st, "UNKNOWN")))
        return out

    def register(self, frame: Any, objects: list[ObjectSpec], masks: dict[str, np.ndarray],
                 depth: np.ndarray) -> list[MultiObjectPoseEstimate]:
        self._create_group(frame, objects)
        view = RgbdFrame(frame.rgb, depth, frame.k).to_image_view(with_mask=False)
        arrays = [None if masks.get(o.name) is None else np.ascontiguousarray(masks[o.name], np.uint8)
                  for o in self.objects]
        ptrs = (C.POINTER(C.c_uint8) * len(arrays))(
            *[C.POINTER(C.c_uint8)() if a is None else a.ctypes.data_as(C.POINTER(C.c_uint8)) for a in arrays])
        results = (PoseResult * len(self.objects))()
        statuses = (C.c_int * len(self.objects))()
        err = C.create_string_buffer(4096)
        rc = self.lib.fp_group_register_frame(self.group, C.byref(view), ptrs, self.options.n_refine,
                                              self.options.n_hypotheses, results, statuses, err, len(err))
        if rc != 0:
            raise RuntimeError(f"fp_group_register_frame failed for {rc} object(s): "
                               f"{err.value.decode(errors='replace')}")
        return self._estimates(results, statuses)

    def track(self, frame: Any, depth: np.ndarray, *, active=None, n_refine: int = -1):
        if not self.group:
            raise RuntimeError("track requires a prior successful register call")
        view = RgbdFrame(frame.rgb, depth, frame.k).to_image_view(with_mask=False)
        active_arr = None
        if active is not None:
            if isinstance(active, dict):
                flags = [1 if active.get(o.name, True) else 0 for o in self.objects]
            else:
                flags = [1 if v else 0 for v in active]
                if len(flags) != len(self.objects):
                    raise ValueError(f"active has {len(flags)} entries, expected {len(self.objects)}")
            active_arr = (C.c_int * len(self.objects))(*flags)
        results = (PoseResult * len(self.objects))()
        statuses = (C.c_int * len(self.objects))()
        err = C.create_string_buffer(4096)
        rc = self.lib.fp_group_track_frame(self.group, C.byref(view), active_arr, n_refine, results,
                                           statuses, err, len(err))
        if rc != 0:
            raise RuntimeError(f"fp_group_track_frame failed for {rc} object(s): "
                               f"{err.value.decode(errors='replace')}")
        return self._estimates(results, statuses)
