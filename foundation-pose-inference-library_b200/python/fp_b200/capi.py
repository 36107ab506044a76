"""ctypes binding of the stable fp_* C ABI of libfoundation_pose_nvidia.so.

This is the thin Python handle the tests and the benchmark use to drive the
library exactly as an FFI caller would: plain structs, raw pointers, return
codes and error buffers. Applications keep using the reference's own Python
package (python/src/foundation_pose_nvidia in the reference) unchanged; point
its loader at this library with FP_LIBRARY.

The struct classes below mirror include/foundation_pose_nvidia/c_api.h, which
keeps the reference's layouts (reference include/foundation_pose_nvidia/
c_api.h:174-269): field order and types are the ABI and must not change.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Sequence

import numpy as np

LIBRARY = Path(__file__).resolve().parents[2] / "lib" / "libfoundation_pose_nvidia.so"

FP_PRECISION_FP32, FP_PRECISION_TF32, FP_PRECISION_FP16, FP_PRECISION_BF16 = 0, 1, 2, 3
FP_OBJECT_OK, FP_OBJECT_FAILED, FP_OBJECT_SKIPPED = 0, 1, 2
SCORE_FEATURE_DIM = 512  # floats per hypothesis exchanged by the sharded register

_str = C.c_char_p
_u8p = C.POINTER(C.c_uint8)
_f32p = C.POINTER(C.c_float)


class fp_create_options_t(C.Structure):
    _fields_ = [("cad_path", _str), ("device_id", C.c_int), ("mesh_unit_scale", C.c_float),
                ("refine_model_path", _str), ("score_model_path", _str), ("engine_cache_dir", _str),
                ("refine_model_name", _str), ("score_model_name", _str), ("rendered_input_name", _str),
                ("observed_input_name", _str), ("refine_translation_output_name", _str),
                ("refine_rotation_output_name", _str), ("score_output_name", _str)]


class fp_config_t(C.Structure):
    _fields_ = [("n_hypotheses", C.c_int), ("n_refine_iters", C.c_int), ("n_track_iters", C.c_int),
                ("crop_ratio", C.c_float), ("input_width", C.c_int), ("input_height", C.c_int),
                ("max_image_width", C.c_int), ("max_image_height", C.c_int),
                ("capture_cuda_graph", C.c_int), ("model_free_sample_stride", C.c_int),
                ("model_free_max_vertices", C.c_int), ("model_free_depth_edge_threshold", C.c_float),
                ("tensorrt_precision", C.c_int), ("batch_size", C.c_int)]


class fp_image_view_t(C.Structure):
    _fields_ = [("width", C.c_int), ("height", C.c_int), ("rgb_u8", _u8p), ("depth_m", _f32p),
                ("mask_u8", _u8p), ("k_row_major", _f32p)]


class fp_reference_image_view_t(C.Structure):
    _fields_ = [("width", C.c_int), ("height", C.c_int), ("rgb_u8", _u8p), ("depth_m", _f32p),
                ("mask_u8", _u8p), ("k_row_major", _f32p), ("camera_to_world_row_major", _f32p)]


class fp_pose_result_t(C.Structure):
    _fields_ = [("pose_row_major", C.c_float * 16), ("score", C.c_float)]


class FpError(RuntimeError):
    """A non-zero return (or NULL handle) from the library, with its message."""


@dataclass
class CallResult:
    rc: int
    pose: np.ndarray  # 4x4 float32, object -> camera
    score: float
    error: str


def _address(buf: Any) -> int:
    """Device or host address of a torch tensor, a __cuda_array_interface__
    object or a numpy array (which must stay alive while the view is used)."""
    cai = getattr(buf, "__cuda_array_interface__", None)
    if cai is not None:
        return int(cai["data"][0])
    if hasattr(buf, "data_ptr"):
        return int(buf.data_ptr())
    return int(buf.ctypes.data)


def _host(a: Any, dtype) -> Any:
    if getattr(a, "__cuda_array_interface__", None) is not None or hasattr(a, "data_ptr"):
        return a  # a device tensor: the caller keeps it contiguous and alive
    return np.ascontiguousarray(a, dtype=dtype)


def image_view(rgb: Any, depth: Any, K: Any, mask: Any = None) -> fp_image_view_t:
    """fp_image_view_t over host (numpy) or device (torch / CUDA-array) buffers:
    rgb [H,W,3] u8, depth [H,W] f32 metres, K 3x3 (host), mask [H,W] u8 or None.
    The view holds references to every buffer it points into."""
    rgb, depth = _host(rgb, np.uint8), _host(depth, np.float32)
    mask = None if mask is None else _host(mask, np.uint8)
    k = np.ascontiguousarray(np.asarray(K, np.float32).reshape(9))
    h, w = int(depth.shape[0]), int(depth.shape[1])
    v = fp_image_view_t(w, h, C.cast(_address(rgb), _u8p), C.cast(_address(depth), _f32p),
                        C.cast(_address(mask), _u8p) if mask is not None else _u8p(),
                        k.ctypes.data_as(_f32p))
    v._keep = (rgb, depth, mask, k)
    return v


def reference_view(rgb: np.ndarray, depth: np.ndarray, mask: np.ndarray | None, K: Any,
                   camera_to_world: Any = None) -> fp_reference_image_view_t:
    """fp_reference_image_view_t for fp_create_model_free (host buffers only)."""
    rgb = np.ascontiguousarray(rgb, np.uint8)
    depth = np.ascontiguousarray(depth, np.float32)
    mask = None if mask is None else np.ascontiguousarray(mask, np.uint8)
    k = np.ascontiguousarray(np.asarray(K, np.float32).reshape(9))
    c2w = None if camera_to_world is None else np.ascontiguousarray(np.asarray(camera_to_world, np.float32).reshape(16))
    v = fp_reference_image_view_t(depth.shape[1], depth.shape[0], rgb.ctypes.data_as(_u8p),
                                  depth.ctypes.data_as(_f32p),
                                  mask.ctypes.data_as(_u8p) if mask is not None else _u8p(),
                                  k.ctypes.data_as(_f32p), c2w.ctypes.data_as(_f32p) if c2w is not None else _f32p())
    v._keep = (rgb, depth, mask, k, c2w)
    return v


_P = C.c_void_p
_ERR = [C.c_char_p, C.c_size_t]
_SIGNATURES = {
    "fp_default_config": (None, [C.POINTER(fp_config_t)]),
    "fp_create": (_P, [C.POINTER(fp_create_options_t), C.POINTER(fp_config_t)] + _ERR),
    "fp_create_model_free": (_P, [C.POINTER(fp_reference_image_view_t), C.c_size_t,
                                  C.POINTER(fp_create_options_t), C.POINTER(fp_config_t)] + _ERR),
    "fp_prepare": (C.c_int, [_P, C.c_int] + _ERR),
    "fp_destroy": (None, [_P]),
    "fp_register_frame": (C.c_int, [_P, C.POINTER(fp_image_view_t), C.c_int, C.c_int,
                                    C.POINTER(fp_pose_result_t)] + _ERR),
    "fp_track_frame": (C.c_int, [_P, C.POINTER(fp_image_view_t), C.c_int, C.POINTER(fp_pose_result_t)] + _ERR),
    "fp_register_shard_begin": (C.c_int, [_P, C.POINTER(fp_image_view_t), C.c_int, C.c_int, C.c_int, C.c_int,
                                          _P, _P] + _ERR),
    "fp_register_shard_finish": (C.c_int, [_P, _P, _P, C.c_int, C.POINTER(fp_pose_result_t)] + _ERR),
    "fp_group_create": (_P, [C.POINTER(fp_create_options_t), C.c_size_t, C.POINTER(fp_config_t)] + _ERR),
    "fp_group_size": (C.c_size_t, [_P]),
    "fp_group_handle": (_P, [_P, C.c_size_t]),
    "fp_group_prepare": (C.c_int, [_P, C.c_int] + _ERR),
    "fp_group_register_frame": (C.c_int, [_P, C.POINTER(fp_image_view_t), C.POINTER(_u8p), C.c_int, C.c_int,
                                          C.POINTER(fp_pose_result_t), C.POINTER(C.c_int)] + _ERR),
    "fp_group_track_frame": (C.c_int, [_P, C.POINTER(fp_image_view_t), C.POINTER(C.c_int), C.c_int,
                                       C.POINTER(fp_pose_result_t), C.POINTER(C.c_int)] + _ERR),
    "fp_group_destroy": (None, [_P]),
    "fp_synchronize_device": (C.c_int, _ERR),
    "fp_build_info": (C.c_char_p, []),
}


def _pose(r: fp_pose_result_t) -> np.ndarray:
    return np.array(r.pose_row_major, np.float32).reshape(4, 4)


class Api:
    """libfoundation_pose_nvidia.so with every fp_* entry point declared."""

    def __init__(self, path: Path | str | None = None):
        self.path = Path(path) if path is not None else LIBRARY
        if not self.path.is_file():
            raise FileNotFoundError(f"{self.path} is not built (python foundation-pose-inference-library_b200/build.py)")
        self.lib = C.CDLL(str(self.path))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(self.lib, name)
            fn.restype, fn.argtypes = res, args

    @property
    def build_info(self) -> str:
        return self.lib.fp_build_info().decode()

    def default_config(self, **overrides) -> fp_config_t:
        c = fp_config_t()
        self.lib.fp_default_config(C.byref(c))
        for k, v in overrides.items():
            setattr(c, k, int(v) if isinstance(v, bool) else v)
        return c

    @staticmethod
    def options(cad: Any, refine: Any, score: Any, device_id: int = 0, cache_dir: Any = None,
                mesh_unit_scale: float = 1.0) -> fp_create_options_t:
        enc = lambda p: None if p is None else str(p).encode()  # noqa: E731
        o = fp_create_options_t(enc(cad), device_id, mesh_unit_scale, enc(refine), enc(score), enc(cache_dir))
        o._keep = (cad, refine, score, cache_dir)
        return o

    def create(self, options: fp_create_options_t, config: fp_config_t | None = None) -> int:
        err = C.create_string_buffer(2048)
        h = self.lib.fp_create(C.byref(options), C.byref(config) if config is not None else None, err, len(err))
        if not h:
            raise FpError(err.value.decode())
        return h

    def create_model_free(self, refs: Sequence[fp_reference_image_view_t], options: fp_create_options_t,
                          config: fp_config_t | None = None) -> int:
        arr = (fp_reference_image_view_t * len(refs))(*refs)
        err = C.create_string_buffer(2048)
        h = self.lib.fp_create_model_free(arr, len(refs), C.byref(options),
                                          C.byref(config) if config is not None else None, err, len(err))
        if not h:
            raise FpError(err.value.decode())
        return h

    def prepare(self, handle: int, batch: int) -> None:
        err = C.create_string_buffer(2048)
        if self.lib.fp_prepare(handle, batch, err, len(err)) != 0:
            raise FpError(err.value.decode())

    def destroy(self, handle: int | None) -> None:
        self.lib.fp_destroy(handle)

    def register_frame(self, handle: int, view: fp_image_view_t, n_refine: int = -1,
                       n_hypotheses: int = -1) -> CallResult:
        res, err = fp_pose_result_t(), C.create_string_buffer(2048)
        rc = self.lib.fp_register_frame(handle, C.byref(view), n_refine, n_hypotheses, C.byref(res), err, len(err))
        return CallResult(rc, _pose(res), float(res.score), err.value.decode())

    def track_frame(self, handle: int, view: fp_image_view_t, n_refine: int = -1) -> CallResult:
        res, err = fp_pose_result_t(), C.create_string_buffer(2048)
        rc = self.lib.fp_track_frame(handle, C.byref(view), n_refine, C.byref(res), err, len(err))
        return CallResult(rc, _pose(res), float(res.score), err.value.decode())

    def register(self, handle: int, view: fp_image_view_t, n_refine: int = -1, n_hypotheses: int = -1):
        r = self.register_frame(handle, view, n_refine, n_hypotheses)
        if r.rc != 0:
            raise FpError(r.error)
        return r.pose, r.score

    def track(self, handle: int, view: fp_image_view_t, n_refine: int = -1):
        r = self.track_frame(handle, view, n_refine)
        if r.rc != 0:
            raise FpError(r.error)
        return r.pose, r.score

    def synchronize(self) -> None:
        err = C.create_string_buffer(1024)
        if self.lib.fp_synchronize_device(err, len(err)) != 0:
            raise FpError(err.value.decode())

    # -- groups -------------------------------------------------------------
    def group_create(self, objects: Sequence[fp_create_options_t], config: fp_config_t | None = None) -> int:
        arr = (fp_create_options_t * len(objects))(*objects)
        err = C.create_string_buffer(2048)
        g = self.lib.fp_group_create(arr, len(objects), C.byref(config) if config is not None else None, err,
                                     len(err))
        if not g:
            raise FpError(err.value.decode())
        return g

    def group_register(self, group: int, view: fp_image_view_t, masks: Sequence[Any], n_refine: int = -1,
                       n_hypotheses: int = -1):
        """Returns (failures, poses [n,4,4], scores [n], statuses [n], error)."""
        n = len(masks)
        keep = [None if m is None else np.ascontiguousarray(m, np.uint8) for m in masks]
        ptrs = (_u8p * n)(*[_u8p() if m is None else m.ctypes.data_as(_u8p) for m in keep])
        res, st = (fp_pose_result_t * n)(), (C.c_int * n)()
        err = C.create_string_buffer(2048)
        fails = self.lib.fp_group_register_frame(group, C.byref(view), ptrs, n_refine, n_hypotheses, res, st, err,
                                                 len(err))
        return fails, np.stack([_pose(r) for r in res]), np.array([r.score for r in res], np.float32), \
            list(st), err.value.decode()

    def group_track(self, group: int, view: fp_image_view_t, active: Sequence[int] | None, n: int,
                    n_refine: int = -1):
        act = None if active is None else (C.c_int * n)(*active)
        res, st = (fp_pose_result_t * n)(), (C.c_int * n)()
        err = C.create_string_buffer(2048)
        fails = self.lib.fp_group_track_frame(group, C.byref(view), act, n_refine, res, st, err, len(err))
        return fails, np.stack([_pose(r) for r in res]), np.array([r.score for r in res], np.float32), \
            list(st), err.value.decode()

    # -- sharded register ----------------------------------------------------
    def shard_begin(self, handle: int, view: fp_image_view_t, n_refine: int, n_hypotheses: int, begin: int,
                    count: int, features_ptr: int, poses_ptr: int) -> None:
        err = C.create_string_buffer(2048)
        if self.lib.fp_register_shard_begin(handle, C.byref(view), n_refine, n_hypotheses, begin, count,
                                            features_ptr, poses_ptr, err, len(err)) != 0:
            raise FpError(err.value.decode())

    def shard_finish(self, handle: int, features_ptr: int, poses_ptr: int, n_hypotheses: int):
        res, err = fp_pose_result_t(), C.create_string_buffer(2048)
        if self.lib.fp_register_shard_finish(handle, features_ptr, poses_ptr, n_hypotheses, C.byref(res), err,
                                             len(err)) != 0:
            raise FpError(err.value.decode())
        return _pose(res), float(res.score)
