"""Typed ctypes wrapper around libfoundation_pose_nvidia.so."""
from __future__ import annotations

import ctypes as C
from pathlib import Path

from foundation_pose_nvidia.bindings._ctypes_types import (Config, CreateOptions, ImageView,
                                                          PoseResult, ReferenceImageView)
from foundation_pose_nvidia.bindings._loader import resolve_library_path
from foundation_pose_nvidia.exceptions import FoundationPoseError

_P = C.c_void_p


class FPLibrary:
    """Low-level bindings; `cdll` exposes the raw handle."""

    def __init__(self, path: Path | str | None = None, *, print_build_info: bool = True):
        self.path = resolve_library_path(path)
        self._lib = C.CDLL(str(self.path))
        self._bind_core()
        if print_build_info:
            print(self.build_info)

    @property
    def cdll(self) -> C.CDLL:
        return self._lib

    @property
    def build_info(self) -> str:
        return self._lib.fp_build_info().decode("utf-8")

    def default_config(self) -> Config:
        cfg = Config()
        self._lib.fp_default_config(C.byref(cfg))
        return cfg

    def synchronize(self, err_size: int = 1024) -> None:
        err = C.create_string_buffer(err_size)
        if self._lib.fp_synchronize_device(err, len(err)) != 0:
            raise FoundationPoseError(err.value.decode("utf-8"))

    def bind_group_api(self, object_count: int) -> None:
        lib = self._lib
        masks = C.POINTER(C.c_uint8) * object_count
        sig = {
            "fp_group_create": (_P, [C.POINTER(CreateOptions), C.c_size_t, C.POINTER(Config),
                                     C.c_char_p, C.c_size_t]),
            "fp_group_size": (C.c_size_t, [_P]),
            "fp_group_handle": (_P, [_P, C.c_size_t]),
            "fp_group_prepare": (C.c_int, [_P, C.c_int, C.c_char_p, C.c_size_t]),
            "fp_group_register_frame": (C.c_int, [_P, C.POINTER(ImageView), masks, C.c_int,
                                                  C.c_int, C.POINTER(PoseResult),
                                                  C.POINTER(C.c_int), C.c_char_p, C.c_size_t]),
            "fp_group_track_frame": (C.c_int, [_P, C.POINTER(ImageView), C.POINTER(C.c_int),
                                               C.c_int, C.POINTER(PoseResult),
                                               C.POINTER(C.c_int), C.c_char_p, C.c_size_t]),
            "fp_group_destroy": (None, [_P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(lib, name)
            fn.restype, fn.argtypes = res, args

    def _bind_core(self) -> None:
        sig = {
            "fp_default_config": (None, [C.POINTER(Config)]),
            "fp_create": (_P, [C.POINTER(CreateOptions), C.POINTER(Config), C.c_char_p, C.c_size_t]),
            "fp_create_model_free": (_P, [C.POINTER(ReferenceImageView), C.c_size_t,
                                          C.POINTER(CreateOptions), C.POINTER(Config),
                                          C.c_char_p, C.c_size_t]),
            "fp_prepare": (C.c_int, [_P, C.c_int, C.c_char_p, C.c_size_t]),
            "fp_destroy": (None, [_P]),
            "fp_register_frame": (C.c_int, [_P, C.POINTER(ImageView), C.c_int, C.c_int,
                                            C.POINTER(PoseResult), C.c_char_p, C.c_size_t]),
            "fp_track_frame": (C.c_int, [_P, C.POINTER(ImageView), C.c_int,
                                         C.POINTER(PoseResult), C.c_char_p, C.c_size_t]),
            "fp_register_shard_begin": (C.c_int, [_P, C.POINTER(ImageView), C.c_int, C.c_int, C.c_int,
                                                  C.c_int, _P, _P, C.c_char_p, C.c_size_t]),
            "fp_register_shard_finish": (C.c_int, [_P, _P, _P, C.c_int, C.POINTER(PoseResult),
                                                   C.c_char_p, C.c_size_t]),
            "fp_synchronize_device": (C.c_int, [C.c_char_p, C.c_size_t]),
            "fp_build_info": (C.c_char_p, []),
        }
        for name, (res, args) in sig.items():
            fn = getattr(self._lib, name)
            fn.restype, fn.argtypes = res, args


def load_library(path: Path | str | None = None, *, print_build_info: bool = True) -> FPLibrary:
    return FPLibrary(path, print_build_info=print_build_info)
