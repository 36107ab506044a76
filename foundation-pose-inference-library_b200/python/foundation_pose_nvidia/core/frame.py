"""RgbdFrame: host (numpy) or device (__cuda_array_interface__) frame buffers
laid out as fp_image_view_t expects (reference core/frame.py:68-138)."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Any

import numpy as np

from foundation_pose_nvidia.bindings._ctypes_types import ImageView


def _cai(buf: Any) -> dict | None:
    return getattr(buf, "__cuda_array_interface__", None)


def _check_device(buf: Any, typestrs: tuple[str, ...], ndim: int, name: str) -> Any:
    cai = buf.__cuda_array_interface__
    ts = cai.get("typestr")
    if ts not in typestrs:
        raise ValueError(f"{name}: GPU buffer has typestr {ts!r}, expected one of {typestrs}; "
                         "convert before passing (torch: .to(torch.float32) / .to(torch.uint8)).")
    shape = tuple(cai["shape"])
    if len(shape) != ndim:
        raise ValueError(f"{name}: GPU buffer must be {ndim}-D, got shape {shape}.")
    strides = cai.get("strides")
    if strides is not None:
        item = int(ts[2:])
        expect, acc = [], item
        for s in reversed(shape):
            expect.append(acc)
            acc *= s
        if tuple(strides) != tuple(reversed(expect)):
            raise ValueError(f"{name}: GPU buffer must be C-contiguous (torch: .contiguous()).")
    return buf


def _ptr(buf: Any, ctype):
    cai = _cai(buf)
    if cai is not None:
        return C.cast(C.c_void_p(cai["data"][0]), C.POINTER(ctype))
    return buf.ctypes.data_as(C.POINTER(ctype))


@dataclass
class RgbdFrame:
    rgb: Any
    depth_m: Any
    intrinsics: np.ndarray
    mask: Any | None = None

    def __post_init__(self) -> None:
        if _cai(self.rgb) is not None:
            _check_device(self.rgb, ("|u1",), 3, "rgb")
        else:
            self.rgb = np.ascontiguousarray(self.rgb, dtype=np.uint8)
        if _cai(self.depth_m) is not None:
            _check_device(self.depth_m, ("<f4", "=f4"), 2, "depth_m")
        else:
            self.depth_m = np.ascontiguousarray(self.depth_m, dtype=np.float32)
        if _cai(self.intrinsics) is not None:
            raise ValueError("intrinsics must be host memory (numpy), not a GPU array")
        self.intrinsics = np.ascontiguousarray(np.asarray(self.intrinsics).reshape(3, 3), np.float32)
        if self.mask is not None:
            if _cai(self.mask) is not None:
                _check_device(self.mask, ("|u1",), 2, "mask")
            else:
                self.mask = np.ascontiguousarray(self.mask, dtype=np.uint8)

    @property
    def width(self) -> int:
        return int(self.rgb.shape[1])

    @property
    def height(self) -> int:
        return int(self.rgb.shape[0])

    def to_image_view(self, *, with_mask: bool) -> ImageView:
        if with_mask and self.mask is None:
            raise ValueError("register requires a mask on RgbdFrame")
        mask = self.mask if with_mask else None
        k = np.ascontiguousarray(self.intrinsics.reshape(9), np.float32)
        view = ImageView(self.width, self.height, _ptr(self.rgb, C.c_uint8),
                         _ptr(self.depth_m, C.c_float),
                         _ptr(mask, C.c_uint8) if mask is not None else C.POINTER(C.c_uint8)(),
                         k.ctypes.data_as(C.POINTER(C.c_float)))
        view._keepalive = (self.rgb, self.depth_m, mask, k)  # ctypes keeps only addresses
        return view
