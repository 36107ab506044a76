"""ctypes bindings for the fpk_* kernel-level C ABI (include/fpk.h).

Device buffers are passed as integer addresses (e.g. ``tensor.data_ptr()``);
streams as integer ``cudaStream_t`` handles (0 = legacy default stream).
Every wrapper raises :class:`FpkError` with the library's message on failure.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PKG = Path(__file__).resolve().parents[2]
LIB_PATH = PKG / "lib" / "libfoundation_pose_nvidia.so"

FPK_DTYPE_F32 = 0
FPK_DTYPE_F16 = 1
FPK_DTYPE_BF16 = 2
FPK_DTYPE_F32_EXACT = 3  # fp32 kept exact (strict-FP32 networks)
FPK_STATS_INTS = 8 + 65536


class FpkError(RuntimeError):
    pass


class Params(C.Structure):
    _fields_ = [
        ("depth_min", C.c_float), ("depth_max", C.c_float),
        ("erosion_radius", C.c_int), ("bilateral_radius", C.c_int),
        ("depth_diff_threshold", C.c_float), ("erosion_ratio_threshold", C.c_float),
        ("bilateral_sigma_d", C.c_float), ("bilateral_sigma_r", C.c_float),
        ("crop_ratio", C.c_float),
        ("input_width", C.c_int), ("input_height", C.c_int),
        ("rotation_normalizer_rad", C.c_float), ("znear", C.c_float), ("zfar", C.c_float),
        ("ambient_weight", C.c_float), ("diffuse_weight", C.c_float),
    ]


class Intrinsics(C.Structure):
    _fields_ = [("fx", C.c_float), ("fy", C.c_float), ("cx", C.c_float), ("cy", C.c_float)]


class Mesh(C.Structure):
    _fields_ = [
        ("vertices", C.c_void_p), ("normals", C.c_void_p), ("colors", C.c_void_p),
        ("uvs", C.c_void_p), ("texture", C.c_void_p), ("faces", C.c_void_p),
        ("n_vertices", C.c_int), ("n_faces", C.c_int),
        ("texture_width", C.c_int), ("texture_height", C.c_int),
    ]


_P = C.c_void_p
_SIGS = {
    "fpk_last_error": (C.c_char_p, []),
    "fpk_default_params": (None, [C.POINTER(Params)]),
    "fpk_preprocess": (C.c_int, [_P, _P, C.c_int, C.c_int, Intrinsics, C.POINTER(Params),
                                 _P, _P, _P, _P, _P]),
    "fpk_seed_poses": (C.c_int, [_P, _P, C.c_int, Intrinsics, C.POINTER(Params), _P, _P, _P]),
    "fpk_crop_boxes": (C.c_int, [_P, C.c_int, Intrinsics, C.c_float, C.POINTER(Params), _P, _P]),
    "fpk_render_workspace_bytes": (C.c_size_t, [C.c_int, C.c_int, C.POINTER(Params)]),
    "fpk_render": (C.c_int, [C.POINTER(Mesh), _P, _P, C.c_int, Intrinsics, C.POINTER(Params),
                             _P, _P, _P, _P, C.c_size_t, _P]),
    "fpk_pack": (C.c_int, [_P, _P, C.c_int, C.c_int, Intrinsics, C.POINTER(Params), _P, _P, _P,
                           _P, C.c_int, C.c_float, C.c_float, _P, _P, _P]),
    "fpk_render_pack": (C.c_int, [C.POINTER(Mesh), _P, C.c_int, _P, _P, C.c_int, C.c_int,
                                  Intrinsics, C.POINTER(Params), C.c_float, C.c_float, C.c_int,
                                  _P, C.c_longlong, _P, _P, C.c_size_t, _P]),
    "fpk_apply_deltas": (C.c_int, [_P, _P, _P, C.c_int, C.c_float, C.POINTER(Params), _P]),
    "fpk_select_best": (C.c_int, [_P, _P, C.c_int, C.POINTER(C.c_float), _P, _P]),
    "fpk_gemm": (C.c_int, [_P, _P]),
    "fpk_gemm_set_cta_pairs": (C.c_int, [C.c_int]),
    "fpk_gemm_set_tma_store": (C.c_int, [C.c_int]),
    "fpk_gemm_test_withhold_loads": (C.c_int, [C.c_int]),
    "fpk_attention": (C.c_int, [_P, C.c_longlong, C.c_int, C.c_int, C.c_int, C.c_int, _P, C.c_longlong,
                                C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _P, _P]),
    "fpk_net_create": (C.c_void_p, [C.c_char_p, C.c_char_p, C.c_int, C.c_int]),
    "fpk_net_destroy": (None, [_P]),
    "fpk_net_refine": (C.c_int, [_P, _P, _P, C.c_int, _P, _P, _P]),
    "fpk_net_score": (C.c_int, [_P, _P, _P, C.c_int, _P, _P]),
    "fpk_net_error": (C.c_int, [_P, C.POINTER(C.c_int)]),
}


def exported_symbols() -> list[str]:
    return list(_SIGS)


class FpkLibrary:
    def __init__(self, path: str | os.PathLike | None = None):
        self.path = Path(path) if path else LIB_PATH
        if not self.path.is_file():
            raise FpkError(f"{self.path} is not built (run foundation-pose-inference-library_b200/build.py)")
        self.lib = C.CDLL(str(self.path))
        for name, (res, args) in _SIGS.items():
            fn = getattr(self.lib, name)
            fn.restype = res
            fn.argtypes = args

    def _check(self, rc: int, what: str) -> None:
        if rc != 0:
            raise FpkError(f"{what}: {self.lib.fpk_last_error().decode()}")

    def default_params(self) -> Params:
        p = Params()
        self.lib.fpk_default_params(C.byref(p))
        return p

    def preprocess(self, depth_raw, mask, width, height, k, params, depth_filtered, eroded=0,
                   xyz=0, stats=0, stream=0):
        self._check(self.lib.fpk_preprocess(depth_raw, mask or None, width, height, k,
                                            C.byref(params), depth_filtered, eroded or None,
                                            xyz or None, stats or None, stream or None),
                    "fpk_preprocess")

    def seed_poses(self, stats, rotations, n, k, params, t0, poses, stream=0):
        self._check(self.lib.fpk_seed_poses(stats, rotations, n, k, C.byref(params), t0 or None,
                                            poses, stream or None), "fpk_seed_poses")

    def crop_boxes(self, poses, n, k, diameter, params, boxes, stream=0):
        self._check(self.lib.fpk_crop_boxes(poses, n, k, diameter, C.byref(params), boxes,
                                            stream or None), "fpk_crop_boxes")

    def render_workspace_bytes(self, n, n_vertices, params) -> int:
        return int(self.lib.fpk_render_workspace_bytes(n, n_vertices, C.byref(params)))

    def render(self, mesh, poses, boxes, n, k, params, out_rgb, out_xyz, tri_ids=0, stream=0,
               workspace=0, workspace_bytes=0):
        """workspace 0: the library allocates it stream-ordered for the call."""
        self._check(self.lib.fpk_render(C.byref(mesh), poses, boxes, n, k, C.byref(params),
                                        out_rgb, out_xyz, tri_ids or None, workspace or None,
                                        workspace_bytes, stream or None),
                    "fpk_render")

    def pack(self, rgb, depth_filtered, width, height, k, params, rend_rgb, rend_xyz, poses,
             boxes, n, diameter, invalid_threshold, net_r, net_o, stream=0):
        self._check(self.lib.fpk_pack(rgb, depth_filtered, width, height, k, C.byref(params),
                                      rend_rgb, rend_xyz, poses, boxes, n, diameter,
                                      invalid_threshold, net_r, net_o, stream or None),
                    "fpk_pack")

    def render_pack(self, mesh, poses, n, rgb, depth_filtered, width, height, k, params,
                    diameter, invalid_threshold, dtype, net, plane_stride, boxes, stream=0,
                    workspace=0, workspace_bytes=0):
        self._check(self.lib.fpk_render_pack(C.byref(mesh), poses, n, rgb, depth_filtered, width,
                                             height, k, C.byref(params), diameter,
                                             invalid_threshold, dtype, net, plane_stride,
                                             boxes or None, workspace or None, workspace_bytes,
                                             stream or None), "fpk_render_pack")

    def apply_deltas(self, poses, dt, dr, n, diameter, params, stream=0):
        self._check(self.lib.fpk_apply_deltas(poses, dt, dr, n, diameter, C.byref(params),
                                              stream or None), "fpk_apply_deltas")

    def select_best(self, poses, scores, n, center3, result, stream=0):
        c = (C.c_float * 3)(*[float(v) for v in center3])
        self._check(self.lib.fpk_select_best(poses, scores, n, c, result, stream or None),
                    "fpk_select_best")


FPK_DST_SAME = 0
FPK_DST_S2D = 1
FPK_DST_CONCAT = 2
FPK_DST_TOKENS = 3


class GemmDesc(C.Structure):
    _fields_ = [
        ("a", C.c_void_p), ("a_plane_stride", C.c_longlong), ("rows", C.c_int), ("cin", C.c_int),
        ("taps", C.c_int), ("tap_off", C.c_int * 16), ("w", C.c_void_p), ("cout", C.c_int),
        ("bias", C.c_void_p), ("residual", C.c_void_p), ("res_plane_stride", C.c_longlong),
        ("relu", C.c_int), ("dst", C.c_void_p), ("dst_plane_stride", C.c_longlong),
        ("dst_mode", C.c_int), ("img_rows", C.c_int), ("grid_w", C.c_int), ("valid_h", C.c_int),
        ("valid_w", C.c_int), ("dst_img_rows", C.c_int), ("dst_grid_w", C.c_int),
        ("img_mod", C.c_int), ("ch_step", C.c_int), ("pos", C.c_void_p), ("dtype", C.c_int),
        ("error_flag", C.c_void_p), ("splitk_ws", C.c_void_p), ("splitk_ws_bytes", C.c_longlong),
    ]


def _bind_gemm(lib) -> None:
    lib.fpk_gemm.restype = C.c_int
    lib.fpk_gemm.argtypes = [C.POINTER(GemmDesc), C.c_void_p]


def gemm(fl: "FpkLibrary", desc: GemmDesc, stream=0) -> None:
    if not getattr(fl, "_gemm_bound", False):
        _bind_gemm(fl.lib)
        fl._gemm_bound = True
    fl._check(fl.lib.fpk_gemm(C.byref(desc), stream or None), "fpk_gemm")


def attention(fl: FpkLibrary, qkv: int, qkv_plane_stride: int, qkv_layer_channels: int, q_channel: int,
              k_channel: int, v_channel: int, out: int, out_plane_stride: int, out_layer_channels: int,
              layers: int, heads: int, seq_len: int, n_seq: int, dtype: int, error_flag: int,
              stream: int | None = None) -> None:
    """fpk_attention: multi-head self-attention over planar activations (see include/fpk.h)."""
    fl._check(fl.lib.fpk_attention(qkv, qkv_plane_stride, qkv_layer_channels, q_channel, k_channel, v_channel,
                                   out, out_plane_stride, out_layer_channels, layers, heads, seq_len, n_seq,
                                   dtype, error_flag, stream or None), "fpk_attention")


class Networks:
    """RefineNet + ScoreNet handle (fpk_net_*); precision 2 = FP16, 3 = BF16."""

    def __init__(self, fl: FpkLibrary, refine_pack, score_pack, precision: int, max_batch: int):
        self.fl = fl
        self.h = fl.lib.fpk_net_create(str(refine_pack).encode(), str(score_pack).encode(),
                                       int(precision), int(max_batch))
        if not self.h:
            raise FpkError(f"fpk_net_create: {fl.lib.fpk_last_error().decode()}")

    def refine(self, rendered, observed, n, trans, rot, stream=0):
        self.fl._check(self.fl.lib.fpk_net_refine(self.h, rendered, observed, n, trans, rot,
                                                  stream or None), "fpk_net_refine")

    def score(self, rendered, observed, n, scores, stream=0):
        self.fl._check(self.fl.lib.fpk_net_score(self.h, rendered, observed, n, scores,
                                                 stream or None), "fpk_net_score")

    def error_flag(self) -> int:
        v = C.c_int(0)
        self.fl._check(self.fl.lib.fpk_net_error(self.h, C.byref(v)), "fpk_net_error")
        return v.value

    def close(self):
        if self.h:
            self.fl.lib.fpk_net_destroy(self.h)
            self.h = None

    __del__ = close
