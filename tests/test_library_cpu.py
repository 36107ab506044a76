"""CPU: the C-ABI library loads without a GPU, exports every entry point its
headers declare, keeps the reference's struct layouts and defaults, and
reports the reference's errors for invalid calls that never reach CUDA."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

from fp_b200.capi import (Api, fp_config_t as Config, fp_create_options_t as CreateOptions,
                         fp_image_view_t as ImageView, fp_pose_result_t as PoseResult,
                         fp_reference_image_view_t as ReferenceImageView)

ROOT = Path(__file__).resolve().parents[1]
LIB = ROOT / "foundation-pose-inference-library_b200" / "lib" / "libfoundation_pose_nvidia.so"


def declared_symbols() -> set[str]:
    names = set()
    for h in (ROOT / "include").rglob("*.h"):
        text = h.read_text()
        for m in re.finditer(r"FP_API\s+[\w\s\*]+?\b(\w+)\s*\(", text):
            names.add(m.group(1))
    return names


@pytest.fixture(scope="module")
def lib():
    assert LIB.is_file(), "library not built"
    return Api(LIB)


def test_every_declared_symbol_is_exported(lib):
    names = declared_symbols()
    reference_abi = {"fp_default_config", "fp_create", "fp_create_model_free", "fp_prepare",
                     "fp_destroy", "fp_register_frame", "fp_track_frame", "fp_group_create",
                     "fp_group_size", "fp_group_handle", "fp_group_prepare",
                     "fp_group_register_frame", "fp_group_track_frame", "fp_group_destroy",
                     "fp_synchronize_device", "fp_build_info"}
    assert reference_abi <= names
    for n in sorted(names):
        assert hasattr(lib.lib, n), f"{n} declared in include/ but not exported"


def test_struct_layouts_match_reference():
    # reference c_api.h:174-269
    assert C.sizeof(Config) == 56
    assert C.sizeof(CreateOptions) == 96
    assert CreateOptions.mesh_unit_scale.offset == 12
    assert C.sizeof(ImageView) == 40
    assert C.sizeof(ReferenceImageView) == 48
    assert C.sizeof(PoseResult) == 68
    assert Config.batch_size.offset == 52


def test_default_config_matches_reference(lib):
    c = lib.default_config()
    # reference config.hpp:20-67 and c_api.cpp:264-283
    assert (c.n_hypotheses, c.n_refine_iters, c.n_track_iters) == (252, 5, 2)
    assert abs(c.crop_ratio - 1.2) < 1e-6
    assert (c.input_width, c.input_height, c.max_image_width, c.max_image_height) == (160, 160, 1280, 720)
    assert c.capture_cuda_graph == 0 and c.tensorrt_precision == 1 and c.batch_size == 252
    assert (c.model_free_sample_stride, c.model_free_max_vertices) == (4, 250000)
    assert abs(c.model_free_depth_edge_threshold - 0.02) < 1e-7


def test_build_info(lib):
    assert "B200" in lib.build_info


def _err():
    return C.create_string_buffer(512)


def test_error_paths_without_gpu(lib, tmp_path):
    L = lib.lib
    e = _err()
    assert not L.fp_create(None, None, e, len(e))
    assert e.value.decode() == "cad_path is required"
    opts = CreateOptions(str(tmp_path / "missing.obj").encode(), 0, 1.0, None, None, None)
    assert not L.fp_create(C.byref(opts), None, e, len(e))
    assert "Failed to open OBJ mesh" in e.value.decode()
    opts = CreateOptions(str(tmp_path / "mesh.stl").encode(), 0, 1.0, None, None, None)
    assert not L.fp_create(C.byref(opts), None, e, len(e))
    assert "Unsupported mesh extension" in e.value.decode()
    assert not L.fp_create_model_free(None, 0, None, None, e, len(e))
    assert "At least one model-free reference image is required" in e.value.decode()
    assert L.fp_prepare(None, 1, e, len(e)) == 1 and e.value.decode() == "Invalid handle"
    res = PoseResult()
    assert L.fp_register_frame(None, None, -1, -1, C.byref(res), e, len(e)) == 1
    assert e.value.decode() == "Invalid handle or image"
    assert L.fp_track_frame(None, None, -1, C.byref(res), e, len(e)) == 1
    assert not L.fp_group_create(None, 0, None, e, len(e))
    assert e.value.decode() == "At least one object is required"
    assert L.fp_group_size(None) == 0
    assert not L.fp_group_handle(None, 0)
    assert L.fp_group_prepare(None, 1, e, len(e)) == 1 and e.value.decode() == "Invalid group"
    L.fp_destroy(None)
    L.fp_group_destroy(None)
    # Error strings are truncated to the buffer and NUL-terminated.
    small = C.create_string_buffer(6)
    assert not L.fp_create(None, None, small, len(small))
    assert small.value.decode() == "cad_p"


def test_fpk_param_defaults():
    from fp_b200.kernels import FpkLibrary

    p = FpkLibrary(LIB).default_params()
    assert p.erosion_radius == 2 and p.bilateral_radius == 2
    assert abs(p.depth_min - 0.001) < 1e-9 and abs(p.rotation_normalizer_rad - 0.34906585) < 1e-7
    assert abs(p.ambient_weight - 0.8) < 1e-7 and abs(p.diffuse_weight - 0.5) < 1e-7


def test_cta_pair_switch_round_trip():
    """fpk_gemm_set_cta_pairs returns the previous setting (pairs on by
    default) and touches no device state, so it is callable without a GPU."""
    from fp_b200.kernels import FpkLibrary

    fpk = FpkLibrary(LIB)
    first = fpk.lib.fpk_gemm_set_cta_pairs(0)
    try:
        assert first == 1
        assert fpk.lib.fpk_gemm_set_cta_pairs(0) == 0
        assert fpk.lib.fpk_gemm_set_cta_pairs(7) == 0  # any non-zero value enables
        assert fpk.lib.fpk_gemm_set_cta_pairs(1) == 1
    finally:
        fpk.lib.fpk_gemm_set_cta_pairs(first)
