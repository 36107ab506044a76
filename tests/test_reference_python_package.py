"""CPU: the reference's own Python package (python/src/foundation_pose_nvidia in
the reference, unchanged) drives this library through FP_LIBRARY.

The Python drop-in surface is not re-implemented here: users keep the
reference's ctypes package and point its loader at libfoundation_pose_nvidia.so
(reference bindings/_loader.py:40-41). These tests import that package from the
reference source tree, so they run where the reference is mounted (the build
container) and skip elsewhere. They need no GPU: binding every symbol, the
RuntimeConfig -> fp_config_t mapping, the struct layouts and the create error
path all stay on the host.
"""
from __future__ import annotations

import ctypes as C
import os
import sys
from pathlib import Path

import pytest

from fp_b200 import capi

ROOT = Path(__file__).resolve().parents[1]
REFERENCE = Path(os.environ.get("FP_REFERENCE_ROOT", "/root/reference"))
REF_PKG = REFERENCE / "python" / "src"
LIB = capi.LIBRARY

pytestmark = pytest.mark.skipif(not (REF_PKG / "foundation_pose_nvidia").is_dir(),
                                reason="reference Python package not mounted")


@pytest.fixture(scope="module")
def fpn(monkeypatch_module):
    monkeypatch_module.setenv("FP_LIBRARY", str(LIB))
    monkeypatch_module.syspath_prepend(str(REF_PKG))
    for name in [m for m in sys.modules if m == "foundation_pose_nvidia" or m.startswith("foundation_pose_nvidia.")]:
        del sys.modules[name]
    import foundation_pose_nvidia

    assert Path(foundation_pose_nvidia.__file__).resolve().is_relative_to(REF_PKG.resolve())
    return foundation_pose_nvidia


@pytest.fixture(scope="module")
def monkeypatch_module():
    mp = pytest.MonkeyPatch()
    yield mp
    mp.undo()


def test_reference_loader_binds_this_library(fpn):
    lib = fpn.load_library(print_build_info=False)  # resolves FP_LIBRARY, declares every fp_* signature
    assert Path(lib.path) == LIB.resolve()
    lib.bind_group_api(3)
    assert "B200" in lib.build_info


def test_reference_structs_have_this_library_layout(fpn):
    from foundation_pose_nvidia.bindings import _ctypes_types as ref

    pairs = [(ref.Config, capi.fp_config_t), (ref.CreateOptions, capi.fp_create_options_t),
             (ref.ImageView, capi.fp_image_view_t), (ref.ReferenceImageView, capi.fp_reference_image_view_t),
             (ref.PoseResult, capi.fp_pose_result_t)]
    for theirs, ours in pairs:
        assert C.sizeof(theirs) == C.sizeof(ours), theirs.__name__
        assert [f[0] for f in theirs._fields_] == [f[0] for f in ours._fields_], theirs.__name__


def test_reference_runtime_config_maps_onto_defaults(fpn):
    lib = fpn.load_library(print_build_info=False)
    rc = fpn.RuntimeConfig(n_hypotheses=42, tensorrt_precision=fpn.Precision.FP16, batch_size=21,
                           capture_cuda_graph=True)
    c = rc.to_ctypes(lib)  # fp_default_config of this library, then the overrides
    assert (c.n_hypotheses, c.tensorrt_precision, c.batch_size, c.capture_cuda_graph) == (42, 2, 21, 1)
    assert (c.n_refine_iters, c.n_track_iters, c.input_width, c.max_image_width) == (5, 2, 160, 1280)
    back = fpn.RuntimeConfig.from_ctypes(c)
    assert back.n_hypotheses == 42 and back.tensorrt_precision == fpn.Precision.FP16
    default = fpn.RuntimeConfig.from_ctypes(lib.default_config())
    assert default.tensorrt_precision == fpn.Precision.TF32 and default.n_hypotheses == 252


def test_reference_estimator_reports_this_library_errors(fpn, tmp_path):
    opts = fpn.EstimatorOptions(cad_path=tmp_path / "missing.obj", refine_model_path=tmp_path / "r.fpw",
                                score_model_path=tmp_path / "s.fpw", engine_cache_dir=tmp_path)
    lib = fpn.load_library(print_build_info=False)
    with pytest.raises(fpn.FoundationPoseError, match="Failed to open OBJ mesh"):
        fpn.Estimator(opts, fpn.RuntimeConfig(), library=lib)
