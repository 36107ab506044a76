"""Model-free objects on the GPU.

The mesh that fp_create_model_free builds from reference RGB-D views
(fpk_model_free_mesh, built on the GPU) against the reference's own host
reconstruction (src/foundation_pose.cpp:91-182, compiled unmodified into
oracle/_ref/libfpref_full.so): vertices, colours, normals and faces
bit-identical, for close and distant views and sampling strides from 1 to 16
(a small vertex budget widens the stride). Then the whole
model-free flow -- create from 16 views on a Fibonacci sphere at 0.7 m,
register, track a random walk -- through this library and through the
reference's own fp_create_model_free / fp_register_frame / fp_track_frame
(its kernels, torch fp32 networks in place of TensorRT): poses within 1 mm /
0.1 deg at every step.
"""
from __future__ import annotations

import ctypes as C
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import reflib_util  # noqa: E402
from fp_b200 import capi  # noqa: E402
from fp_b200 import synthetic as syn  # noqa: E402
from fp_b200.weights import make_default_packs, read_pack  # noqa: E402
from scene_util import model_free_views, render_query  # noqa: E402

pytestmark = pytest.mark.gpu
TF32 = 1


def ours_mesh(api, views, K, c2ws, cfg):
    refs = [capi.reference_view(r, d, m, K, c) for (r, d, m), c in zip(views, c2ws)]
    arr = (capi.fp_reference_image_view_t * len(refs))(*refs)
    fn = api.lib.fpk_model_free_mesh
    fn.restype = C.c_int
    fn.argtypes = [C.POINTER(capi.fp_reference_image_view_t), C.c_size_t, C.POINTER(capi.fp_config_t),
                   C.POINTER(C.c_int), C.POINTER(C.c_int), C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
    nv, nf = C.c_int(), C.c_int()
    assert fn(arr, len(refs), C.byref(cfg), C.byref(nv), C.byref(nf), None, None, None, None) == 0
    v = np.zeros((nv.value, 3), np.float32)
    c = np.zeros((nv.value, 3), np.uint8)
    n = np.zeros((nv.value, 3), np.float32)
    f = np.zeros((nf.value, 3), np.int32)
    assert fn(arr, len(refs), C.byref(cfg), C.byref(nv), C.byref(nf), v.ctypes.data, c.ctypes.data, n.ctypes.data,
              f.ctypes.data) == 0
    return v, c, n, f


@pytest.fixture(scope="module")
def reflib():
    if not reflib_util.REF_FULL_SO.is_file():
        pytest.skip("reference library build (oracle/_ref/libfpref_full.so) not present")
    return reflib_util.load()


@pytest.mark.parametrize("n_views,distance,max_vertices,stride", [(6, 0.7, 250000, 4), (3, 0.12, 9000, 2),
                                                                  (2, 0.5, 250000, 1)])
def test_model_free_mesh_matches_reference(oracle, reflib, n_views, distance, max_vertices, stride):
    parts, K, views, c2ws = model_free_views(oracle, n_views, seed=n_views, distance=distance)
    api = capi.Api()
    cfg = api.default_config(model_free_max_vertices=max_vertices, model_free_sample_stride=stride)
    v, c, n, f = ours_mesh(api, views, K, c2ws, cfg)
    rv, rc, rn, rf = reflib_util.reconstruct(reflib["lib"], views, K, c2ws, stride, max_vertices,
                                             cfg.model_free_depth_edge_threshold)
    print(f"model-free mesh: {len(v)} vertices, {len(f)} faces (reference {len(rv)}, {len(rf)})")
    assert len(v) >= 4 and len(f) > 0
    np.testing.assert_array_equal(v, rv)
    np.testing.assert_array_equal(c, rc)
    np.testing.assert_array_equal(f, rf)
    np.testing.assert_array_equal(n, rn)


def test_model_free_rejects_empty_views(oracle):
    parts, K, views, c2ws = model_free_views(oracle, 1, seed=0)
    rgb, depth, mask = views[0]
    api = capi.Api()
    opts = api.options(None, "r.fpw", "s.fpw")
    ref = capi.reference_view(rgb, depth, np.zeros_like(mask), K, c2ws[0])
    with pytest.raises(capi.FpError, match="too little geometry"):
        api.create_model_free([ref], opts, api.default_config())


def rot_err_deg(a, b):
    r = a[:3, :3] @ b[:3, :3].T
    return math.degrees(math.acos(max(-1.0, min(1.0, (np.trace(r) - 1) / 2))))


def test_model_free_register_track_matches_reference_library(oracle, tmp_path):
    """configs[3] at test size: 16 views, TF32, a register refined from the
    first rotation of the grid (one hypothesis: with random-init weights the
    ScoreNet scores of different hypotheses tie to within rounding, so a
    many-hypothesis arg-max would compare tie-breaks rather than poses), 2
    refinement passes, then 3 tracked frames of a seeded random walk."""
    if not reflib_util.REF_FULL_SO.is_file():
        pytest.skip("reference library build not present")
    refine, score = make_default_packs(tmp_path, seed=11)
    ref = reflib_util.load(read_pack(refine)[1], read_pack(score)[1])
    rl = ref["lib"]
    parts, K, views, c2ws = model_free_views(oracle, 16, seed=4)
    api = capi.Api()
    cfg = api.default_config(n_hypotheses=42, batch_size=42, tensorrt_precision=TF32, max_image_width=640,
                             max_image_height=480)
    opts = api.options(None, refine, score, 0, tmp_path)
    refs = [capi.reference_view(r, d, m, K, c) for (r, d, m), c in zip(views, c2ws)]
    h = api.create_model_free(refs, opts, cfg)
    err = C.create_string_buffer(4096)
    arr = (capi.fp_reference_image_view_t * len(refs))(*refs)
    rh = rl.fp_create_model_free(arr, len(refs), C.byref(opts), C.byref(cfg), err, len(err))
    assert rh, err.value.decode()
    rng = np.random.default_rng(5)
    pose = syn.random_pose(rng, dist=(0.6, 0.8), lateral=0.03)
    try:
        for step in range(4):
            rgb, depth, mask = render_query(oracle, parts, pose, K, seed=step)
            view = capi.image_view(rgb, depth, K, mask if step == 0 else None)
            res = capi.fp_pose_result_t()
            if step == 0:
                ours, score_ours = api.register(h, view, 2, 1)
                assert rl.fp_register_frame(rh, C.byref(view), 2, 1, C.byref(res), err, len(err)) == 0, \
                    err.value.decode()
            else:
                ours, score_ours = api.track(h, view, 2)
                assert rl.fp_track_frame(rh, C.byref(view), 2, C.byref(res), err, len(err)) == 0, err.value.decode()
            theirs = np.array(res.pose_row_major, np.float32).reshape(4, 4)
            t_err = float(np.linalg.norm(ours[:3, 3] - theirs[:3, 3]) * 1000.0)
            r_err = rot_err_deg(ours, theirs)
            print(f"model-free step {step}: dt={t_err:.4f} mm dR={r_err:.4f} deg, score {score_ours:.5f} vs "
                  f"{res.score:.5f}")
            if step == 0:
                assert abs(score_ours - res.score) <= 1e-3 * max(1.0, abs(res.score))
            assert t_err <= 1.0 and r_err <= 0.1
            pose = syn.random_walk(rng, pose)
    finally:
        api.destroy(h)
        rl.fp_destroy(rh)
