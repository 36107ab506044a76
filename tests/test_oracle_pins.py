"""CPU: the oracle (oracle/fp_oracle.c) pinned against golden vectors produced
by the reference's own builds (tests/golden/make_golden.py): its CPU functions
(ref_cpu.npz) and its CUDA kernels (ref_gpu.npz, generated on the B200).
The reference ships no golden vectors of its own, so these are the pins."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle_lib import REF_CPU_SO, RefCpu

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def cpu():
    return np.load(GOLDEN / "ref_cpu.npz")


@pytest.fixture(scope="module")
def gpu():
    p = GOLDEN / "ref_gpu.npz"
    if not p.is_file():
        pytest.skip("reference CUDA golden vectors not generated yet")
    return np.load(p)


def test_rotation_grid_bit_exact(oracle, cpu):
    rots = oracle.rotation_grid()
    assert rots.shape == (252, 9)
    np.testing.assert_array_equal(rots, cpu["rotations"])
    # every rotation is orthonormal with det +1
    r = rots.reshape(-1, 3, 3).astype(np.float64)
    np.testing.assert_allclose(r @ r.transpose(0, 2, 1), np.broadcast_to(np.eye(3), r.shape), atol=1e-5)
    np.testing.assert_allclose(np.linalg.det(r), 1.0, atol=1e-5)


def test_cpu_preprocess_and_xyz_bit_exact(oracle, cpu):
    cfg = oracle.config()
    out = oracle.preprocess_cpu(cpu["depth"], cfg)
    np.testing.assert_array_equal(out, cpu["preprocess"])
    np.testing.assert_array_equal(oracle.depth_to_xyz(out, cpu["k4"], cfg), cpu["xyz"])


def test_cpu_translation_bit_exact(oracle, cpu):
    t = oracle.guess_translation_cpu(cpu["preprocess"], cpu["mask"], cpu["k4"], oracle.config())
    np.testing.assert_array_equal(t, cpu["translation"])
    assert t[2] > 0


def test_crop_boxes_match_cpu_reference(oracle, cpu):
    # Oracle follows the GPU kernel (reciprocal-multiply projection); the CPU
    # twin divides. Both round to the same integer box here.
    b = oracle.crop_boxes(cpu["poses"], cpu["k4"], 0.12, oracle.config())
    np.testing.assert_array_equal(b, cpu["boxes"])


def test_pose_delta_matches_cpu_reference(oracle, cpu):
    # Same rotation (exp map, transposed) and translation update; the CPU twin
    # builds exp() from the skew matrix instead of the expanded Rodrigues form.
    got = oracle.apply_deltas(cpu["poses"], cpu["dt"], cpu["dr"], 0.12, oracle.config())
    np.testing.assert_allclose(got, cpu["deltas"], rtol=1e-5, atol=2e-7)


def test_mesh_centre_diameter_normals(oracle, cpu):
    c, d, centered = oracle.mesh_center_diameter(cpu["mesh_in_vertices"])
    np.testing.assert_array_equal(c, cpu["mesh_center"])
    assert np.float32(d) == cpu["mesh_diameter"]
    np.testing.assert_array_equal(centered, cpu["mesh_vertices"])
    n = oracle.vertex_normals(centered, cpu["mesh_faces"])
    np.testing.assert_array_equal(n, cpu["mesh_normals"])


def test_oracle_erosion_border_semantics_differ(oracle):
    """The GPU erosion counts in-bounds neighbours only; the CPU twin counts
    out-of-image neighbours as bad with a fixed 25-tap denominator (reference
    pipeline_utils.cpp:35-64 vs cuda_pipeline.cu:103-119). A corner pixel with
    5 of its 8 in-image neighbours invalid is kept by the GPU (5/9 <= 0.8) and
    eroded by the CPU twin ((16 + 5)/25 > 0.8); the bilateral pass then refills
    it from its neighbours only on the CPU side."""
    d = np.full((8, 8), 0.5, np.float32)
    d[0, 0] = 0.5005
    for y, x in ((0, 1), (0, 2), (1, 0), (1, 1), (2, 0)):
        d[y, x] = 0.0
    cfg = oracle.config()
    assert oracle.erode(d, cfg)[0, 0] == np.float32(0.5005)
    gpu_sem = oracle.bilateral(oracle.erode(d, cfg), cfg)[0, 0]
    cpu_sem = oracle.preprocess_cpu(d, cfg)[0, 0]
    assert cpu_sem == np.float32(0.5) and gpu_sem > np.float32(0.5)


def test_gpu_reference_preprocess(oracle, gpu):
    cfg = oracle.config()
    ero = oracle.erode(gpu["depth"], cfg)
    np.testing.assert_array_equal(ero, gpu["eroded"])
    fil = oracle.bilateral(ero, cfg)
    np.testing.assert_allclose(fil, gpu["filtered"], rtol=2e-6, atol=0)
    np.testing.assert_allclose(oracle.depth_to_xyz(gpu["filtered"], gpu["k4"], cfg), gpu["xyz"],
                               rtol=2e-6, atol=1e-9)
    t = oracle.initial_translation(gpu["filtered"], gpu["mask"], gpu["k4"], cfg)
    np.testing.assert_allclose(t, gpu["t0"], rtol=1e-6)


def test_gpu_reference_render_and_pack(oracle, gpu):
    crop = int(gpu["crop"])
    cfg = oracle.config(input_width=crop, input_height=crop)
    boxes = oracle.crop_boxes(gpu["poses"], gpu["k4"], float(gpu["diameter"]), cfg)
    np.testing.assert_array_equal(boxes, gpu["boxes"])
    colors = (gpu["colors"].astype(np.float32) / np.float32(255.0)).astype(np.float32)
    rgb, xyz, rast = oracle.render(gpu["verts"], gpu["normals"], colors, gpu["faces"], gpu["poses"],
                                   boxes, gpu["k4"], cfg)
    tri, ref_tri = rast[..., 3].astype(np.int32), gpu["rast"][..., 3].astype(np.int32)
    assert (ref_tri > 0).mean() > 0.05
    # The CPU oracle evaluates the edge functions without FMA contraction:
    # pixels on triangle edges may resolve to the neighbour.
    assert (tri != ref_tri).mean() <= 2e-3
    same = np.flip(tri == ref_tri, axis=1)
    np.testing.assert_allclose(xyz[same], gpu["render_xyz"][same], rtol=1e-4, atol=1e-6)
    err = np.abs(rgb[same] - gpu["render_rgb"][same])
    assert np.mean(err > 1e-4) <= 1e-3 and err.max() <= 1e-2
    xyz_map = oracle.depth_to_xyz(gpu["filtered"], gpu["k4"], cfg)
    r, o = oracle.pack(gpu["rgb"], xyz_map, gpu["render_rgb"], gpu["render_xyz"], gpu["poses"], boxes,
                       float(gpu["diameter"]), 0.001, cfg)
    np.testing.assert_allclose(o, gpu["net_o"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(r, gpu["net_r"], rtol=1e-5, atol=1e-6)


def test_gpu_reference_deltas_and_select(oracle, gpu):
    cfg = oracle.config()
    moved = oracle.apply_deltas(gpu["poses"], gpu["dt"], gpu["dr"], float(gpu["diameter"]), cfg)
    np.testing.assert_allclose(moved, gpu["moved"], rtol=1e-5, atol=2e-7)
    pose, score, idx = oracle.select_best(gpu["moved"], gpu["scores"], gpu["center"])
    assert idx == int(gpu["best_idx"]) == 2  # first of two equal maxima
    np.testing.assert_allclose(pose, gpu["best_pose"], rtol=1e-6, atol=1e-7)
    assert score == float(gpu["best_score"])


@pytest.mark.skipif(not REF_CPU_SO.is_file(), reason="reference CPU build not present")
def test_live_reference_cpu_rotation_grid(oracle):
    np.testing.assert_array_equal(oracle.rotation_grid(), RefCpu().rotation_grid())
