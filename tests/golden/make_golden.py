"""Generate golden vectors from the reference's own builds (test fixtures).

  python tests/golden/make_golden.py cpu   # needs oracle/_ref/libfpref_cpu.so (build container)
  python tests/golden/make_golden.py gpu [OUT_DIR]  # needs oracle/_ref/libfpref_gpu.so and a CUDA GPU

OUT_DIR (default: this folder) lets a run on a remote GPU machine write the
file where that machine's results are collected; copy it here afterwards.

The reference ships no golden vectors or known-answer tests, so these are
outputs of the reference itself: its CPU functions (src/pipeline_utils.cpp,
src/mesh.cpp) and its CUDA kernels (src/cuda_pipeline.cu,
src/builtin_raster_renderer.cu), compiled unmodified by oracle/Makefile, on
small seeded inputs. The CPU oracle (oracle/fp_oracle.c) is pinned against
them by tests/test_oracle_pins.py, which needs neither the reference nor a GPU.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT / "tests"))
sys.path.insert(0, str(ROOT / "foundation-pose-inference-library_b200" / "python"))


def small_scene(seed: int = 0):
    from oracle_lib import Oracle
    from scene_util import make_scene

    return make_scene(Oracle(), "ellipsoid_small", seed=seed, width=160, height=120)


def make_cpu() -> Path:
    from oracle_lib import RefCpu
    from scene_util import write_obj

    ref = RefCpu()
    s = small_scene(0)
    rng = np.random.default_rng(5)
    depth = s.depth.copy()
    depth[rng.random(depth.shape) < 0.02] = 0.0
    depth[rng.random(depth.shape) < 0.005] = 200.0  # out of range
    mask = s.mask
    k4 = s.k4
    rots = ref.rotation_grid()
    poses = np.stack([np.eye(4, dtype=np.float32)] * 6)
    poses[:, :3, :3] = rots[:6].reshape(6, 3, 3)
    poses[:, :3, 3] = rng.uniform([-0.05, -0.05, 0.5], [0.05, 0.05, 0.9], size=(6, 3))
    poses = poses.reshape(6, 16).astype(np.float32)
    dt = rng.normal(0, 0.4, size=(6, 3)).astype(np.float32)
    dr = rng.normal(0, 1.0, size=(6, 3)).astype(np.float32)
    dr[0] = 0.0
    deltas = np.stack([ref.apply_delta(poses[i], dt[i], dr[i], 0.12) for i in range(6)])
    obj = HERE / "_tmp_mesh.obj"
    write_obj(obj, s.verts, s.faces, s.colors_u8)
    mesh = ref.load_mesh(str(obj))
    obj.unlink()
    out = HERE / "ref_cpu.npz"
    np.savez_compressed(
        out, rotations=rots, depth=depth, mask=mask, k4=k4,
        preprocess=ref.preprocess_depth(depth), xyz=ref.depth_to_xyz(ref.preprocess_depth(depth), k4),
        translation=ref.guess_translation(ref.preprocess_depth(depth), mask, k4),
        poses=poses, boxes=ref.crop_boxes(poses, k4, 0.12), dt=dt, dr=dr, deltas=deltas,
        mesh_in_vertices=s.verts, mesh_in_faces=s.faces, mesh_in_colors=s.colors_u8,
        mesh_vertices=mesh["vertices"], mesh_normals=mesh["normals"], mesh_colors=mesh["colors"],
        mesh_faces=mesh["faces"].astype(np.int32), mesh_center=mesh["center"],
        mesh_diameter=np.float32(mesh["diameter"]))
    return out


def make_gpu(out_dir: Path = HERE) -> Path:
    from oracle_lib import Oracle, RefGpu
    from scene_util import hypotheses

    o = Oracle()
    ref = RefGpu()
    s = small_scene(1)
    rng = np.random.default_rng(7)
    depth = s.depth.copy()
    depth[rng.random(depth.shape) < 0.02] = 0.0
    depth[rng.random(depth.shape) < 0.005] = np.nan
    cfg = o.config(input_width=64, input_height=64)
    rots = o.rotation_grid()
    pre = ref.preprocess(s.rgb, depth, s.mask, s.k4, cfg, rots[:8])
    poses = hypotheses(o, s, 4, seed=3)
    rp = ref.render_pass(s.verts, s.normals, s.colors_u8, s.faces, s.diameter, poses, s.rgb, depth,
                         s.k4, cfg, 0.001)
    dt = rng.normal(0, 0.4, size=(4, 3)).astype(np.float32)
    dr = rng.normal(0, 1.0, size=(4, 3)).astype(np.float32)
    moved = ref.apply_deltas(poses, dt, dr, s.diameter, cfg.rotation_normalizer_rad)
    scores = rng.normal(size=4).astype(np.float32)
    scores[2] = scores.max() + 1.0
    scores[3] = scores[2]
    best_pose, best_score, best_idx = ref.select_best(moved, scores, s.center)
    out_dir.mkdir(parents=True, exist_ok=True)
    out = out_dir / "ref_gpu.npz"
    np.savez_compressed(
        out, rgb=s.rgb, depth=depth, mask=s.mask, k4=s.k4, verts=s.verts, normals=s.normals,
        colors=s.colors_u8, faces=s.faces, diameter=np.float32(s.diameter), center=s.center,
        eroded=pre["eroded"], filtered=pre["filtered"], xyz=pre["xyz"], t0=pre["t0"],
        seeded=pre["seeded"], poses=poses, boxes=rp["boxes"], render_rgb=rp["rgb"],
        render_xyz=rp["xyz"], rast=rp["rast"], net_r=rp["net_r"], net_o=rp["net_o"], dt=dt, dr=dr,
        moved=moved, scores=scores, best_pose=best_pose, best_score=np.float32(best_score),
        best_idx=np.int32(best_idx), crop=np.int32(64))
    return out


if __name__ == "__main__":
    which = sys.argv[1] if len(sys.argv) > 1 else "cpu"
    if which == "cpu":
        print(make_cpu())
    else:
        print(make_gpu(Path(sys.argv[2]) if len(sys.argv) > 2 else HERE))
