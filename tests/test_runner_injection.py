"""The C++ seam with a caller's IInferenceRunner (reference
include/foundation_pose_nvidia/foundation_pose.hpp:27-31, inference_runner.hpp:12-30).

runner_injection/inject_runner.cpp is compiled with g++ against the public
headers and linked to libfoundation_pose_nvidia.so, so this also checks that
the library exports its C++ API (FoundationPose, BuiltinRasterRenderer,
TensorRtRunner, loadMesh / preprocessMesh, FoundationPoseError). CPU: the
program builds and links. GPU: an estimator given a counting runner that
forwards to TensorRtRunner, plus BuiltinRasterRenderer, goes through the NCHW
fp32 seam (one refine call per pass, one score call, every hypothesis) and
registers and tracks to the pose of the built-in fused estimator."""
from __future__ import annotations

import json
import os
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
LIB_DIR = ROOT / "foundation-pose-inference-library_b200" / "lib"
SRC = Path(__file__).resolve().parent / "runner_injection" / "inject_runner.cpp"
CUDA_INC = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "include"


def build(out_dir: Path) -> Path:
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    if not (LIB_DIR / "libfoundation_pose_nvidia.so").exists():
        pytest.skip("main library not built")
    exe = out_dir / "inject_runner"
    cmd = ["g++", "-std=c++20", "-O1", f"-I{ROOT / 'include'}", f"-I{CUDA_INC}", str(SRC), "-o", str(exe),
           f"-L{LIB_DIR}", "-l:libfoundation_pose_nvidia.so", f"-Wl,-rpath,{LIB_DIR}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_cpp_api_links(tmp_path):
    exe = build(tmp_path)
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 2 and "usage" in r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("precision", [2, 1])  # FP16, TF32
def test_injected_runner_matches_builtin(tmp_path, oracle, precision):
    from fp_b200.weights import make_default_packs
    from scene_util import make_scene, write_obj

    exe = build(tmp_path)
    refine, score = make_default_packs(tmp_path, seed=2)
    scene = make_scene(oracle, "ellipsoid", seed=8)
    obj = tmp_path / "object.obj"
    write_obj(obj, scene.verts, scene.faces, scene.colors_u8)
    frame = tmp_path / "frame.bin"
    h, w = scene.depth.shape
    with open(frame, "wb") as f:
        f.write(np.array([w, h], np.int32).tobytes())
        f.write(np.asarray(scene.K, np.float32).tobytes())
        f.write(np.ascontiguousarray(scene.rgb).tobytes())
        f.write(np.ascontiguousarray(scene.depth, np.float32).tobytes())
        f.write(np.ascontiguousarray(scene.mask).tobytes())
    n_hyp, n_refine = 42, 3
    r = subprocess.run([str(exe), str(obj), str(refine), str(score), str(frame), str(n_hyp), str(n_refine),
                        str(precision)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert out["prepares"] == 1
    assert out["refines"] == n_refine + 2 and out["refine_items"] == n_hyp * n_refine + 2  # + 2 track passes at B=1
    assert out["scores"] == 1 and out["score_items"] == n_hyp
    for key in ("", "_track"):
        a = np.array(out["injected" + key]).reshape(4, 4)
        b = np.array(out["builtin" + key]).reshape(4, 4)
        assert np.abs(a - b).max() <= 1e-5, (key, a, b)
    assert abs(out["injected_score"] - out["builtin_score"]) <= 1e-5
