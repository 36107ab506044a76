"""FP_RENDERER plugin loader (reference src/foundation_pose.cpp:40-68).

With FP_RENDERER=nvdiffrast the estimator builds its renderer through
`fp_plugin_create_renderer(const Config*, int device_id, int max_batch)` of
libfoundation_pose_nvdiffrast.so; otherwise it uses the built-in rasterizer.
The plugin here (renderer_plugin/fp_test_renderer_plugin.cpp, built with g++ at
test time) renders through fpk_render, so a register through it runs the
unfused IRenderer path (NHWC fp32 images -> NCHW pack -> networks) and must
return the pose of the fused built-in path.

Each case runs in a fresh interpreter (renderer_plugin/plugin_worker.py): the
runtime loads the plugin once per process. CPU cases: plugin missing, plugin
without the factory, factory returning NULL, factory arguments. GPU case:
register through the plugin equals the built-in register.
"""
from __future__ import annotations

import json
import os
import shutil
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "foundation-pose-inference-library_b200"
LIB_DIR = PKG / "lib"
SRC = Path(__file__).resolve().parent / "renderer_plugin" / "fp_test_renderer_plugin.cpp"
WORKER = Path(__file__).resolve().parent / "renderer_plugin" / "plugin_worker.py"
SONAME = "libfoundation_pose_nvdiffrast.so"
CUDA_INC = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "include"

TETRA = """v 0 0 0 1 0 0
v 0.05 0 0 0 1 0
v 0 0.05 0 0 0 1
v 0 0 0.05 1 1 0
f 1 3 2
f 1 2 4
f 1 4 3
f 2 3 4
"""


def build_plugin(out_dir: Path, variant: str = "") -> Path:
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    if not (LIB_DIR / "libfoundation_pose_nvidia.so").exists():
        pytest.skip("main library not built")
    out_dir.mkdir(parents=True, exist_ok=True)
    so = out_dir / SONAME
    cmd = ["g++", "-std=c++20", "-O2", "-fPIC", "-shared", "-fvisibility=hidden", *([f"-D{variant}"] if variant else []),
           f"-I{ROOT / 'include'}", f"-I{CUDA_INC}", str(SRC), "-o", str(so), f"-Wl,-soname,{SONAME}",
           f"-L{LIB_DIR}", "-l:libfoundation_pose_nvidia.so", f"-Wl,-rpath,{LIB_DIR}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return so


def run_worker(*args: str, timeout: int = 300) -> dict:
    env = dict(os.environ)
    env.pop("FP_RENDERER", None)
    r = subprocess.run([sys.executable, str(WORKER), *args], capture_output=True, text=True, timeout=timeout,
                       env=env)
    assert r.returncode == 0, r.stderr[-4000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


@pytest.fixture(scope="module")
def tetra(tmp_path_factory) -> Path:
    p = tmp_path_factory.mktemp("plugin_mesh") / "tetra.obj"
    p.write_text(TETRA)
    return p


def test_missing_plugin_is_an_error(tetra):
    if (LIB_DIR / SONAME).exists():
        pytest.skip("a renderer plugin is installed next to the main library")
    out = run_worker("--obj", str(tetra))
    assert not out["created"]
    assert "FP_RENDERER=nvdiffrast requested but the renderer plugin could not be loaded" in out["error"]
    assert SONAME in out["error"]


def test_plugin_without_factory_is_an_error(tetra, tmp_path):
    so = build_plugin(tmp_path / "nofactory", "FP_TEST_PLUGIN_NO_FACTORY")
    out = run_worker("--obj", str(tetra), "--plugin", str(so))
    assert not out["created"]
    assert out["error"] == "nvdiffrast renderer plugin is missing fp_plugin_create_renderer"


def test_plugin_factory_returning_null_is_an_error(tetra, tmp_path):
    so = build_plugin(tmp_path / "null", "FP_TEST_PLUGIN_NULL_FACTORY")
    out = run_worker("--obj", str(tetra), "--plugin", str(so))
    assert not out["created"]
    assert out["error"] == "nvdiffrast renderer plugin failed to create a renderer"


def test_factory_receives_config_device_and_max_batch(tetra, tmp_path):
    so = build_plugin(tmp_path / "ok")
    out = run_worker("--obj", str(tetra), "--plugin", str(so), "--n-hyp", "37")
    assert out["factory_calls"] == 1
    assert out["device_id"] == 0
    assert out["max_batch"] == 37
    # Without a GPU the estimator then fails on its first CUDA call, not in the loader.
    assert "renderer plugin" not in out["error"]


def test_other_renderer_names_use_the_builtin(tetra, tmp_path):
    so = build_plugin(tmp_path / "ok2")
    out = run_worker("--obj", str(tetra), "--plugin", str(so), "--renderer", "builtin")
    assert out["factory_calls"] == 0


@pytest.mark.gpu
def test_register_through_plugin_matches_builtin(tmp_path, oracle):
    import numpy as np

    from fp_b200.weights import make_default_packs
    from scene_util import make_scene, write_obj

    refine, score = make_default_packs(tmp_path, seed=3)
    scene = make_scene(oracle, "ellipsoid", seed=4)
    obj = tmp_path / "object.obj"
    write_obj(obj, scene.verts, scene.faces, scene.colors_u8)
    so = build_plugin(tmp_path / "plugin")
    common = ["--obj", str(obj), "--refine", str(refine), "--score", str(score), "--workdir", str(tmp_path),
              "--scene-seed", "4", "--n-hyp", "42"]
    via_plugin = run_worker(*common, "--plugin", str(so))
    builtin = run_worker(*common, "--renderer", "")
    assert via_plugin["created"], via_plugin["error"]
    assert builtin["created"], builtin["error"]
    assert via_plugin["register_rc"] == 0, via_plugin["register_error"]
    assert builtin["register_rc"] == 0, builtin["register_error"]
    assert via_plugin["factory_calls"] == 1
    assert via_plugin["render_calls"] >= 3  # 2 refinement passes + the scoring render
    a = np.asarray(via_plugin["pose"], np.float32).reshape(4, 4)
    b = np.asarray(builtin["pose"], np.float32).reshape(4, 4)
    assert np.abs(a[:3, 3] - b[:3, 3]).max() < 1e-5
    assert np.abs(a[:3, :3] - b[:3, :3]).max() < 1e-5
    assert abs(via_plugin["score"] - builtin["score"]) < 1e-4 * max(1.0, abs(builtin["score"]))
