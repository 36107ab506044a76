"""GPU tests of the sharded register (fp_register_shard_begin / _finish): the
hypotheses of one frame split into contiguous shards, features and poses
gathered, cross-hypothesis ScoreNet head + arg-max on the gathered set. The
result must equal a single-GPU fp_register_frame of the same frame bit for bit
(RefineNet and the per-hypothesis ScoreNet part are per-sample, the gathered
set is in hypothesis order). On one GPU the shards run as separate handles;
with two or more GPUs the same path runs under torchrun over NCCL."""
from __future__ import annotations

import ctypes as C
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import foundation_pose_nvidia as fpn  # noqa: E402
from foundation_pose_nvidia.bindings import CreateOptions, PoseResult  # noqa: E402
from fp_b200.weights import make_default_packs  # noqa: E402
from scene_util import make_scene, write_obj  # noqa: E402

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
FP16 = 2


@pytest.fixture(scope="module")
def env(tmp_path_factory, oracle):
    d = tmp_path_factory.mktemp("sharded")
    refine, score = make_default_packs(d, seed=5)
    scene = make_scene(oracle, "ellipsoid", seed=6)
    obj = d / "object.obj"
    write_obj(obj, scene.verts, scene.faces, scene.colors_u8)
    lib = fpn.load_library(print_build_info=False)
    return dict(dir=d, refine=refine, score=score, scene=scene, obj=obj, lib=lib)


def create(env, n_hyp, batch=None):
    lib = env["lib"]
    cfg = lib.default_config()
    cfg.n_hypotheses, cfg.tensorrt_precision = n_hyp, FP16
    cfg.max_image_width, cfg.max_image_height = 640, 480
    cfg.batch_size = batch or n_hyp
    s = [str(env["obj"]).encode(), str(env["refine"]).encode(), str(env["score"]).encode(),
         str(env["dir"]).encode()]
    opts = CreateOptions(s[0], 0, 1.0, s[1], s[2], s[3])
    err = C.create_string_buffer(1024)
    h = lib.cdll.fp_create(C.byref(opts), C.byref(cfg), err, len(err))
    assert h, err.value.decode()
    return h, s


def frame_view(scene, mask=True):
    return fpn.RgbdFrame(scene.rgb, scene.depth, scene.K, scene.mask if mask else None).to_image_view(
        with_mask=mask)


@pytest.mark.parametrize("n_hyp,cuts", [(42, [0, 21, 42]), (42, [0, 11, 22, 32, 42]), (7, [0, 4, 7])])
def test_sharded_register_equals_single_register(env, n_hyp, cuts):
    lib, scene = env["lib"], env["scene"]
    L = lib.cdll
    err = C.create_string_buffer(1024)
    ref_h, _ = create(env, n_hyp)
    ref = PoseResult()
    assert L.fp_register_frame(ref_h, C.byref(frame_view(scene)), 2, n_hyp, C.byref(ref), err, len(err)) == 0, \
        err.value.decode()
    handles, feats, poses = [], [], []
    for b, e in zip(cuts, cuts[1:]):
        h, _ = create(env, n_hyp)  # micro-batch = min(batch_size, shard size) = the shard
        f = torch.full((e - b, 512), float("nan"), device="cuda")
        p = torch.full((e - b, 16), float("nan"), device="cuda")
        rc = L.fp_register_shard_begin(h, C.byref(frame_view(scene)), 2, n_hyp, b, e - b, f.data_ptr(), p.data_ptr(),
                                       err, len(err))
        assert rc == 0, err.value.decode()
        assert torch.isfinite(f).all() and torch.isfinite(p).all()
        handles.append(h)
        feats.append(f)
        poses.append(p)
    all_f = torch.cat(feats).contiguous()
    all_p = torch.cat(poses).contiguous()
    torch.cuda.synchronize()
    out = PoseResult()
    rc = L.fp_register_shard_finish(handles[0], all_f.data_ptr(), all_p.data_ptr(), n_hyp, C.byref(out), err,
                                    len(err))
    assert rc == 0, err.value.decode()
    assert list(out.pose_row_major) == list(ref.pose_row_major) and out.score == ref.score
    # The finishing handle tracks on from the selected pose, like a registered one.
    t_ref, t_out = PoseResult(), PoseResult()
    assert L.fp_track_frame(ref_h, C.byref(frame_view(scene, False)), 2, C.byref(t_ref), err, len(err)) == 0
    assert L.fp_track_frame(handles[0], C.byref(frame_view(scene, False)), 2, C.byref(t_out), err, len(err)) == 0
    assert list(t_out.pose_row_major) == list(t_ref.pose_row_major)
    for h in handles + [ref_h]:
        L.fp_destroy(h)


def test_shard_arguments_are_checked(env):
    lib, scene = env["lib"], env["scene"]
    L = lib.cdll
    err = C.create_string_buffer(1024)
    h, _ = create(env, 42)
    f = torch.zeros(42, 512, device="cuda")
    p = torch.zeros(42, 16, device="cuda")
    assert L.fp_register_shard_begin(h, C.byref(frame_view(scene)), 2, 42, 40, 5, f.data_ptr(), p.data_ptr(),
                                     err, len(err)) != 0
    assert "outside the 42 active hypotheses" in err.value.decode()
    assert L.fp_register_shard_begin(h, C.byref(frame_view(scene)), 2, 42, 0, 10, None, p.data_ptr(), err,
                                     len(err)) != 0
    assert "shard outputs are required" in err.value.decode()
    out = PoseResult()
    assert L.fp_register_shard_finish(h, f.data_ptr(), p.data_ptr(), 0, C.byref(out), err, len(err)) != 0
    L.fp_destroy(h)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_sharded_register_over_nccl(env, tmp_path):
    n_gpu = min(torch.cuda.device_count(), 4)
    out = tmp_path / "result.json"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n_gpu}",
           "--master-addr=127.0.0.1", "--master-port=29517", str(ROOT / "tests" / "sharded_worker.py"),
           str(env["obj"]), str(env["refine"]), str(env["score"]), str(env["dir"]), str(out)]
    envv = dict(os.environ, NCCL_NVLS_ENABLE="0",
                PYTHONPATH=os.pathsep.join([str(ROOT / "foundation-pose-inference-library_b200" / "python"),
                                            str(ROOT / "tests"), os.environ.get("PYTHONPATH", "")]))
    r = subprocess.run(["timeout", "-k", "30", "600"] + cmd, env=envv, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads(out.read_text())
    assert res["world"] == n_gpu
    assert res["sharded_pose"] == res["single_pose"] and res["sharded_score"] == res["single_score"]
    assert res["all_ranks_equal"]
