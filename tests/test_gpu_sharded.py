"""GPU tests of the sharded register (fp_register_shard_begin / _finish): the
hypotheses of one frame split into contiguous shards, features and poses
gathered, cross-hypothesis ScoreNet head + arg-max on the gathered set. The
result must equal a single-GPU fp_register_frame of the same frame bit for bit
(RefineNet and the per-hypothesis ScoreNet part are per-sample, the gathered
set is in hypothesis order). On one GPU the shards run as separate handles;
with two or more GPUs the same path runs under torchrun over NCCL."""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from fp_b200.capi import Api, FpError, image_view  # noqa: E402
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
    return dict(dir=d, refine=refine, score=score, scene=scene, obj=obj, lib=Api())


def create(env, n_hyp, batch=None):
    lib = env["lib"]
    cfg = lib.default_config(n_hypotheses=n_hyp, tensorrt_precision=FP16, max_image_width=640,
                             max_image_height=480, batch_size=batch or n_hyp)
    return lib.create(Api.options(env["obj"], env["refine"], env["score"], 0, env["dir"]), cfg)


def frame_view(scene, mask=True):
    return image_view(scene.rgb, scene.depth, scene.K, scene.mask if mask else None)


@pytest.mark.parametrize("n_hyp,cuts", [(42, [0, 21, 42]), (42, [0, 11, 22, 32, 42]), (7, [0, 4, 7])])
def test_sharded_register_equals_single_register(env, n_hyp, cuts):
    lib, scene = env["lib"], env["scene"]
    ref_h = create(env, n_hyp)
    ref_pose, ref_score = lib.register(ref_h, frame_view(scene), 2, n_hyp)
    handles, feats, poses = [], [], []
    for b, e in zip(cuts, cuts[1:]):
        h = create(env, n_hyp)  # micro-batch = min(batch_size, shard size) = the shard
        f = torch.full((e - b, 512), float("nan"), device="cuda")
        p = torch.full((e - b, 16), float("nan"), device="cuda")
        lib.shard_begin(h, frame_view(scene), 2, n_hyp, b, e - b, f.data_ptr(), p.data_ptr())
        assert torch.isfinite(f).all() and torch.isfinite(p).all()
        handles.append(h)
        feats.append(f)
        poses.append(p)
    all_f = torch.cat(feats).contiguous()
    all_p = torch.cat(poses).contiguous()
    torch.cuda.synchronize()
    pose, score = lib.shard_finish(handles[0], all_f.data_ptr(), all_p.data_ptr(), n_hyp)
    assert np.array_equal(pose, ref_pose) and score == ref_score
    # The finishing handle tracks on from the selected pose, like a registered one.
    t_ref = lib.track(ref_h, frame_view(scene, False), 2)[0]
    t_out = lib.track(handles[0], frame_view(scene, False), 2)[0]
    assert np.array_equal(t_out, t_ref)
    for h in handles + [ref_h]:
        lib.destroy(h)


def test_shard_arguments_are_checked(env):
    lib, scene = env["lib"], env["scene"]
    h = create(env, 42)
    f = torch.zeros(42, 512, device="cuda")
    p = torch.zeros(42, 16, device="cuda")
    with pytest.raises(FpError, match="outside the 42 active hypotheses"):
        lib.shard_begin(h, frame_view(scene), 2, 42, 40, 5, f.data_ptr(), p.data_ptr())
    with pytest.raises(FpError, match="shard outputs are required"):
        lib.shard_begin(h, frame_view(scene), 2, 42, 0, 10, None, p.data_ptr())
    with pytest.raises(FpError):
        lib.shard_finish(h, f.data_ptr(), p.data_ptr(), 0)
    lib.destroy(h)


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
