"""Multi-object groups (fp_group_*, BASELINE configs[4]) with one object per GPU.

Each object of a group runs on its own device through the group's persistent
per-device workers; the reference's invariant (tests/test_group_api.py:167-183)
is that a group register equals a single-estimator register of the same object
(|dpose| < 1e-5), and a NULL mask / inactive flag skips the object. Runs on as
many GPUs as the box has (up to 4 objects); on one GPU every object shares
device 0."""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from fp_b200.capi import FP_OBJECT_OK, FP_OBJECT_SKIPPED, Api, image_view  # noqa: E402
from fp_b200.weights import make_default_packs  # noqa: E402
from scene_util import make_scene, write_obj  # noqa: E402

pytestmark = pytest.mark.gpu
FP16 = 2


@pytest.fixture(scope="module")
def group_env(tmp_path_factory, oracle):
    d = tmp_path_factory.mktemp("group")
    refine, score = make_default_packs(d, seed=6)
    n_dev = torch.cuda.device_count()
    n_obj = max(2, min(4, n_dev))
    kinds = ["ellipsoid", "sphere50k", "ellipsoid_small", "cube"]
    scenes, objs = [], []
    for i in range(n_obj):
        s = make_scene(oracle, kinds[i], seed=20 + i)
        obj = d / f"object{i}.obj"
        write_obj(obj, s.verts, s.faces, s.colors_u8)
        scenes.append(s)
        objs.append(obj)
    return dict(dir=d, refine=refine, score=score, scenes=scenes, objs=objs,
                devices=[i % n_dev for i in range(n_obj)])


def test_group_one_object_per_gpu_matches_single(group_env):
    api = Api()
    cfg = api.default_config(n_hypotheses=42, batch_size=42, tensorrt_precision=FP16, max_image_width=640,
                             max_image_height=480)
    env = group_env
    opts = [api.options(o, env["refine"], env["score"], dev, env["dir"]) for o, dev in zip(env["objs"], env["devices"])]
    g = api.group_create(opts, cfg)
    try:
        n = len(opts)
        # One shared frame of the first scene; every object registers against its own mask.
        frame = env["scenes"][0]
        masks = [s.mask for s in env["scenes"]]
        view = image_view(frame.rgb, frame.depth, frame.K)
        fails, poses, scores, statuses, err = api.group_register(g, view, masks, n_refine=2)
        assert fails == 0, err
        assert statuses == [FP_OBJECT_OK] * n
        for i in range(n):
            torch.cuda.set_device(env["devices"][i])
            h = api.create(opts[i], cfg)
            pose, score = api.register(h, image_view(frame.rgb, frame.depth, frame.K, masks[i]), 2)
            assert np.abs(poses[i] - pose).max() < 1e-5 and abs(scores[i] - score) < 1e-5, i
            api.destroy(h)
        torch.cuda.set_device(0)
        # Track on: object 1 inactive this frame.
        active = [1] * n
        active[1] = 0
        fails, tposes, _, statuses, err = api.group_track(g, view, active, n, n_refine=2)
        assert fails == 0, err
        assert statuses[1] == FP_OBJECT_SKIPPED and all(statuses[i] == FP_OBJECT_OK for i in range(n) if i != 1)
        assert all(np.isfinite(tposes[i]).all() for i in range(n) if i != 1)
        # A NULL mask skips an object at register.
        masks[0] = None
        fails, _, _, statuses, err = api.group_register(g, view, masks, n_refine=2)
        assert fails == 0 and statuses[0] == FP_OBJECT_SKIPPED, err
    finally:
        api.lib.fp_group_destroy(g)


def test_group_reports_failing_object(group_env):
    """A frame larger than the objects' configured maximum fails every active
    object; the first failure message names its object index."""
    api = Api()
    cfg = api.default_config(n_hypotheses=6, batch_size=6, tensorrt_precision=FP16, max_image_width=320,
                             max_image_height=240)
    env = group_env
    opts = [api.options(o, env["refine"], env["score"], dev, env["dir"]) for o, dev in zip(env["objs"], env["devices"])]
    g = api.group_create(opts, cfg)
    try:
        s = env["scenes"][0]
        fails, _, _, statuses, err = api.group_register(g, image_view(s.rgb, s.depth, s.K), [s.mask] * len(opts), 1)
        assert fails == len(opts) and all(st == 1 for st in statuses)
        assert err.startswith("object 0: ") and "max_image_width" in err
    finally:
        api.lib.fp_group_destroy(g)
