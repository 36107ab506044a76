"""Fresh-process worker for tests/test_renderer_plugin.py. The runtime loads the
renderer plugin once per process, so every loader case runs in its own
interpreter: optionally pre-load a plugin build (found by its soname), set
FP_RENDERER, call fp_create and, with --register, register one seeded scene.
Prints one JSON line."""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "foundation-pose-inference-library_b200" / "python"))
sys.path.insert(0, str(ROOT / "tests"))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--plugin", default="")
    ap.add_argument("--renderer", default="nvdiffrast")
    ap.add_argument("--obj", required=True)
    ap.add_argument("--refine", default="refine.fpw")
    ap.add_argument("--score", default="score.fpw")
    ap.add_argument("--workdir", default=".")
    ap.add_argument("--n-hyp", type=int, default=42)
    ap.add_argument("--scene-seed", type=int, default=-1)
    args = ap.parse_args()

    from fp_b200.capi import Api, FpError, image_view

    api = Api()
    plugin = C.CDLL(args.plugin) if args.plugin else None
    if args.renderer:
        os.environ["FP_RENDERER"] = args.renderer
    else:
        os.environ.pop("FP_RENDERER", None)
    cfg = api.default_config(n_hypotheses=args.n_hyp, batch_size=args.n_hyp, tensorrt_precision=2,  # FP16
                             max_image_width=640, max_image_height=480)
    try:
        h, error = api.create(Api.options(args.obj, args.refine, args.score, 0, args.workdir), cfg), ""
    except FpError as e:
        h, error = None, str(e)
    out = {"created": bool(h), "error": error}
    if plugin is not None and hasattr(plugin, "fp_test_plugin_created"):
        out.update(factory_calls=plugin.fp_test_plugin_created(), device_id=plugin.fp_test_plugin_device_id(),
                   max_batch=plugin.fp_test_plugin_max_batch())
    if h and args.scene_seed >= 0:
        from oracle_lib import Oracle
        from scene_util import make_scene

        scene = make_scene(Oracle(), "ellipsoid", seed=args.scene_seed)
        r = api.register_frame(h, image_view(scene.rgb, scene.depth, scene.K, scene.mask), 2, -1)
        out.update(register_rc=r.rc, register_error=r.error, pose=r.pose.reshape(-1).tolist(), score=r.score)
        if plugin is not None and hasattr(plugin, "fp_test_plugin_render_calls"):
            out["render_calls"] = plugin.fp_test_plugin_render_calls()
    if h:
        api.destroy(h)
    print(json.dumps(out))


if __name__ == "__main__":
    main()
