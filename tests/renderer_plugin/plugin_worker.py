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

    import foundation_pose_nvidia as fpn
    from foundation_pose_nvidia.bindings import CreateOptions, PoseResult

    lib = fpn.load_library(print_build_info=False)
    plugin = C.CDLL(args.plugin) if args.plugin else None
    if args.renderer:
        os.environ["FP_RENDERER"] = args.renderer
    else:
        os.environ.pop("FP_RENDERER", None)
    cfg = lib.default_config()
    cfg.n_hypotheses = args.n_hyp
    cfg.batch_size = args.n_hyp
    cfg.tensorrt_precision = 2  # FP16
    cfg.max_image_width, cfg.max_image_height = 640, 480
    strings = [args.obj.encode(), args.refine.encode(), args.score.encode(), args.workdir.encode()]
    opts = CreateOptions(strings[0], 0, 1.0, strings[1], strings[2], strings[3])
    err = C.create_string_buffer(2048)
    h = lib.cdll.fp_create(C.byref(opts), C.byref(cfg), err, len(err))
    out = {"created": bool(h), "error": err.value.decode()}
    if plugin is not None and hasattr(plugin, "fp_test_plugin_created"):
        out.update(factory_calls=plugin.fp_test_plugin_created(), device_id=plugin.fp_test_plugin_device_id(),
                   max_batch=plugin.fp_test_plugin_max_batch())
    if h and args.scene_seed >= 0:
        from oracle_lib import Oracle
        from scene_util import make_scene

        scene = make_scene(Oracle(), "ellipsoid", seed=args.scene_seed)
        view = fpn.RgbdFrame(scene.rgb, scene.depth, scene.K, scene.mask).to_image_view(with_mask=True)
        res = PoseResult()
        rc = lib.cdll.fp_register_frame(h, C.byref(view), 2, -1, C.byref(res), err, len(err))
        out.update(register_rc=rc, register_error=err.value.decode(), pose=list(res.pose_row_major),
                   score=float(res.score))
        if plugin is not None and hasattr(plugin, "fp_test_plugin_render_calls"):
            out["render_calls"] = plugin.fp_test_plugin_render_calls()
    if h:
        lib.cdll.fp_destroy(h)
    print(json.dumps(out))


if __name__ == "__main__":
    main()
