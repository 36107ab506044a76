"""torchrun worker for tests/test_gpu_sharded.py: every rank registers the same
seeded scene with its shard of the hypotheses (NCCL all-gather of ScoreNet
features and poses); rank 0 also runs a single-GPU register and writes both
results to a JSON file."""
from __future__ import annotations

import datetime
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist


def main() -> None:
    obj, refine, score, workdir, out = sys.argv[1:6]
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    import foundation_pose_nvidia as fpn
    from oracle_lib import Oracle
    from scene_util import make_scene

    scene = make_scene(Oracle(), "ellipsoid", seed=6)
    n_hyp = 42
    cfg = fpn.RuntimeConfig(n_hypotheses=n_hyp, tensorrt_precision=fpn.Precision.FP16, max_image_width=640,
                            max_image_height=480, batch_size=n_hyp)
    from pathlib import Path

    opts = fpn.EstimatorOptions(cad_path=Path(obj), refine_model_path=Path(refine), score_model_path=Path(score),
                                engine_cache_dir=Path(workdir), device_id=local, prepare=False)
    lib = fpn.load_library(print_build_info=False)
    frame = fpn.RgbdFrame(scene.rgb, scene.depth, scene.K, scene.mask)
    with fpn.Estimator(opts, cfg, library=lib) as est:
        r = fpn.register_sharded(est, frame, n_hypotheses=n_hyp, n_refine=2)
    pose = torch.tensor(np.asarray(r.pose, np.float32).reshape(-1), device="cuda")
    gathered = [torch.empty_like(pose) for _ in range(world)]
    dist.all_gather(gathered, pose)
    same = all(torch.equal(g, gathered[0]) for g in gathered)
    if rank == 0:
        with fpn.Estimator(opts, cfg, library=lib) as est:
            s = est.register(frame, n_refine=2, n_hypotheses=n_hyp)
        with open(out, "w") as f:
            json.dump({"world": world, "sharded_pose": np.asarray(r.pose, np.float32).reshape(-1).tolist(),
                       "single_pose": np.asarray(s.pose, np.float32).reshape(-1).tolist(),
                       "sharded_score": float(r.score), "single_score": float(s.score),
                       "all_ranks_equal": bool(same)}, f)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
