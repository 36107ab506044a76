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
    from fp_b200.capi import Api, image_view
    from fp_b200.sharded import register_sharded
    from oracle_lib import Oracle
    from scene_util import make_scene

    scene = make_scene(Oracle(), "ellipsoid", seed=6)
    n_hyp = 42
    api = Api()
    cfg = api.default_config(n_hypotheses=n_hyp, tensorrt_precision=2, max_image_width=640, max_image_height=480,
                             batch_size=n_hyp)
    opts = Api.options(obj, refine, score, local, workdir)
    view = image_view(scene.rgb, scene.depth, scene.K, scene.mask)
    h = api.create(opts, cfg)
    r_pose, r_score = register_sharded(api, h, view, n_hyp, n_refine=2)
    api.destroy(h)
    pose = torch.tensor(r_pose.reshape(-1), device="cuda")
    gathered = [torch.empty_like(pose) for _ in range(world)]
    dist.all_gather(gathered, pose)
    same = all(torch.equal(g, gathered[0]) for g in gathered)
    if rank == 0:
        h = api.create(opts, cfg)
        s_pose, s_score = api.register(h, view, 2, n_hyp)
        api.destroy(h)
        with open(out, "w") as f:
            json.dump({"world": world, "sharded_pose": r_pose.reshape(-1).tolist(),
                       "single_pose": s_pose.reshape(-1).tolist(),
                       "sharded_score": float(r_score), "single_score": float(s_score),
                       "all_ranks_equal": bool(same)}, f)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
