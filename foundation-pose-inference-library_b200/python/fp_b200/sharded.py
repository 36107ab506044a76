"""Register one frame with its hypotheses split across GPUs (one process per
GPU, torch.distributed over NCCL).

Every rank owns an estimator handle on its own device, created from the same
mesh and configuration. The n hypotheses are cut into contiguous ranges (the
first n % world ranks take one more); each rank refines its range and
computes the per-hypothesis ScoreNet features with fp_register_shard_begin;
the features and refined poses are all-gathered; every rank then runs the
cross-hypothesis ScoreNet head and the arg-max with fp_register_shard_finish,
so all ranks return the same pose, bit-identical to a one-GPU register of the
same frame. The reference registers on one GPU only
(src/foundation_pose.cpp:312-377); this is the sharding of its hot path.
"""
from __future__ import annotations

from .capi import SCORE_FEATURE_DIM, Api, fp_image_view_t


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """(begin, count) of rank's contiguous share of n hypotheses."""
    if n <= 0 or world <= 0 or not 0 <= rank < world:
        raise ValueError("need n > 0 and 0 <= rank < world")
    q, r = divmod(n, world)
    return rank * q + min(rank, r), q + (rank < r)


def gather_shards(local, n: int, group=None):
    """Every rank's first `count` rows of `local` ([ceil(n/world), d]) stacked
    in rank order into [n, d] on every rank. NCCL takes one flat all-gather;
    other backends (gloo on CPU) a list all-gather."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rows = -(-n // world)
    if local.shape[0] != rows:
        raise ValueError(f"local shard buffer must have {rows} rows")
    counts = [shard_range(n, world, r)[1] for r in range(world)]
    local = local.contiguous()
    if dist.get_backend(group) == "nccl":
        flat = local.new_empty((world * rows,) + tuple(local.shape[1:]))
        dist.all_gather_into_tensor(flat, local, group=group)
        chunks = flat.split(rows)
    else:
        chunks = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(chunks, local, group=group)
    return torch.cat([c[:k] for c, k in zip(chunks, counts)]).contiguous()


def register_sharded(api: Api, handle: int, view: fp_image_view_t, n_hypotheses: int, n_refine: int = -1,
                     group=None):
    """One sharded register; every rank of `group` calls it with its own handle
    and the same arguments. Returns (pose 4x4, score), equal on every rank."""
    import torch
    import torch.distributed as dist

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    dev = torch.device("cuda", torch.cuda.current_device())
    begin, count = shard_range(n_hypotheses, world, rank)
    rows = -(-n_hypotheses // world)
    feats = torch.zeros((rows, SCORE_FEATURE_DIM), dtype=torch.float32, device=dev)
    poses = torch.zeros((rows, 16), dtype=torch.float32, device=dev)
    torch.cuda.synchronize(dev)
    api.shard_begin(handle, view, n_refine, n_hypotheses, begin, count, feats.data_ptr(), poses.data_ptr())
    all_feats = gather_shards(feats, n_hypotheses, group)
    all_poses = gather_shards(poses, n_hypotheses, group)
    torch.cuda.synchronize(dev)
    return api.shard_finish(handle, all_feats.data_ptr(), all_poses.data_ptr(), n_hypotheses)
