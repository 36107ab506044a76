"""Register one frame with its hypotheses split across GPUs (one process per
GPU, torch.distributed over NCCL).

Each rank owns an Estimator on its own device, created from the same mesh and
configuration. The n hypotheses are split into contiguous ranges (the first
n % world ranks take one extra); every rank refines its range and computes its
ScoreNet features through fp_register_shard_begin, the features and refined
poses are all-gathered (NCCL over NVLink on GPUs), and every rank runs the
cross-hypothesis ScoreNet head and the arg-max through fp_register_shard_finish,
so all ranks return the same pose, equal to a single-GPU register of the same
frame. This path has no counterpart in the reference (whose register runs on
one GPU, src/foundation_pose.cpp:410-462); it is the sharding described for its
hot path.
"""
from __future__ import annotations

import ctypes as C
import time

from foundation_pose_nvidia.bindings import PoseResult
from foundation_pose_nvidia.core.frame import RgbdFrame
from foundation_pose_nvidia.core.types import PoseEstimate
from foundation_pose_nvidia.exceptions import FoundationPoseError

FEATURE_DIM = 512  # FP_SCORE_FEATURE_DIM


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [begin, begin + count) of n hypotheses for `rank` of `world`."""
    if n <= 0 or world <= 0 or not 0 <= rank < world:
        raise ValueError("need n > 0 and 0 <= rank < world")
    base, extra = divmod(n, world)
    count = base + (1 if rank < extra else 0)
    begin = rank * base + min(rank, extra)
    return begin, count


def gather_shards(local, n: int, group=None):
    """All-gather every rank's shard rows (`local`: [ceil(n/world), d], its
    first `count` rows valid) into [n, d] in hypothesis order, on every rank."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    per = -(-n // world)
    if local.shape[0] != per:
        raise ValueError(f"local shard buffer must have {per} rows")
    if dist.get_backend(group) == "nccl":
        flat = torch.empty((world * per,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(flat, local.contiguous(), group=group)
        parts = [flat[r * per: r * per + shard_range(n, world, r)[1]] for r in range(world)]
    else:
        bufs = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(bufs, local.contiguous(), group=group)
        parts = [bufs[r][: shard_range(n, world, r)[1]] for r in range(world)]
    return torch.cat(parts, 0).contiguous()


def register_sharded(estimator, frame: RgbdFrame, *, n_hypotheses: int, n_refine: int = -1,
                     group=None) -> PoseEstimate:
    """Sharded register of `frame` over the ranks of `group`; every rank calls
    it with its own estimator (on its own GPU) and the same arguments."""
    import torch
    import torch.distributed as dist

    if frame.mask is None:
        raise ValueError("register requires a mask")
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    device = torch.device("cuda", torch.cuda.current_device())
    begin, count = shard_range(n_hypotheses, world, rank)
    per = -(-n_hypotheses // world)
    feats = torch.zeros((per, FEATURE_DIM), dtype=torch.float32, device=device)
    poses = torch.zeros((per, 16), dtype=torch.float32, device=device)
    view = frame.to_image_view(with_mask=True)
    err = C.create_string_buffer(4096)
    lib = estimator.lib
    t0 = time.perf_counter()
    torch.cuda.synchronize(device)
    if lib.fp_register_shard_begin(estimator.handle, C.byref(view), n_refine, n_hypotheses, begin, count,
                                   C.c_void_p(feats.data_ptr()), C.c_void_p(poses.data_ptr()), err,
                                   len(err)) != 0:
        raise FoundationPoseError(err.value.decode("utf-8"))
    all_feats = gather_shards(feats, n_hypotheses, group)
    all_poses = gather_shards(poses, n_hypotheses, group)
    torch.cuda.synchronize(device)
    result = PoseResult()
    if lib.fp_register_shard_finish(estimator.handle, C.c_void_p(all_feats.data_ptr()),
                                    C.c_void_p(all_poses.data_ptr()), n_hypotheses, C.byref(result), err,
                                    len(err)) != 0:
        raise FoundationPoseError(err.value.decode("utf-8"))
    return PoseEstimate.from_ctypes(result.pose_row_major, result.score, time.perf_counter() - t0)
