#!/usr/bin/env python
"""Benchmark of the FoundationPose B200 runtime: register throughput.

Workload (synthetic stand-in for BOP YCB-V): one 640x480
RGB-D frame + mask rendered from a ground-truth pose of a seeded 50k-triangle
displaced sphere with per-vertex colours; register = 252 hypotheses, 5
RefineNet iterations, ScoreNet over all 252, FP16, batch_size 252; weights are
a seeded random init of the RefineNet/ScoreNet architecture (no checkpoint is
available offline). One step = one fp_register_frame call through the C ABI.

  value   hypotheses/s over all ranks with the frame already in HBM
  e2e     same metric with pinned host frame buffers (H2D + pose D2H inside)
  roofline  the tensor-core GEMM kernel: algorithmic FLOPs / CUDA-event time
  cpu_baseline  the CPU restatement (oracle) + torch CPU networks, bounded sample

Multi-GPU (torchrun): every rank registers its own frame (replicas, weak
scaling); timing is the max over ranks. `--impl reference` times the CPU
implementation of the same path (reference CPU preprocessing from oracle/_ref,
CPU oracle for render/pack/pose kernels, torch fp32 networks on all host cores).
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "foundation-pose-inference-library_b200"
sys.path.insert(0, str(PKG / "python"))

N_HYP = 252
# gemmKernel DRAM traffic per TFLOP of algorithmic GEMM work, from one ncu
# capture over whole register calls (profiles/gemm_dram_traffic_register.md).
GEMM_DRAM_BYTES_PER_TFLOP = 28596.3e6 / 28.99
N_ITERS = 5
W, H = 640, 480
FP16 = 2
METRIC = "register hypotheses/s (252 hyp, 5 refine iters + ScoreNet, 640x480, FP16)"
WORKLOAD = "configs[1]: register, 50k-tri displaced sphere, 640x480 RGB-D+mask, 252 hyp, 5 iters, batch 252, FP16"


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ---------------------------------------------------------------------------
# Scene
# ---------------------------------------------------------------------------

def build_scene(workdir: Path, seed: int):
    from fp_b200 import synthetic as syn
    from fp_b200.weights import make_default_packs

    mesh = syn.displaced_sphere(seed)
    obj = workdir / "object.obj"
    with open(obj, "w") as f:
        for v, c in zip(mesh.vertices, mesh.colors):
            enc = [1.0 if x >= 255 else (float(x) + 0.5) / 255.0 for x in c]
            f.write("v %.9g %.9g %.9g %.9g %.9g %.9g\n" % (v[0], v[1], v[2], *enc))
        for t in mesh.faces:
            f.write("f %d %d %d\n" % (t[0] + 1, t[1] + 1, t[2] + 1))
    refine, score = make_default_packs(workdir / "weights", seed=0)
    rng = np.random.default_rng(seed + 17)
    gt = syn.random_pose(rng, dist=(0.65, 0.75), lateral=0.03)
    return mesh, obj, refine, score, gt


def render_frame(mesh, gt):
    from fp_b200 import synthetic as syn
    from fp_b200.kernels import FpkLibrary

    fpk = FpkLibrary()
    normals = syn.vertex_normals(mesh.vertices, mesh.faces)
    rgb, depth = syn.render_frame_gpu(fpk, mesh, normals, gt, syn.K_640, W, H)
    mask = (depth > 0).astype(np.uint8)
    return rgb, depth, mask


# ---------------------------------------------------------------------------
# Clock sampling during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, path: Path):
        self.path = path
        self.proc = None
        try:
            self.fh = open(path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-i", str(gpu_index), "-lms", "200"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU implementation (oracle + reference CPU functions + torch CPU networks)
# ---------------------------------------------------------------------------

def cpu_register_sample(n_sample: int, mesh, rgb, depth, mask, refine_pack, score_pack,
                        iters: int = N_ITERS) -> float:
    """Seconds for n_sample hypotheses through preprocess + `iters` refine
    passes + one score pass on the host (one pass each over the sample)."""
    sys.path.insert(0, str(ROOT / "tests"))
    sys.path.insert(0, str(ROOT / "oracle"))
    import torch
    from fp_b200.weights import read_pack
    from fp_net_ref import NetRef
    from oracle_lib import REF_CPU_SO, Oracle, RefCpu

    from fp_b200 import synthetic as syn

    torch.set_num_threads(os.cpu_count() or 1)
    o = Oracle()
    cfg = o.config()
    k4 = np.array([600.0, 600.0, 320.0, 240.0], np.float32)
    center, diameter, verts = o.mesh_center_diameter(mesh.vertices)
    normals = o.vertex_normals(verts, mesh.faces)
    colors = (mesh.colors.astype(np.float32) / np.float32(255.0)).astype(np.float32)
    nr = NetRef(read_pack(refine_pack)[1])
    ns = NetRef(read_pack(score_pack)[1])
    t0 = time.perf_counter()
    if REF_CPU_SO.is_file():
        filt = RefCpu().preprocess_depth(depth)  # the reference's own CPU preprocessing
    else:
        filt = o.preprocess_cpu(depth, cfg)
    xyz = o.depth_to_xyz(filt, k4, cfg)
    tr = o.initial_translation(filt, mask, k4, cfg)
    rots = o.rotation_grid()[:n_sample]
    poses = o.seed_poses(rots, tr)
    for it in range(iters + 1):
        boxes = o.crop_boxes(poses, k4, diameter, cfg)
        rr, rx, _ = o.render(verts, normals, colors, mesh.faces, poses, boxes, k4, cfg)
        thr = cfg.depth_min if it < iters else 0.1
        a, b = o.pack(rgb, xyz, rr, rx, poses, boxes, diameter, thr, cfg)
        A, B = torch.from_numpy(a), torch.from_numpy(b)
        if it < iters:
            dt, dr = nr.refine(A, B)
            poses = o.apply_deltas(poses, dt.numpy(), dr.numpy(), diameter, cfg)
        else:
            scores = ns.score(A, B).numpy()
            o.select_best(poses, scores, center)
    return time.perf_counter() - t0


def run_reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    work = Path(tempfile.mkdtemp(prefix="fpbench_ref_"))
    mesh, obj, refine, score, gt = build_scene(work, seed=args.seed)
    sys.path.insert(0, str(ROOT / "tests"))
    from oracle_lib import Oracle
    from fp_b200 import synthetic as syn

    # The frame comes from the CPU oracle renderer (no GPU on this arm).
    o = Oracle()
    c, d, verts = o.mesh_center_diameter(mesh.vertices)
    normals = o.vertex_normals(verts, mesh.faces)
    cfg = o.config(input_width=W, input_height=H)
    k4 = np.array([600.0, 600.0, 320.0, 240.0], np.float32)
    gt_c = gt.copy()
    rgbf, xyz, _ = o.render(verts, normals, (mesh.colors / np.float32(255.0)).astype(np.float32),
                            mesh.faces, gt_c.reshape(1, 16), np.array([[0, 0, W, H]], np.float32), k4, cfg)
    rgb = (np.clip(rgbf[0], 0, 1) * 255 + 0.5).astype(np.uint8)
    depth = xyz[0, ..., 2].astype(np.float32)
    mask = (depth > 0).astype(np.uint8)
    n_sample = args.cpu_sample
    for _ in range(args.warmup if args.warmup < 1 else 1):
        cpu_register_sample(n_sample, mesh, rgb, depth, mask, refine, score, iters=1)
    times = [cpu_register_sample(n_sample, mesh, rgb, depth, mask, refine, score) for _ in range(args.steps)]
    per = statistics.mean(times)
    value = n_sample / per
    cores = os.cpu_count() or 1
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "hyp/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per * 1000.0,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": WORKLOAD, "sample": f"{n_sample} of {N_HYP} hypotheses"},
        "cpu_baseline": {"value": value, "unit": "hyp/s", "cores": cores, "kind": "port",
                         "sample": f"{n_sample} hypotheses x (preprocess + 5 refine + 1 score pass); "
                                   "reference CPU preprocessDepth (oracle/_ref), CPU oracle render/pack/pose, "
                                   "torch fp32 networks"},
        "e2e": {"value": value, "unit": "hyp/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.is_file():
        d = json.loads(p.read_text())
        sustained = d.get("bf16_tflops_sustained")
        return {"bf16": sustained or d.get("bf16_tflops"), "hbm": d.get("hbm_gbs"),
                "note": "of measured (" + ("sustained" if sustained else "burst") + " bf16)"}
    # The recipe's fallback: the burst cuBLAS figure (sustained settles near 1.4 PFLOP/s).
    return {"bf16": 1590.0, "hbm": 6650.0, "note": "of fallback (1.59 PFLOP/s burst bf16)"}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--cpu-sample", type=int, default=2)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--track-frames", type=int, default=50)
    ap.add_argument("--e2e-steps", type=int, default=None, help="host-buffer steps (default: --steps)")
    ap.add_argument("--no-graph", dest="graph", action="store_false",
                    help="capture_cuda_graph=0; by default the refinement pass replays as one CUDA graph "
                         "(capture_cuda_graph=1, the reference's own Config option)")
    ap.add_argument("--hyp", type=int, default=252,
                    help="hypotheses per register; values other than 252 are for profiling captures only "
                         "(the workload line then names the reduced count)")
    args = ap.parse_args()
    global N_HYP, WORKLOAD
    if args.hyp != N_HYP:
        N_HYP = args.hyp
        WORKLOAD = WORKLOAD.replace("252 hyp", f"{N_HYP} hyp (profiling)").replace("batch 252", f"batch {N_HYP}")
    if args.impl == "reference":
        run_reference_arm(args)
        return

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300))

    from fp_b200.capi import SCORE_FEATURE_DIM, Api, FP_PRECISION_FP16, image_view
    from fp_b200.kernels import FpkLibrary
    from fp_b200.sharded import gather_shards, shard_range

    work = Path(tempfile.mkdtemp(prefix=f"fpbench_{rank}_"))
    # Every rank builds the same seeded scene: at N > 1 the ranks share one
    # register, each refining its shard of the 252 hypotheses.
    mesh, obj, refine, score, gt = build_scene(work, seed=args.seed)
    rgb, depth, mask = render_frame(mesh, gt)

    api = Api()
    fpk = FpkLibrary()
    fpk.lib.fpk_profile_enable.argtypes = [C.c_int]
    fpk.lib.fpk_profile_read.argtypes = [C.c_void_p] * 4
    cfg = api.default_config(n_hypotheses=N_HYP, n_refine_iters=N_ITERS, batch_size=N_HYP,
                             tensorrt_precision=FP_PRECISION_FP16, capture_cuda_graph=args.graph,
                             max_image_width=W, max_image_height=H)
    opts = Api.options(obj, refine, score, local, work)
    h = api.create(opts, cfg)
    api.prepare(h, N_HYP)

    dev = torch.device("cuda", local)
    d_rgb, d_depth, d_mask = (torch.from_numpy(x).to(dev) for x in (rgb, depth, mask))
    p_rgb, p_depth, p_mask = (torch.from_numpy(x).pin_memory() for x in (rgb, depth, mask))
    K = np.array([[600, 0, 320], [0, 600, 240], [0, 0, 1]], np.float32)
    dev_view = image_view(d_rgb, d_depth, K, d_mask)
    host_view = image_view(p_rgb, p_depth, K, p_mask)
    shard_begin, shard_count = shard_range(N_HYP, world, rank)
    per = -(-N_HYP // world)
    feats = torch.zeros((per, SCORE_FEATURE_DIM), dtype=torch.float32, device=dev)
    shard_poses = torch.zeros((per, 16), dtype=torch.float32, device=dev)
    last = {}

    def register(v, handle=None):
        hh = h if handle is None else handle
        if world == 1:
            last["pose"], _ = api.register(hh, v)
            return
        # Sharded register: local shard, NCCL all-gather of ScoreNet features
        # and refined poses, cross-hypothesis head + arg-max on every rank.
        api.shard_begin(hh, v, -1, N_HYP, shard_begin, shard_count, feats.data_ptr(), shard_poses.data_ptr())
        all_f = gather_shards(feats, N_HYP)
        all_p = gather_shards(shard_poses, N_HYP)
        torch.cuda.synchronize(dev)
        last["pose"], _ = api.shard_finish(hh, all_f.data_ptr(), all_p.data_ptr(), N_HYP)

    from fp_b200.dist_utils import barrier
    from fp_b200.dist_utils import max_over_ranks as _max

    def max_over_ranks(x: float) -> float:
        return _max(x, dev)

    sampler = ClockSampler(local, work / "clocks.csv")  # samples warm-up + timed region (GPU busy)
    for _ in range(args.warmup):
        register(dev_view)
    torch.cuda.synchronize()

    # Timed region: device-resident frame (stage profiling off; see below).
    stream = torch.cuda.current_stream(dev)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        register(dev_view)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    ms_per_step = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    value = N_HYP / (ms_per_step / 1000.0)  # one 252-hypothesis register per step, across all ranks
    pose_dev = last["pose"].copy()

    # End-to-end: pinned host buffers, H2D of the frame and D2H of the pose inside each step.
    e2e_steps = args.steps if args.e2e_steps is None else args.e2e_steps
    e2e_ms, pose_host = float("nan"), None
    if e2e_steps > 0:
        for _ in range(2):
            register(host_view)
        barrier()
        torch.cuda.synchronize()
        e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2.record(stream)
        for _ in range(e2e_steps):
            register(host_view)
        e3.record(stream)
        torch.cuda.synchronize()
        barrier()
        e2e_ms = max_over_ranks(e2.elapsed_time(e3) / e2e_steps)
        pose_host = last["pose"].copy()

    # Stage split, GEMM roofline and launch counts: CUDA events per stage on
    # eager registers (a replayed graph hides its launches from the host-side
    # profiler), on a second estimator without graph capture when the timed one
    # uses it. Same work per register.
    prof_steps = 2
    hp = h
    if args.graph:
        cfg_eager = api.default_config(n_hypotheses=N_HYP, n_refine_iters=N_ITERS, batch_size=N_HYP,
                                       tensorrt_precision=FP_PRECISION_FP16, capture_cuda_graph=False,
                                       max_image_width=W, max_image_height=H)
        hp = api.create(opts, cfg_eager)
    register(dev_view, hp)
    torch.cuda.synchronize()
    fpk.lib.fpk_profile_reset()
    fpk.lib.fpk_profile_enable(1)
    for _ in range(prof_steps):
        register(dev_view, hp)
    torch.cuda.synchronize()
    fpk.lib.fpk_profile_enable(0)
    ms_tot = (C.c_double * 5)()
    work_tot = (C.c_double * 5)()
    timed = (C.c_longlong * 5)()
    launches = (C.c_longlong * 5)()
    fpk.lib.fpk_profile_read(ms_tot, work_tot, timed, launches)
    if hp != h:
        api.destroy(hp)
    launches_per_register = sum(launches[i] for i in range(5)) / prof_steps

    # Track rate on the same estimator (B=1, 2 iterations), device-resident frame.
    track_view = image_view(d_rgb, d_depth, K)
    track_hz = None
    if args.track_frames > 0:
        for _ in range(5):
            api.track(h, track_view)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.track_frames):
            api.track(h, track_view)
        torch.cuda.synchronize()
        track_hz = args.track_frames / (time.perf_counter() - t0)
    api.destroy(h)

    if rank == 0:
        pk = peaks()
        gemm_ms, gemm_flops, gemm_n = ms_tot[0], work_tot[0], timed[0]
        achieved = gemm_flops / (gemm_ms / 1000.0) / 1e12 if gemm_ms > 0 else None
        render_ms, render_bytes = ms_tot[1], work_tot[1]
        cpu_base = None
        if not args.no_cpu_baseline and world == 1:
            t = cpu_register_sample(args.cpu_sample, mesh, rgb, depth, mask, refine, score)
            cpu_base = {"value": args.cpu_sample / t, "unit": "hyp/s", "cores": os.cpu_count() or 1,
                        "kind": "port",
                        "sample": f"{args.cpu_sample} hypotheses x (preprocess + 5 refine + 1 score pass) "
                                  "on the host: reference CPU preprocessDepth, CPU oracle render/pack/pose, "
                                  "torch fp32 networks"}
        line = {
            "metric": METRIC, "value": value, "unit": "hyp/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded scene; random-init weights)",
            "config": {"workload": WORKLOAD, "global_batch": N_HYP, "register_ms": ms_per_step,
                       "l2": "not flushed: each register streams ~2.5 GB of activations (> 126 MB L2)",
                       "cuda_graph": bool(args.graph),
                       "parallelism": ("single GPU" if world == 1 else
                                       f"hypothesis shards x{world} ({N_HYP // world}-{per} per GPU), NCCL all-gather "
                                       "of ScoreNet features + refined poses, cross-hypothesis head on every rank")},
            "e2e": {"value": N_HYP / (e2e_ms / 1000.0) if e2e_steps > 0 else None, "unit": "hyp/s",
                    "h2d_bytes_per_step": int(rgb.nbytes + depth.nbytes + mask.nbytes),
                    "d2h_bytes_per_step": 72, "register_ms": e2e_ms},
            "roofline": {"kernel": "gemmKernel (tcgen05 implicit-GEMM conv/linear)", "bound": "tensor",
                         "achieved": achieved, "peak": pk["bf16"], "unit": "TFLOP/s",
                         "frac": (achieved / pk["bf16"]) if achieved else None, "peak_note": pk["note"],
                         "traffic": GEMM_DRAM_BYTES_PER_TFLOP * (gemm_flops / 1e12) / max(1, gemm_n),
                         "traffic_note": "DRAM bytes per launch (read + write) from one ncu capture of whole "
                                         "register calls (profiles/gemm_dram_traffic_register.md), scaled by the "
                                         "launch's average work",
                         "launches_timed": gemm_n, "gemm_ms_per_step": gemm_ms / prof_steps,
                         "gemm_tflop_per_step": gemm_flops / prof_steps / 1e12,
                         "measured_on": f"{prof_steps} eager registers (CUDA events per GEMM launch)"},
            "render_pack": {"ms_per_step": render_ms / prof_steps,
                            "achieved_gbs": render_bytes / (render_ms / 1000.0) / 1e9 if render_ms > 0 else None,
                            "peak_gbs": pk["hbm"]},
            "stage_ms_per_step": {k: ms_tot[i] / prof_steps for i, k in
                                  enumerate(["gemm", "render_pack", "attention", "other", "preprocess"])},
            # Our kernels per register (counted on the eager profiling registers) x
            # timed steps; with graph capture the refinement passes replay them.
            "gpu_launches": int(round(launches_per_register * args.steps)),
            "track_hz": track_hz,
            "clocks": clocks,
            "cpu_baseline": cpu_base,
            "pose_host_equals_device": None if pose_host is None else bool(np.array_equal(pose_dev, pose_host)),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
