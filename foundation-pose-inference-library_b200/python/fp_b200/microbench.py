"""Single-kernel drivers for profiling and tuning (one process, one GPU).

  python -m fp_b200.microbench gemm   --batch 128 [--cin 256 --cout 256 --grid 41 --iters 20]
  python -m fp_b200.microbench render --batch 252 [--faces 50000]
  python -m fp_b200.microbench attention --batch 252

Each prints one JSON line with the CUDA-event time per launch and the
achieved rate against the layer's algorithmic work (un-padded FLOPs for the
GEMM and attention; mesh + frame + written network input bytes for render).
Sizes default to one RefineNet layer of the register workload; inputs are
random (GEMM/attention) or a synthetic scene (render).
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import math
import sys
from pathlib import Path

import numpy as np


def _torch():
    import torch

    assert torch.cuda.is_available(), "microbench needs a CUDA GPU"
    return torch


class Planar:
    """KP8 activation buffer with zero guard rows (see include/fpk.h)."""

    def __init__(self, torch, rows: int, channels: int, dtype):
        per = 8
        total = (256 + rows + 512 + 15) // 16 * 16
        self.t = torch.zeros((channels // per, total, per), dtype=dtype, device="cuda")
        self.base = self.t.data_ptr() + 256 * 16
        self.stride = total * 16
        self.rows = rows


def time_fn(torch, fn, iters: int, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def bench_gemm(args) -> dict:
    torch = _torch()
    from fp_b200.kernels import FPK_DST_SAME, FPK_DTYPE_BF16, FPK_DTYPE_F16, FpkLibrary, GemmDesc, gemm

    fpk = FpkLibrary()
    fpk.lib.fpk_gemm_set_cta_pairs(args.pairs)
    dt = torch.float16 if args.dtype == "f16" else torch.bfloat16
    g = args.grid
    valid = g - 1
    rows = args.batch * g * g
    a = Planar(torch, rows, args.cin, dt)
    a.t.uniform_(-1, 1)
    out = Planar(torch, rows, args.cout, dt)
    taps = [(ky - 1) * g + (kx - 1) for ky in range(3) for kx in range(3)] if args.taps == 9 else [0]
    w = (torch.randn(args.cout, len(taps) * args.cin, device="cuda") / math.sqrt(len(taps) * args.cin)).to(dt)
    bias = torch.zeros(args.cout, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    d = GemmDesc()
    d.a, d.a_plane_stride, d.rows, d.cin, d.taps = a.base, a.stride, rows, args.cin, len(taps)
    for i, o in enumerate(taps):
        d.tap_off[i] = o
    d.w, d.cout, d.bias = w.data_ptr(), args.cout, bias.data_ptr()
    d.relu, d.dst, d.dst_plane_stride, d.dst_mode = 1, out.base, out.stride, FPK_DST_SAME
    d.img_rows, d.grid_w, d.valid_h, d.valid_w = g * g, g, valid, valid
    d.img_mod, d.dtype, d.error_flag = 1, FPK_DTYPE_F16 if args.dtype == "f16" else FPK_DTYPE_BF16, err.data_ptr()
    ms = time_fn(torch, lambda: gemm(fpk, d), args.iters)
    flops = 2.0 * args.batch * valid * valid * args.cout * len(taps) * args.cin
    return {"kernel": "gemmKernel", "cta_pairs": args.pairs, "batch": args.batch, "cin": args.cin, "cout": args.cout,
            "grid": g, "taps": len(taps), "ms": ms, "tflops": flops / ms / 1e9,
            "hbm_bytes": (rows * (args.cin + args.cout)) * 2, "error_flag": int(err.item())}


def bench_render(args) -> dict:
    torch = _torch()
    from fp_b200 import synthetic as syn
    from fp_b200.kernels import FPK_DTYPE_F16, FpkLibrary, Intrinsics, Mesh

    fpk = FpkLibrary()
    n_lat = int(round(args.faces / 400)) + 2
    mesh = syn.displaced_sphere(1, n_lat=n_lat, n_lon=200)
    normals = syn.vertex_normals(mesh.vertices, mesh.faces)
    rng = np.random.default_rng(0)
    gt = syn.random_pose(rng, dist=(0.65, 0.75), lateral=0.03)
    rgb, depth = syn.render_frame_gpu(fpk, mesh, normals, gt, syn.K_640, 640, 480)
    dev = "cuda"
    v = torch.from_numpy(mesh.vertices).to(dev)
    nr = torch.from_numpy(normals).to(dev)
    col = torch.from_numpy(mesh.colors.astype(np.float32) / np.float32(255.0)).to(dev)
    f = torch.from_numpy(mesh.faces).to(dev)
    m = Mesh(v.data_ptr(), nr.data_ptr(), col.data_ptr(), None, None, f.data_ptr(), v.shape[0],
             f.shape[0], 0, 0)
    poses = np.repeat(gt.reshape(1, 16), args.batch, 0).astype(np.float32)
    rots = np.stack([syn.rotation_matrix(rng) for _ in range(args.batch)]).astype(np.float32)
    poses.reshape(-1, 4, 4)[:, :3, :3] = rots
    P = torch.from_numpy(poses).to(dev)
    d_rgb, d_depth = torch.from_numpy(rgb).to(dev), torch.from_numpy(depth).to(dev)
    params = fpk.default_params()
    k = Intrinsics(600.0, 600.0, 320.0, 240.0)
    net = Planar(torch, 2 * args.batch * 83 * 83, 32, torch.float16)
    boxes = torch.empty((args.batch, 4), device=dev)
    diam = float(np.linalg.norm(mesh.vertices.max(0) - mesh.vertices.min(0)))

    ws_bytes = fpk.render_workspace_bytes(args.batch, v.shape[0], params)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)

    def run():
        fpk.render_pack(m, P.data_ptr(), args.batch, d_rgb.data_ptr(), d_depth.data_ptr(), 640, 480, k,
                        params, diam, 0.001, FPK_DTYPE_F16, net.base, net.stride, boxes.data_ptr(),
                        workspace=ws.data_ptr(), workspace_bytes=ws_bytes)

    ms = time_fn(torch, run, args.iters)
    px = args.batch * 160 * 160
    nbytes = v.shape[0] * 36 + f.shape[0] * 12 + 640 * 480 * 7 + px * 12 * 2
    return {"kernel": "render+pack (vertex, raster, shade kernels), fp16", "batch": args.batch, "faces": int(f.shape[0]), "ms": ms,
            "gbs": nbytes / ms / 1e6, "tris_per_s": args.batch * f.shape[0] / ms * 1e3}


def bench_attention(args) -> dict:
    torch = _torch()
    from fp_b200.kernels import FpkLibrary, Networks
    from fp_b200.weights import make_default_packs

    import tempfile

    fpk = FpkLibrary()
    d = Path(tempfile.mkdtemp())
    refine, score = make_default_packs(d, seed=0)
    netw = Networks(fpk, refine, score, 2, args.batch)
    A = torch.rand(args.batch, 6, 160, 160, device="cuda")
    B = torch.rand(args.batch, 6, 160, 160, device="cuda")
    t = torch.zeros(args.batch, 3, device="cuda")
    r = torch.zeros(args.batch, 3, device="cuda")
    ms = time_fn(torch, lambda: netw.refine(A.data_ptr(), B.data_ptr(), args.batch, t.data_ptr(), r.data_ptr()),
                 args.iters)
    return {"kernel": "RefineNet forward", "batch": args.batch, "ms": ms}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["gemm", "render", "attention"])
    ap.add_argument("--batch", type=int, default=128)
    ap.add_argument("--cin", type=int, default=256)
    ap.add_argument("--cout", type=int, default=256)
    ap.add_argument("--grid", type=int, default=41)
    ap.add_argument("--taps", type=int, default=9, choices=[1, 9])
    ap.add_argument("--faces", type=int, default=50000)
    ap.add_argument("--dtype", default="f16", choices=["f16", "bf16"])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--pairs", type=int, default=1, choices=[0, 1],
                    help="gemm: allow CTA-pair (cta_group::2) tiles (1, default) or single-CTA tiles only (0)")
    args = ap.parse_args()
    fn = {"gemm": bench_gemm, "render": bench_render, "attention": bench_attention}[args.what]
    print(json.dumps(fn(args)), flush=True)


if __name__ == "__main__":
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    main()
