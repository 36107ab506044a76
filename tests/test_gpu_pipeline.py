"""GPU parity of the pipeline kernels (fpk_* C ABI) against
  (a) the reference's own CUDA kernels compiled from source (oracle/_ref/libfpref_gpu.so), and
  (b) the CPU oracle (oracle/liboracle.so).

Bars (from the path's parity contract): integer/index outputs bit-exact
(triangle ids may differ only on shared-edge tie pixels, <= 1e-4 of pixels);
xyz/depth within 1e-5 relative; everything else bit-exact against the
reference build where the arithmetic is the same expression.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle_lib import REF_GPU_SO, RefGpu
from scene_util import hypotheses, make_scene

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DEV = "cuda"


def t(a, dtype=None):
    x = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        x = x.to(dtype)
    return x.to(DEV)


def k_struct(scene):
    from fp_b200.kernels import Intrinsics

    return Intrinsics(*[float(v) for v in scene.k4])


def mesh_struct(scene, keep):
    from fp_b200.kernels import Mesh

    v = t(scene.verts)
    n = t(scene.normals)
    c = t(scene.colors_f)
    f = t(scene.faces.astype(np.int32))
    keep += [v, n, c, f]
    return Mesh(v.data_ptr(), n.data_ptr(), c.data_ptr(), None, None, f.data_ptr(),
                v.shape[0], f.shape[0], 0, 0)


def tf32_rna(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest TF32 (10 mantissa bits), ties away from zero."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    mag = u & np.uint32(0x7FFFFFFF)
    r = (u & np.uint32(0x80000000)) | ((mag + np.uint32(0x1000)) & np.uint32(0xFFFFE000))
    return np.where(mag < 0x7F800000, r, u).view(np.float32)


def cfg_from(oracle, params):
    return oracle.config(**{name: getattr(params, name) for name, _ in params._fields_})


@pytest.fixture(scope="module")
def refgpu():
    if not REF_GPU_SO.is_file():
        pytest.skip("reference GPU build (oracle/_ref) not present")
    return RefGpu()


def run_preprocess(fpk, scene, params, with_mask=True):
    h, w = scene.depth.shape
    d = t(scene.depth)
    m = t(scene.mask) if with_mask else None
    filt = torch.empty((h, w), device=DEV)
    ero = torch.empty((h, w), device=DEV)
    xyz = torch.empty((h, w, 3), device=DEV)
    stats = torch.empty(8 + 65536, dtype=torch.int32, device=DEV)
    fpk.preprocess(d.data_ptr(), m.data_ptr() if m is not None else 0, w, h, k_struct(scene),
                   params, filt.data_ptr(), ero.data_ptr(), xyz.data_ptr(), stats.data_ptr())
    torch.cuda.synchronize()
    return filt, ero, xyz, stats


@pytest.mark.parametrize("seed,size", [(0, (640, 480)), (3, (1280, 720)), (5, (97, 61))])
def test_preprocess_matches_reference_gpu(fpk, oracle, refgpu, seed, size):
    w, h = size
    rng = np.random.default_rng(seed)
    scene = make_scene(oracle, "ellipsoid_small", seed=seed)
    # Arbitrary-size frame: tile the scene's depth and add NaN / out-of-range values.
    depth = np.resize(scene.depth, (h, w)).astype(np.float32)
    depth[rng.random((h, w)) < 0.01] = np.nan
    depth[rng.random((h, w)) < 0.01] = 150.0
    mask = (rng.random((h, w)) < 0.3).astype(np.uint8) * (depth > 0)
    scene.depth, scene.mask = depth, mask.astype(np.uint8)
    scene.rgb = np.resize(scene.rgb, (h, w, 3))
    params = fpk.default_params()
    filt, ero, xyz, stats = run_preprocess(fpk, scene, params)
    rots = oracle.rotation_grid()
    ref = refgpu.preprocess(scene.rgb, depth, scene.mask, scene.k4, cfg_from(oracle, params), rots)
    np.testing.assert_array_equal(ero.cpu().numpy(), ref["eroded"])
    np.testing.assert_array_equal(filt.cpu().numpy(), ref["filtered"])
    np.testing.assert_array_equal(xyz.cpu().numpy(), ref["xyz"])
    r = t(rots)
    t0 = torch.empty(3, device=DEV)
    poses = torch.empty((rots.shape[0], 16), device=DEV)
    fpk.seed_poses(stats.data_ptr(), r.data_ptr(), rots.shape[0], k_struct(scene), params,
                   t0.data_ptr(), poses.data_ptr())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(t0.cpu().numpy(), ref["t0"])
    np.testing.assert_array_equal(poses.cpu().numpy(), ref["seeded"])


def test_preprocess_matches_oracle(fpk, oracle):
    scene = make_scene(oracle, "ellipsoid_small", seed=1)
    params = fpk.default_params()
    filt, ero, xyz, stats = run_preprocess(fpk, scene, params)
    cfg = cfg_from(oracle, params)
    o_ero = oracle.erode(scene.depth, cfg)
    o_fil = oracle.bilateral(o_ero, cfg)
    np.testing.assert_array_equal(ero.cpu().numpy(), o_ero)
    np.testing.assert_allclose(filt.cpu().numpy(), o_fil, rtol=1e-5, atol=0)
    o_xyz = oracle.depth_to_xyz(o_fil, scene.k4, cfg)
    np.testing.assert_allclose(xyz.cpu().numpy(), o_xyz, rtol=1e-5, atol=1e-7)
    o_t = oracle.initial_translation(o_fil, scene.mask, scene.k4, cfg)
    t0 = torch.empty(3, device=DEV)
    eye = t(np.eye(3, dtype=np.float32).reshape(1, 9))
    fpk.seed_poses(stats.data_ptr(), eye.data_ptr(), 0, k_struct(scene), params, t0.data_ptr(), 0)
    torch.cuda.synchronize()
    np.testing.assert_allclose(t0.cpu().numpy(), o_t, rtol=1e-5)


def test_translation_empty_mask(fpk, oracle):
    scene = make_scene(oracle, "ellipsoid_small", seed=2)
    scene.mask[:] = 0
    params = fpk.default_params()
    _, _, _, stats = run_preprocess(fpk, scene, params)
    t0 = torch.full((3,), 7.0, device=DEV)
    eye = t(np.eye(3, dtype=np.float32).reshape(1, 9))
    fpk.seed_poses(stats.data_ptr(), eye.data_ptr(), 0, k_struct(scene), params, t0.data_ptr(), 0)
    torch.cuda.synchronize()
    assert t0.cpu().numpy().tolist() == [0.0, 0.0, 0.0]


def render_case(fpk, oracle, kind, n, seed, size=(640, 480), holes=0.05):
    scene = make_scene(oracle, kind, seed=seed, width=size[0], height=size[1], holes=holes)
    poses = hypotheses(oracle, scene, n, seed=seed)
    params = fpk.default_params()
    keep = []
    mesh = mesh_struct(scene, keep)
    P = t(poses)
    boxes = torch.empty((n, 4), device=DEV)
    fpk.crop_boxes(P.data_ptr(), n, k_struct(scene), scene.diameter, params, boxes.data_ptr())
    rgb = torch.empty((n, 160, 160, 3), device=DEV)
    xyz = torch.empty((n, 160, 160, 3), device=DEV)
    tri = torch.empty((n, 160, 160), dtype=torch.int32, device=DEV)
    fpk.render(mesh, P.data_ptr(), boxes.data_ptr(), n, k_struct(scene), params, rgb.data_ptr(),
               xyz.data_ptr(), tri.data_ptr())
    torch.cuda.synchronize()
    return scene, poses, params, dict(boxes=boxes.cpu().numpy(), rgb=rgb.cpu().numpy(),
                                      xyz=xyz.cpu().numpy(), tri=tri.cpu().numpy()), keep


@pytest.mark.parametrize("kind,n", [("cube", 4), ("ellipsoid", 6), ("sphere50k", 3)])
def test_render_matches_reference_gpu(fpk, oracle, refgpu, kind, n):
    scene, poses, params, out, _ = render_case(fpk, oracle, kind, n, seed=11)
    ref = refgpu.render_pass(scene.verts, scene.normals, scene.colors_u8, scene.faces,
                             scene.diameter, poses, scene.rgb, scene.depth, scene.k4,
                             cfg_from(oracle, params), 0.001)
    np.testing.assert_array_equal(out["boxes"], ref["boxes"])
    ref_tri = ref["rast"][..., 3].astype(np.int32)
    mism = (out["tri"] != ref_tri)
    assert mism.mean() <= 1e-4, f"triangle-id mismatch fraction {mism.mean():.2e}"
    same = ~np.flip(mism, axis=1)  # rgb/xyz rows are top-down
    assert (ref_tri > 0).mean() > 0.01, "scene rendered nothing"
    np.testing.assert_allclose(out["xyz"][same], ref["xyz"][same], rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(out["rgb"][same], ref["rgb"][same], rtol=1e-5, atol=1e-6)


# The configurations the benchmark runs: 252 hypotheses take one row band per
# crop, 96 take two (64 <= n < 128), fewer than 64 take eight. The 250k-triangle
# mesh is mostly sub-pixel triangles at 1280x720; the
# triangle soup overflows the per-CTA list of shared large triangles.
@pytest.mark.parametrize("kind,n,size", [("sphere50k", 252, (640, 480)), ("sphere50k", 96, (640, 480)),
                                         ("dense250k", 252, (1280, 720)), ("dense250k", 21, (1280, 720)),
                                         ("bigtris", 252, (640, 480)), ("bigtris", 4, (640, 480))])
def test_render_matches_reference_gpu_at_scale(fpk, oracle, refgpu, kind, n, size):
    scene, poses, params, out, _ = render_case(fpk, oracle, kind, n, seed=13, size=size, holes=0.2)
    ref = refgpu.render_pass(scene.verts, scene.normals, scene.colors_u8, scene.faces,
                             scene.diameter, poses, scene.rgb, scene.depth, scene.k4,
                             cfg_from(oracle, params), 0.001)
    np.testing.assert_array_equal(out["boxes"], ref["boxes"])
    ref_tri = ref["rast"][..., 3].astype(np.int32)
    mism = out["tri"] != ref_tri
    covered = (ref_tri > 0).mean()
    print(f"{kind} n={n} {size}: coverage {covered:.3f}, triangle-id mismatch {mism.mean():.2e}")
    assert covered > 0.01, "scene rendered nothing"
    assert mism.mean() <= 1e-4, f"triangle-id mismatch fraction {mism.mean():.2e}"
    same = ~np.flip(mism, axis=1)
    np.testing.assert_allclose(out["xyz"][same], ref["xyz"][same], rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(out["rgb"][same], ref["rgb"][same], rtol=1e-5, atol=1e-6)


def test_fused_render_pack_matches_reference_at_bench_batch(fpk, oracle, refgpu):
    """The benchmark's pass: 252 hypotheses of the 50k-triangle mesh packed
    straight into the fp16 stem layout, against the reference's render +
    prepareNetworkInputs (NCHW fp32) rounded to fp16, on non-tie pixels."""
    from fp_b200.kernels import FPK_DTYPE_F16
    from kp8_util import Planar

    n = 252
    scene, poses, params, out, keep = render_case(fpk, oracle, "sphere50k", n, seed=17)
    h, w = scene.depth.shape
    ref = refgpu.render_pass(scene.verts, scene.normals, scene.colors_u8, scene.faces,
                             scene.diameter, poses, scene.rgb, scene.depth, scene.k4,
                             cfg_from(oracle, params), 0.001)
    filt, _, _, _ = run_preprocess(fpk, scene, params, with_mask=False)
    rgb = t(scene.rgb)
    P = t(poses)
    mesh = mesh_struct(scene, keep)
    net = Planar(2 * n * 83 * 83, 32, torch.float16)
    boxes = torch.empty((n, 4), device=DEV)
    fpk.render_pack(mesh, P.data_ptr(), n, rgb.data_ptr(), filt.data_ptr(), w, h, k_struct(scene), params,
                    scene.diameter, 0.001, FPK_DTYPE_F16, net.base, net.plane_stride, boxes.data_ptr())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(boxes.cpu().numpy(), ref["boxes"])
    g = net.get().float().cpu().numpy().reshape(2 * n, 83, 83, 32)
    ys, xs = np.meshgrid(np.arange(160), np.arange(160), indexing="ij")
    gy, gx = (ys + 3) // 2, (xs + 3) // 2
    sub = ((ys + 3) % 2) * 2 + ((xs + 3) % 2)
    tie = np.flip(out["tri"] != ref["rast"][..., 3].astype(np.int32), axis=1)  # top-down rows
    assert tie.mean() <= 1e-4
    for c in range(6):
        got_r, got_o = g[:n, gy, gx, sub * 8 + c], g[n:, gy, gx, sub * 8 + c]
        want_r = torch.from_numpy(ref["net_r"][:, c]).half().float().numpy()
        want_o = torch.from_numpy(ref["net_o"][:, c]).half().float().numpy()
        np.testing.assert_array_equal(got_o, want_o)  # observed: same frame taps
        d = np.abs(got_r - want_r)[~tie]
        # rendered values agree to 1e-5 relative in fp32; one fp16 rounding step apart at most
        assert np.all(d <= np.abs(want_r[~tie]) * 2.0 ** -10 + 1e-6), f"channel {c}: max diff {d.max():.3e}"


@pytest.mark.parametrize("kind,n", [("cube", 2), ("ellipsoid", 3)])
def test_render_matches_oracle(fpk, oracle, kind, n):
    scene, poses, params, out, _ = render_case(fpk, oracle, kind, n, seed=5)
    cfg = cfg_from(oracle, params)
    o_boxes = oracle.crop_boxes(poses, scene.k4, scene.diameter, cfg)
    np.testing.assert_array_equal(out["boxes"], o_boxes)
    o_rgb, o_xyz, o_rast = oracle.render(scene.verts, scene.normals, scene.colors_f, scene.faces,
                                         poses, o_boxes, scene.k4, cfg)
    mism = out["tri"] != o_rast[..., 3].astype(np.int32)
    # The CPU oracle has no FMA contraction: allow edge pixels to differ.
    assert mism.mean() <= 2e-3, f"triangle-id mismatch fraction {mism.mean():.2e}"
    same = ~np.flip(mism, axis=1)
    # Sliver triangles amplify the FMA-vs-no-FMA rounding in the barycentrics:
    # bound the outlier fraction, and every element loosely.
    for got, want in ((out["xyz"][same], o_xyz[same]), (out["rgb"][same], o_rgb[same])):
        err = np.abs(got - want)
        assert np.mean(err > 1e-5 + 1e-4 * np.abs(want)) <= 1e-3
        assert err.max() <= 1e-2


def test_pack_and_fused_render_pack(fpk, oracle, refgpu):
    scene, poses, params, out, keep = render_case(fpk, oracle, "ellipsoid", 4, seed=21)
    n = poses.shape[0]
    h, w = scene.depth.shape
    ref = refgpu.render_pass(scene.verts, scene.normals, scene.colors_u8, scene.faces,
                             scene.diameter, poses, scene.rgb, scene.depth, scene.k4,
                             cfg_from(oracle, params), 0.001)
    filt, _, _, _ = run_preprocess(fpk, scene, params, with_mask=False)
    rgb = t(scene.rgb)
    P = t(poses)
    boxes = t(out["boxes"])
    net_r = torch.empty((n, 6, 160, 160), device=DEV)
    net_o = torch.empty((n, 6, 160, 160), device=DEV)
    rend_rgb, rend_xyz = t(out["rgb"]), t(out["xyz"])  # keep alive until the kernel ran
    fpk.pack(rgb.data_ptr(), filt.data_ptr(), w, h, k_struct(scene), params,
             rend_rgb.data_ptr(), rend_xyz.data_ptr(), P.data_ptr(), boxes.data_ptr(), n,
             scene.diameter, 0.001, net_r.data_ptr(), net_o.data_ptr())
    torch.cuda.synchronize()
    nr, no = net_r.cpu().numpy(), net_o.cpu().numpy()
    np.testing.assert_array_equal(no, ref["net_o"])
    tri_same = (out["tri"] == ref["rast"][..., 3].astype(np.int32))
    same = np.flip(tri_same, axis=1)[:, None].repeat(6, 1)
    np.testing.assert_allclose(nr[same], ref["net_r"][same], rtol=1e-5, atol=1e-6)

    # Fused render+pack into the stem's space-to-depth layout: same values.
    from fp_b200.kernels import FPK_DTYPE_BF16, FPK_DTYPE_F16, FPK_DTYPE_F32

    mesh = mesh_struct(scene, keep)
    from kp8_util import Planar

    for dtype, tdt in ((FPK_DTYPE_F32, torch.float32), (FPK_DTYPE_F16, torch.float16),
                       (FPK_DTYPE_BF16, torch.bfloat16)):
        net = Planar(2 * n * 83 * 83, 32, tdt)
        b2 = torch.empty((n, 4), device=DEV)
        fpk.render_pack(mesh, P.data_ptr(), n, rgb.data_ptr(), filt.data_ptr(), w, h,
                        k_struct(scene), params, scene.diameter, 0.001, dtype, net.base,
                        net.plane_stride, b2.data_ptr())
        torch.cuda.synchronize()
        np.testing.assert_array_equal(b2.cpu().numpy(), out["boxes"])
        g = net.get().float().cpu().numpy().reshape(2 * n, 83, 83, 32)
        # Undo the space-to-depth layout: crop pixel (y, x) lives at cell
        # ((y+3)//2, (x+3)//2), sub-position ((y+3)%2, (x+3)%2), channels 0..5.
        ys, xs = np.meshgrid(np.arange(160), np.arange(160), indexing="ij")
        gy, gx = (ys + 3) // 2, (xs + 3) // 2
        sub = ((ys + 3) % 2) * 2 + ((xs + 3) % 2)
        full = np.concatenate([nr, no], 0)  # [2n,6,H,W]
        for c in range(6):
            got = g[:, gy, gx, sub * 8 + c]
            want = torch.from_numpy(full[:, c]).to(tdt).float().numpy()
            if tdt == torch.float32:
                want = tf32_rna(want)  # fp32 stem inputs are rounded to TF32 (the seam loader does the same)
            np.testing.assert_array_equal(got, want)
        # Border cells, the two padding channels and the guard rows stay zero.
        assert np.all(g[:, 0] == 0) and np.all(g[..., 6::8] == 0) and np.all(g[..., 7::8] == 0)
        assert torch.count_nonzero(net.t[:, :256]) == 0


def test_apply_deltas_and_select_best(fpk, oracle, refgpu):
    rng = np.random.default_rng(4)
    rots = oracle.rotation_grid()
    poses = oracle.seed_poses(rots, np.array([0.01, -0.02, 0.7], np.float32))
    n = poses.shape[0]
    dt = rng.normal(0, 0.3, size=(n, 3)).astype(np.float32)
    dr = rng.normal(0, 1.0, size=(n, 3)).astype(np.float32)
    dr[0] = 0.0  # theta < 1e-6 branch
    params = fpk.default_params()
    P = t(poses)
    dt_d, dr_d = t(dt), t(dr)  # keep alive until the kernel ran
    fpk.apply_deltas(P.data_ptr(), dt_d.data_ptr(), dr_d.data_ptr(), n, 0.12, params)
    torch.cuda.synchronize()
    got = P.cpu().numpy()
    ref = refgpu.apply_deltas(poses, dt, dr, 0.12, params.rotation_normalizer_rad)
    np.testing.assert_array_equal(got, ref)
    orc = oracle.apply_deltas(poses, dt, dr, 0.12, cfg_from(oracle, params))
    np.testing.assert_allclose(got, orc, rtol=1e-5, atol=2e-7)
    center = np.array([0.003, -0.01, 0.02], np.float32)
    for case in range(4):
        scores = rng.normal(size=n).astype(np.float32)
        if case == 1:
            scores[[7, 100, 200]] = scores.max() + 1.0  # ties: first index wins
        if case == 2:
            scores[[3, 9]] = np.nan
        if case == 3:
            scores[0] = np.nan  # NaN at 0 is never replaced
        res = torch.empty(18, device=DEV)
        sc_d = t(scores)
        fpk.select_best(P.data_ptr(), sc_d.data_ptr(), n, center, res.data_ptr())
        torch.cuda.synchronize()
        r = res.cpu().numpy()
        idx = int(r[17:18].view(np.int32)[0])
        ref_pose, ref_score, ref_idx = refgpu.select_best(got, scores, center)
        assert idx == ref_idx
        np.testing.assert_array_equal(r[:16], ref_pose)
        assert (np.isnan(r[16]) and np.isnan(ref_score)) or r[16] == ref_score
