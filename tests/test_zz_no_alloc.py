"""fpk_initial_translation_noalloc: the allocation-free entry point for callers
that may not allocate device memory (real-time loops, safety-reviewed
deployments, plugin hosts that own every buffer). Its scratch lives in device
arrays built into the library, so this test checks it against the regular
entry points (fpk_preprocess + fpk_seed_poses with caller-allocated scratch) on
two different frames in a row: the shared scratch must not carry anything from
one call into the next. Collected last so a failure here never hides another
test's result."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from scene_util import make_scene

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _bind(fpk):
    from fp_b200.kernels import Intrinsics, Params

    f = fpk.lib.fpk_initial_translation_noalloc
    f.restype = C.c_int
    f.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, Intrinsics, C.POINTER(Params), C.c_void_p,
                  C.c_void_p]
    return f


def _regular(fpk, depth, mask, k, params):
    h, w = depth.shape
    filt = torch.empty((h, w), device="cuda")
    stats = torch.empty(8 + 65536, dtype=torch.int32, device="cuda")
    t0 = torch.empty(3, device="cuda")
    fpk.preprocess(depth.data_ptr(), mask.data_ptr(), w, h, k, params, filt.data_ptr(), 0, 0,
                   stats.data_ptr())
    fpk.seed_poses(stats.data_ptr(), 0, 0, k, params, t0.data_ptr(), 0)
    torch.cuda.synchronize()
    return t0.cpu().numpy()


def test_noalloc_matches_regular_entry_points_twice(fpk, oracle):
    from fp_b200.kernels import Intrinsics

    fn = _bind(fpk)
    params = fpk.default_params()
    frames = []
    for seed, kind in ((2, "ellipsoid_small"), (9, "cube")):
        s = make_scene(oracle, kind, seed=seed)
        frames.append((torch.from_numpy(s.depth).cuda(), torch.from_numpy(s.mask).cuda(),
                       Intrinsics(*[float(v) for v in s.k4])))
    for depth, mask, k in frames:  # two calls in a row on different frames
        want = _regular(fpk, depth, mask, k, params)
        t0 = torch.full((3,), -1.0, device="cuda")
        h, w = depth.shape
        rc = fn(depth.data_ptr(), mask.data_ptr(), w, h, k, C.byref(params), t0.data_ptr(), None)
        assert rc == 0, fpk.lib.fpk_last_error().decode()
        torch.cuda.synchronize()
        got = t0.cpu().numpy()
        assert np.all(np.isfinite(got)) and got[2] > 0
        np.testing.assert_allclose(got, want, rtol=1e-6, atol=0)


def test_noalloc_rejects_oversize_frames(fpk):
    from fp_b200.kernels import Intrinsics

    fn = _bind(fpk)
    params = fpk.default_params()
    depth = torch.zeros(4, device="cuda")
    mask = torch.zeros(4, dtype=torch.uint8, device="cuda")
    t0 = torch.zeros(3, device="cuda")
    k = Intrinsics(600.0, 600.0, 320.0, 240.0)
    rc = fn(depth.data_ptr(), mask.data_ptr(), 1281, 720, k, C.byref(params), t0.data_ptr(), None)
    assert rc != 0 and "exceeds the built-in scratch" in fpk.lib.fpk_last_error().decode()
    rc = fn(depth.data_ptr(), None, 2, 2, k, C.byref(params), t0.data_ptr(), None)
    assert rc != 0 and "required" in fpk.lib.fpk_last_error().decode()
