"""ctypes bindings for the test oracle (oracle/liboracle.so) and, when present,
the reference builds in oracle/_ref/. Test infrastructure only."""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
ORACLE_SO = ROOT / "oracle" / "liboracle.so"
REF_CPU_SO = ROOT / "oracle" / "_ref" / "libfpref_cpu.so"
REF_GPU_SO = ROOT / "oracle" / "_ref" / "libfpref_gpu.so"


class Cfg(C.Structure):
    _fields_ = [
        ("depth_min", C.c_float), ("depth_max", C.c_float),
        ("erosion_radius", C.c_int), ("bilateral_radius", C.c_int),
        ("depth_diff_threshold", C.c_float), ("erosion_ratio_threshold", C.c_float),
        ("bilateral_sigma_d", C.c_float), ("bilateral_sigma_r", C.c_float),
        ("crop_ratio", C.c_float),
        ("input_width", C.c_int), ("input_height", C.c_int),
        ("rotation_normalizer_rad", C.c_float), ("znear", C.c_float), ("zfar", C.c_float),
        ("ambient_weight", C.c_float), ("diffuse_weight", C.c_float),
    ]


def ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, np.float32)


class Oracle:
    """The CPU restatement (fp_oracle.c)."""

    def __init__(self, path: Path = ORACLE_SO):
        if not path.is_file():
            raise FileNotFoundError(f"{path} not built (make -C oracle)")
        self.lib = C.CDLL(str(path))
        self.lib.fpo_rotation_grid.restype = C.c_int
        self.lib.fpo_select_best.restype = C.c_int

    def config(self, **overrides) -> Cfg:
        c = Cfg()
        self.lib.fpo_default_config(C.byref(c))
        for k, v in overrides.items():
            setattr(c, k, v)
        return c

    def rotation_grid(self) -> np.ndarray:
        out = np.zeros((512, 9), np.float32)
        n = self.lib.fpo_rotation_grid(ptr(out), 512)
        return out[:n].copy()

    def erode(self, depth, cfg):
        h, w = depth.shape
        out = np.zeros_like(depth, dtype=np.float32)
        self.lib.fpo_erode(ptr(f32(depth)), ptr(out), w, h, C.byref(cfg))
        return out

    def bilateral(self, depth, cfg):
        h, w = depth.shape
        out = np.zeros_like(depth, dtype=np.float32)
        self.lib.fpo_bilateral(ptr(f32(depth)), ptr(out), w, h, C.byref(cfg))
        return out

    def depth_to_xyz(self, depth, k4, cfg):
        h, w = depth.shape
        out = np.zeros((h, w, 3), np.float32)
        self.lib.fpo_depth_to_xyz(ptr(f32(depth)), ptr(out), w, h, ptr(f32(k4)), C.byref(cfg))
        return out

    def preprocess_cpu(self, depth, cfg):
        h, w = depth.shape
        out = np.zeros_like(depth, dtype=np.float32)
        self.lib.fpo_preprocess_cpu(ptr(f32(depth)), ptr(out), w, h, C.byref(cfg))
        return out

    def initial_translation(self, depth, mask, k4, cfg):
        h, w = depth.shape
        t = np.zeros(3, np.float32)
        self.lib.fpo_initial_translation(ptr(f32(depth)), ptr(np.ascontiguousarray(mask, np.uint8)),
                                         w, h, ptr(f32(k4)), C.byref(cfg), ptr(t))
        return t

    def guess_translation_cpu(self, depth, mask, k4, cfg):
        h, w = depth.shape
        t = np.zeros(3, np.float32)
        self.lib.fpo_guess_translation_cpu(ptr(f32(depth)), ptr(np.ascontiguousarray(mask, np.uint8)),
                                           w, h, ptr(f32(k4)), C.byref(cfg), ptr(t))
        return t

    def seed_poses(self, rots, t):
        n = rots.shape[0]
        out = np.zeros((n, 16), np.float32)
        self.lib.fpo_seed_poses(ptr(f32(rots)), ptr(f32(t)), n, ptr(out))
        return out

    def crop_boxes(self, poses, k4, diameter, cfg):
        n = poses.shape[0]
        out = np.zeros((n, 4), np.float32)
        self.lib.fpo_crop_boxes(ptr(f32(poses)), n, ptr(f32(k4)), C.c_float(diameter),
                                C.byref(cfg), ptr(out))
        return out

    def render(self, verts, normals, colors_f, faces, poses, boxes, k4, cfg):
        n = poses.shape[0]
        H, W = cfg.input_height, cfg.input_width
        rgb = np.zeros((n, H, W, 3), np.float32)
        xyz = np.zeros((n, H, W, 3), np.float32)
        rast = np.zeros((n, H, W, 4), np.float32)
        faces = np.ascontiguousarray(faces, np.int32)
        self.lib.fpo_render(ptr(f32(verts)), ptr(f32(normals)), ptr(f32(colors_f)), verts.shape[0],
                            ptr(faces), faces.shape[0], ptr(f32(poses)), ptr(f32(boxes)), n,
                            ptr(f32(k4)), C.byref(cfg), ptr(rgb), ptr(xyz), ptr(rast))
        return rgb, xyz, rast

    def pack(self, rgb_u8, xyz_map, rend_rgb, rend_xyz, poses, boxes, diameter, thr, cfg):
        h, w = xyz_map.shape[:2]
        n = poses.shape[0]
        H, W = cfg.input_height, cfg.input_width
        r = np.zeros((n, 6, H, W), np.float32)
        o = np.zeros((n, 6, H, W), np.float32)
        self.lib.fpo_pack(ptr(np.ascontiguousarray(rgb_u8, np.uint8)), ptr(f32(xyz_map)), w, h,
                          ptr(f32(rend_rgb)), ptr(f32(rend_xyz)), ptr(f32(poses)), ptr(f32(boxes)),
                          n, W, H, C.c_float(diameter), C.c_float(thr), ptr(r), ptr(o))
        return r, o

    def apply_deltas(self, poses, dt, dr, diameter, cfg):
        out = f32(poses).copy()
        self.lib.fpo_apply_deltas(ptr(out), ptr(f32(dt)), ptr(f32(dr)), out.shape[0],
                                  C.c_float(diameter), C.byref(cfg))
        return out

    def select_best(self, poses, scores, center):
        out = np.zeros(16, np.float32)
        sc = C.c_float(0)
        idx = self.lib.fpo_select_best(ptr(f32(poses)), ptr(f32(scores)), poses.shape[0],
                                       ptr(f32(center)), ptr(out), C.byref(sc))
        return out, sc.value, idx

    def vertex_normals(self, verts, faces):
        out = np.zeros((verts.shape[0], 3), np.float32)
        faces = np.ascontiguousarray(faces, np.int32)
        self.lib.fpo_vertex_normals(ptr(f32(verts)), verts.shape[0], ptr(faces), faces.shape[0],
                                    ptr(out))
        return out

    def mesh_center_diameter(self, verts, sample_points=10000):
        c = np.zeros(3, np.float32)
        d = C.c_float(0)
        centered = np.zeros_like(f32(verts))
        self.lib.fpo_mesh_center_diameter(ptr(f32(verts)), verts.shape[0], sample_points, ptr(c),
                                          C.byref(d), ptr(centered))
        return c, d.value, centered


class RefCpu:
    """The reference's own CPU functions (src/pipeline_utils.cpp, src/mesh.cpp)."""

    def __init__(self, path: Path = REF_CPU_SO):
        if not path.is_file():
            raise FileNotFoundError(str(path))
        self.path = path
        self.lib = C.CDLL(str(path))
        self.lib.refcpu_rotation_grid.restype = C.c_int
        self.lib.refcpu_preprocess_depth.restype = C.c_int
        self.lib.refcpu_load_mesh.restype = C.c_int

    def rotation_grid(self):
        out = np.zeros((512, 9), np.float32)
        n = self.lib.refcpu_rotation_grid(ptr(out), 512)
        return out[:n].copy()

    def preprocess_depth(self, depth):
        h, w = depth.shape
        out = np.zeros_like(depth, dtype=np.float32)
        assert self.lib.refcpu_preprocess_depth(ptr(f32(depth)), w, h, ptr(out)) == 0
        return out

    def depth_to_xyz(self, depth, k4):
        h, w = depth.shape
        out = np.zeros((h, w, 3), np.float32)
        self.lib.refcpu_depth_to_xyz(ptr(f32(depth)), w, h, ptr(f32(k4)), ptr(out))
        return out

    def guess_translation(self, depth, mask, k4):
        h, w = depth.shape
        t = np.zeros(3, np.float32)
        self.lib.refcpu_guess_translation(ptr(f32(depth)), ptr(np.ascontiguousarray(mask, np.uint8)),
                                          w, h, ptr(f32(k4)), ptr(t))
        return t

    def crop_boxes(self, poses, k4, diameter):
        out = np.zeros((poses.shape[0], 4), np.float32)
        self.lib.refcpu_crop_boxes(ptr(f32(poses)), poses.shape[0], ptr(f32(k4)),
                                   C.c_float(diameter), ptr(out))
        return out

    def apply_delta(self, pose, dt, dr, diameter):
        out = np.zeros(16, np.float32)
        self.lib.refcpu_apply_delta(ptr(f32(pose)), ptr(f32(dt)), ptr(f32(dr)),
                                    C.c_float(diameter), ptr(out))
        return out

    def load_mesh(self, path: str):
        """Reference loadMesh + preprocessMesh. Runs in a fresh interpreter that
        never imports numpy: the reference's iostream-based OBJ parser crashes
        when numpy's libstdc++ locale state shares the process."""
        import pickle
        import subprocess
        import sys

        script = (
            "import ctypes as C, pickle, sys\n"
            f"lib = C.CDLL({str(self.path)!r})\n"
            "nv, nf, d = C.c_int(0), C.c_int(0), C.c_float(0)\n"
            "c = (C.c_float * 3)(); err = C.create_string_buffer(512)\n"
            f"p = {str(path)!r}.encode()\n"
            "rc = lib.refcpu_load_mesh(p, C.byref(nv), C.byref(nf), None, None, None, None, c, C.byref(d), err, 512)\n"
            "if rc: sys.stdout.buffer.write(pickle.dumps(('err', err.value.decode()))); sys.exit(0)\n"
            "v = (C.c_float * (3 * nv.value))(); n = (C.c_float * (3 * nv.value))()\n"
            "col = (C.c_uint8 * (3 * nv.value))(); f = (C.c_uint32 * (3 * nf.value))()\n"
            "lib.refcpu_load_mesh(p, C.byref(nv), C.byref(nf), v, n, col, f, c, C.byref(d), err, 512)\n"
            "sys.stdout.buffer.write(pickle.dumps(('ok', bytes(v), bytes(n), bytes(col), bytes(f), bytes(c), d.value)))\n"
        )
        out = subprocess.run([sys.executable, "-c", script], capture_output=True, check=True).stdout
        res = pickle.loads(out)
        if res[0] != "ok":
            raise RuntimeError(res[1])
        _, v, n, col, f, c, diam = res
        return dict(vertices=np.frombuffer(v, np.float32).reshape(-1, 3).copy(),
                    normals=np.frombuffer(n, np.float32).reshape(-1, 3).copy(),
                    colors=np.frombuffer(col, np.uint8).reshape(-1, 3).copy(),
                    faces=np.frombuffer(f, np.uint32).reshape(-1, 3).copy(),
                    center=np.frombuffer(c, np.float32).copy(), diameter=diam)


class RefGpu:
    """The reference's own CUDA kernels (src/cuda_pipeline.cu, src/builtin_raster_renderer.cu)."""

    def __init__(self, path: Path = REF_GPU_SO):
        if not path.is_file():
            raise FileNotFoundError(str(path))
        self.lib = C.CDLL(str(path))
        self.lib.refgpu_last_error.restype = C.c_char_p

    def _ok(self, rc):
        if rc != 0:
            raise RuntimeError(self.lib.refgpu_last_error().decode())

    def preprocess(self, rgb, depth, mask, k4, cfg, rotations=None):
        h, w = depth.shape
        ero = np.zeros((h, w), np.float32)
        fil = np.zeros((h, w), np.float32)
        xyz = np.zeros((h, w, 3), np.float32)
        t0 = np.zeros(3, np.float32)
        n = 0 if rotations is None else rotations.shape[0]
        seeded = np.zeros((max(n, 1), 16), np.float32)
        self._ok(self.lib.refgpu_preprocess(ptr(np.ascontiguousarray(rgb, np.uint8)), ptr(f32(depth)),
                                            ptr(None if mask is None else np.ascontiguousarray(mask, np.uint8)),
                                            w, h, ptr(f32(k4)), C.byref(cfg),
                                            ptr(None if rotations is None else f32(rotations)), n,
                                            ptr(ero), ptr(fil), ptr(xyz), ptr(t0), ptr(seeded)))
        return dict(eroded=ero, filtered=fil, xyz=xyz, t0=t0, seeded=seeded[:n])

    def render_pass(self, verts, normals, colors_u8, faces, diameter, poses, rgb, depth, k4, cfg,
                    invalid_threshold):
        n = poses.shape[0]
        h, w = depth.shape
        H, W = cfg.input_height, cfg.input_width
        out = dict(boxes=np.zeros((n, 4), np.float32), rgb=np.zeros((n, H, W, 3), np.float32),
                   xyz=np.zeros((n, H, W, 3), np.float32), rast=np.zeros((n, H, W, 4), np.float32),
                   net_r=np.zeros((n, 6, H, W), np.float32), net_o=np.zeros((n, 6, H, W), np.float32))
        faces = np.ascontiguousarray(faces, np.int32)
        self._ok(self.lib.refgpu_render_pass(
            ptr(f32(verts)), ptr(f32(normals)), ptr(np.ascontiguousarray(colors_u8, np.uint8)),
            verts.shape[0], ptr(faces), faces.shape[0], C.c_float(diameter), ptr(f32(poses)), n,
            ptr(np.ascontiguousarray(rgb, np.uint8)), ptr(f32(depth)), w, h, ptr(f32(k4)),
            C.byref(cfg), C.c_float(invalid_threshold), ptr(out["boxes"]), ptr(out["rgb"]),
            ptr(out["xyz"]), ptr(out["rast"]), ptr(out["net_r"]), ptr(out["net_o"])))
        return out

    def apply_deltas(self, poses, dt, dr, diameter, rn):
        out = f32(poses).copy()
        self._ok(self.lib.refgpu_apply_deltas(ptr(out), ptr(f32(dt)), ptr(f32(dr)), out.shape[0],
                                              C.c_float(diameter), C.c_float(rn)))
        return out

    def select_best(self, poses, scores, center):
        pose = np.zeros(16, np.float32)
        sc = C.c_float(0)
        idx = C.c_int(0)
        self._ok(self.lib.refgpu_select_best(ptr(f32(poses)), ptr(f32(scores)), poses.shape[0],
                                             ptr(f32(center)), ptr(pose), C.byref(sc), C.byref(idx)))
        return pose, sc.value, idx.value
