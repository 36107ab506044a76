"""Seeded synthetic scenes standing in for BOP YCB-V (not available offline).

Meshes, poses and frame post-processing are numpy; frames are rendered on the
GPU with the library's own rasterizer (fpk_render with the crop box set to the
whole frame), so no oracle code is involved. Shapes follow the benchmark
configurations: 640x480 (or 1280x720) RGB-D, fx=fy=600 (900), per-vertex
colours, Gaussian depth noise and zeroed depth holes.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

K_640 = np.array([[600.0, 0.0, 320.0], [0.0, 600.0, 240.0], [0.0, 0.0, 1.0]], np.float32)
K_1280 = np.array([[900.0, 0.0, 640.0], [0.0, 900.0, 360.0], [0.0, 0.0, 1.0]], np.float32)


@dataclass
class MeshData:
    vertices: np.ndarray  # [V,3] float32 (metres)
    faces: np.ndarray     # [F,3] int32
    colors: np.ndarray    # [V,3] uint8

    @property
    def n_faces(self) -> int:
        return int(self.faces.shape[0])


def icosphere(subdivisions: int) -> tuple[np.ndarray, np.ndarray]:
    t = (1.0 + 5.0 ** 0.5) / 2.0
    v = [(-1, t, 0), (1, t, 0), (-1, -t, 0), (1, -t, 0), (0, -1, t), (0, 1, t), (0, -1, -t),
         (0, 1, -t), (t, 0, -1), (t, 0, 1), (-t, 0, -1), (-t, 0, 1)]
    f = [(0, 11, 5), (0, 5, 1), (0, 1, 7), (0, 7, 10), (0, 10, 11), (1, 5, 9), (5, 11, 4),
         (11, 10, 2), (10, 7, 6), (7, 1, 8), (3, 9, 4), (3, 4, 2), (3, 2, 6), (3, 6, 8),
         (3, 8, 9), (4, 9, 5), (2, 4, 11), (6, 2, 10), (8, 6, 7), (9, 8, 1)]
    verts = [np.array(p, np.float64) / np.linalg.norm(p) for p in v]
    faces = f
    for _ in range(subdivisions):
        cache: dict[tuple[int, int], int] = {}

        def mid(a: int, b: int) -> int:
            key = (min(a, b), max(a, b))
            if key not in cache:
                m = verts[a] + verts[b]
                verts.append(m / np.linalg.norm(m))
                cache[key] = len(verts) - 1
            return cache[key]

        nxt = []
        for a, b, c in faces:
            ab, bc, ca = mid(a, b), mid(b, c), mid(c, a)
            nxt += [(a, ab, ca), (b, bc, ab), (c, ca, bc), (ab, bc, ca)]
        faces = nxt
    return np.array(verts, np.float64), np.array(faces, np.int32)


def ellipsoid_mesh(seed: int, subdivisions: int = 5, extent=(0.10, 0.07, 0.05)) -> MeshData:
    """Icosphere (subdivision 5: 20,480 triangles) scaled to an ellipsoid."""
    rng = np.random.default_rng(seed)
    v, f = icosphere(subdivisions)
    v = v * (np.array(extent) * 0.5)
    colors = rng.integers(0, 256, size=(v.shape[0], 3), dtype=np.uint8)
    return MeshData(v.astype(np.float32), f, colors)


def displaced_sphere(seed: int, n_lat: int = 127, n_lon: int = 200, radius: float = 0.05,
                     amplitude: float = 0.12) -> MeshData:
    """UV sphere with seeded smooth radial displacement; 2*n_lon*(n_lat-2) triangles
    (n_lat=127, n_lon=200 -> 50,000)."""
    rng = np.random.default_rng(seed)
    theta = np.linspace(0.0, np.pi, n_lat)[1:-1]
    phi = np.linspace(0.0, 2.0 * np.pi, n_lon, endpoint=False)
    th, ph = np.meshgrid(theta, phi, indexing="ij")
    dirs = np.stack([np.sin(th) * np.cos(ph), np.sin(th) * np.sin(ph), np.cos(th)], -1).reshape(-1, 3)
    dirs = np.concatenate([[[0.0, 0.0, 1.0]], dirs, [[0.0, 0.0, -1.0]]], 0)
    freqs = rng.normal(size=(6, 3)) * 3.0
    phases = rng.uniform(0, 2 * np.pi, size=6)
    amps = rng.uniform(0.3, 1.0, size=6)
    disp = sum(a * np.sin(dirs @ fr + p) for a, fr, p in zip(amps, freqs, phases)) / amps.sum()
    verts = dirs * radius * (1.0 + amplitude * disp)[:, None]
    rings = n_lat - 2
    idx = lambda i, j: 1 + i * n_lon + (j % n_lon)  # noqa: E731
    faces = []
    for j in range(n_lon):
        faces.append((0, idx(0, j + 1), idx(0, j)))
    for i in range(rings - 1):
        for j in range(n_lon):
            a, b, c, d = idx(i, j), idx(i, j + 1), idx(i + 1, j), idx(i + 1, j + 1)
            faces.append((a, b, c))
            faces.append((b, d, c))
    last = 1 + rings * n_lon
    for j in range(n_lon):
        faces.append((last, idx(rings - 1, j), idx(rings - 1, j + 1)))
    faces = np.array(faces, np.int32)
    colors = rng.integers(0, 256, size=(verts.shape[0], 3), dtype=np.uint8)
    return MeshData(verts.astype(np.float32), faces, colors)


def dense_mesh(seed: int, n_faces_target: int = 250_000) -> MeshData:
    """Displaced UV sphere with ~n_faces_target triangles (many sub-pixel)."""
    n_lon = 400
    n_lat = int(round(n_faces_target / (2 * n_lon))) + 2
    return displaced_sphere(seed, n_lat=n_lat, n_lon=n_lon, radius=0.06, amplitude=0.2)


def vertex_normals(v: np.ndarray, f: np.ndarray) -> np.ndarray:
    """Area-weighted vertex normals (float32), normalised with a +z fallback."""
    v = v.astype(np.float32)
    n = np.zeros_like(v)
    fn = np.cross(v[f[:, 1]] - v[f[:, 0]], v[f[:, 2]] - v[f[:, 0]]).astype(np.float32)
    for col in range(3):
        np.add.at(n, f[:, col], fn)
    ln = np.sqrt(np.maximum((n * n).sum(1), 0.0)).astype(np.float32)
    out = np.where(ln[:, None] < 1e-12, 0.0, n / np.maximum(ln, 1e-30)[:, None]).astype(np.float32)
    bad = np.sqrt((out * out).sum(1)) < 1e-6
    out[bad] = (0.0, 0.0, 1.0)
    return out


def rotation_matrix(rng: np.random.Generator) -> np.ndarray:
    q = rng.normal(size=4)
    q /= np.linalg.norm(q)
    w, x, y, z = q
    return np.array([[1 - 2 * (y * y + z * z), 2 * (x * y - z * w), 2 * (x * z + y * w)],
                     [2 * (x * y + z * w), 1 - 2 * (x * x + z * z), 2 * (y * z - x * w)],
                     [2 * (x * z - y * w), 2 * (y * z + x * w), 1 - 2 * (x * x + y * y)]])


def random_pose(rng: np.random.Generator, dist=(0.6, 1.0), lateral: float = 0.05) -> np.ndarray:
    pose = np.eye(4, dtype=np.float32)
    pose[:3, :3] = rotation_matrix(rng)
    pose[:3, 3] = (rng.uniform(-lateral, lateral), rng.uniform(-lateral, lateral),
                   rng.uniform(*dist))
    return pose


def random_walk(rng: np.random.Generator, pose: np.ndarray, max_t: float = 0.02,
                max_deg: float = 5.0) -> np.ndarray:
    axis = rng.normal(size=3)
    axis /= np.linalg.norm(axis)
    ang = np.deg2rad(rng.uniform(0, max_deg))
    kx = np.array([[0, -axis[2], axis[1]], [axis[2], 0, -axis[0]], [-axis[1], axis[0], 0]])
    r = np.eye(3) + np.sin(ang) * kx + (1 - np.cos(ang)) * kx @ kx
    out = pose.copy()
    out[:3, :3] = (r @ pose[:3, :3]).astype(np.float32)
    step = rng.normal(size=3)
    step *= rng.uniform(0, max_t) / max(np.linalg.norm(step), 1e-9)
    out[:3, 3] = pose[:3, 3] + step.astype(np.float32)
    return out


def degrade_frame(rng: np.random.Generator, depth: np.ndarray, noise_sigma: float,
                  hole_fraction: float) -> np.ndarray:
    d = depth.copy()
    valid = d > 0
    d[valid] += rng.normal(0.0, noise_sigma, size=int(valid.sum())).astype(np.float32)
    holes = rng.random(d.shape) < hole_fraction
    d[holes] = 0.0
    return d.astype(np.float32)


def render_frame_gpu(fpk, mesh: MeshData, normals: np.ndarray, pose: np.ndarray, K: np.ndarray,
                     width: int, height: int, device: str = "cuda"):
    """Render RGB (uint8 HWC) and depth (float32 HW, metres) of `mesh` at `pose`
    with the library rasterizer, using the whole frame as the crop box."""
    import torch

    from .kernels import Intrinsics, Mesh

    dev = torch.device(device)
    verts = torch.from_numpy(np.ascontiguousarray(mesh.vertices, np.float32)).to(dev)
    nrm = torch.from_numpy(np.ascontiguousarray(normals, np.float32)).to(dev)
    cols = torch.from_numpy((mesh.colors.astype(np.float32) / np.float32(255.0))).to(dev)
    faces = torch.from_numpy(np.ascontiguousarray(mesh.faces, np.int32)).to(dev)
    m = Mesh(verts.data_ptr(), nrm.data_ptr(), cols.data_ptr(), None, None, faces.data_ptr(),
             verts.shape[0], faces.shape[0], 0, 0)
    params = fpk.default_params()
    params.input_width = width
    params.input_height = height
    k = Intrinsics(float(K[0, 0]), float(K[1, 1]), float(K[0, 2]), float(K[1, 2]))
    poses = torch.from_numpy(np.ascontiguousarray(pose, np.float32).reshape(1, 16)).to(dev)
    boxes = torch.tensor([[0.0, 0.0, float(width), float(height)]], device=dev)
    rgb = torch.empty((height, width, 3), device=dev)
    xyz = torch.empty((height, width, 3), device=dev)
    fpk.render(m, poses.data_ptr(), boxes.data_ptr(), 1, k, params, rgb.data_ptr(), xyz.data_ptr())
    torch.cuda.synchronize()
    rgb_u8 = (rgb.clamp(0, 1) * 255.0 + 0.5).to(torch.uint8).cpu().numpy()
    depth = xyz[..., 2].cpu().numpy().astype(np.float32)
    return rgb_u8, depth


def fibonacci_directions(n: int) -> np.ndarray:
    """n unit vectors spread evenly over the sphere (Fibonacci lattice)."""
    i = np.arange(n) + 0.5
    z = 1.0 - 2.0 * i / n
    r = np.sqrt(np.maximum(0.0, 1.0 - z * z))
    phi = np.pi * (3.0 - np.sqrt(5.0)) * i
    return np.stack([r * np.cos(phi), r * np.sin(phi), z], 1)


def look_at_origin(camera_position: np.ndarray) -> np.ndarray:
    """camera_to_world (4x4, float32) of a camera at `camera_position` whose
    optical axis (+z) points at the world origin, image rows (+y) downward."""
    c = np.asarray(camera_position, np.float64)
    z = -c / np.linalg.norm(c)
    up = np.array([0.0, 0.0, 1.0]) if abs(z[2]) < 0.95 else np.array([0.0, 1.0, 0.0])
    x = np.cross(z, up)
    x /= np.linalg.norm(x)
    y = np.cross(z, x)
    m = np.eye(4)
    m[:3, 0], m[:3, 1], m[:3, 2], m[:3, 3] = x, y, z, c
    return m.astype(np.float32)


def invert_pose(m: np.ndarray) -> np.ndarray:
    out = np.eye(4, dtype=np.float64)
    r = m[:3, :3].astype(np.float64)
    out[:3, :3] = r.T
    out[:3, 3] = -r.T @ m[:3, 3]
    return out.astype(np.float32)
