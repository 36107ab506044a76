"""Small seeded scenes for the parity tests (test infrastructure).

Frames are rendered with the CPU oracle at full-frame size (the crop box is
the whole image), then degraded with Gaussian depth noise and holes, so the
same inputs are available with or without a GPU.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from fp_b200 import synthetic as syn


@dataclass
class Scene:
    verts: np.ndarray      # centred mesh vertices [V,3]
    normals: np.ndarray    # [V,3]
    colors_u8: np.ndarray  # [V,3]
    colors_f: np.ndarray   # [V,3] float32 = u8 / 255
    faces: np.ndarray      # [F,3] int32
    center: np.ndarray     # mesh bbox centre (original frame)
    diameter: float
    K: np.ndarray          # 3x3
    k4: np.ndarray         # fx, fy, cx, cy
    rgb: np.ndarray        # [H,W,3] uint8
    depth: np.ndarray      # [H,W] float32
    mask: np.ndarray       # [H,W] uint8
    gt_pose: np.ndarray    # 4x4 (centred mesh)


def cube_mesh(seed: int, half: float = 0.04) -> syn.MeshData:
    rng = np.random.default_rng(seed)
    v = np.array([[x, y, z] for x in (-half, half) for y in (-half, half) for z in (-half, half)],
                 np.float32)
    f = np.array([[0, 1, 3], [0, 3, 2], [4, 6, 7], [4, 7, 5], [0, 4, 5], [0, 5, 1],
                  [2, 3, 7], [2, 7, 6], [0, 2, 6], [0, 6, 4], [1, 5, 7], [1, 7, 3]], np.int32)
    return syn.MeshData(v, f, rng.integers(0, 256, size=(8, 3), dtype=np.uint8))


def make_mesh(kind: str, seed: int = 0) -> syn.MeshData:
    if kind == "cube":
        return cube_mesh(seed)
    if kind == "ellipsoid":
        return syn.ellipsoid_mesh(seed, subdivisions=5)
    if kind == "ellipsoid_small":
        return syn.ellipsoid_mesh(seed, subdivisions=3)
    if kind == "sphere50k":
        return syn.displaced_sphere(seed)
    if kind == "dense250k":
        return syn.dense_mesh(seed)
    if kind == "bigtris":
        return big_triangle_soup(seed)
    raise ValueError(kind)


def big_triangle_soup(seed: int, n: int = 3000, radius: float = 0.05) -> syn.MeshData:
    """n independent triangles with corners spread over a ball: nearly every
    triangle covers a large part of the crop, so the rasterizer's list of
    CTA-shared large triangles (1,024 entries per CTA) overflows and the rest
    fall back to per-thread rasterization."""
    rng = np.random.default_rng(seed)
    v = rng.normal(size=(3 * n, 3))
    v *= (radius * rng.uniform(0.3, 1.0, size=(3 * n, 1))) / np.linalg.norm(v, axis=1, keepdims=True)
    f = np.arange(3 * n, dtype=np.int32).reshape(n, 3)
    return syn.MeshData(v.astype(np.float32), f, rng.integers(0, 256, size=(3 * n, 3), dtype=np.uint8))


def make_scene(oracle, kind: str = "ellipsoid_small", seed: int = 0, width: int = 640,
               height: int = 480, noise: float = 0.002, holes: float = 0.05) -> Scene:
    rng = np.random.default_rng(seed + 1000)
    m = make_mesh(kind, seed)
    center, diameter, centered = oracle.mesh_center_diameter(m.vertices)
    normals = oracle.vertex_normals(centered, m.faces)
    colors_f = (m.colors.astype(np.float32) / np.float32(255.0)).astype(np.float32)
    if (width, height) == (640, 480):
        K = syn.K_640
    elif (width, height) == (1280, 720):
        K = syn.K_1280
    else:  # same field of view as the 640x480 camera
        f = 600.0 * width / 640.0
        K = np.array([[f, 0.0, width / 2.0], [0.0, f, height / 2.0], [0.0, 0.0, 1.0]], np.float32)
    k4 = np.array([K[0, 0], K[1, 1], K[0, 2], K[1, 2]], np.float32)
    pose = syn.random_pose(rng, dist=(0.6, 0.8), lateral=0.03)
    cfg = oracle.config(input_width=width, input_height=height)
    boxes = np.array([[0.0, 0.0, float(width), float(height)]], np.float32)
    rgb_f, xyz, _ = oracle.render(centered, normals, colors_f, m.faces, pose.reshape(1, 16), boxes,
                                  k4, cfg)
    rgb = (np.clip(rgb_f[0], 0, 1) * 255.0 + 0.5).astype(np.uint8)
    depth_clean = xyz[0, ..., 2].astype(np.float32)
    mask = (depth_clean > 0).astype(np.uint8)
    depth = syn.degrade_frame(rng, depth_clean, noise, holes)
    return Scene(centered, normals, m.colors, colors_f, m.faces, center, diameter, K, k4, rgb,
                 depth, mask, pose)


def hypotheses(oracle, scene: Scene, n: int, seed: int = 0, jitter_t: float = 0.01) -> np.ndarray:
    """n poses: grid rotations at the scene's translation plus a small jitter."""
    rng = np.random.default_rng(seed)
    rots = oracle.rotation_grid()
    idx = rng.choice(rots.shape[0], size=n, replace=False)
    t = scene.gt_pose[:3, 3] + rng.normal(0, jitter_t, size=3).astype(np.float32)
    return oracle.seed_poses(rots[idx], t.astype(np.float32))


def write_obj(path, verts, faces, colors_u8) -> None:
    """OBJ with per-vertex colours in [0, 1] written as (c + 0.5) / 255 (255 as
    1.0) so the loader's scale-by-255-and-truncate recovers c exactly;
    vertices round-trip in %.9g."""
    def enc(c):
        return 1.0 if c >= 255 else (float(c) + 0.5) / 255.0

    with open(path, "w") as f:
        for v, c in zip(verts, colors_u8):
            f.write("v %.9g %.9g %.9g %.9g %.9g %.9g\n" % (v[0], v[1], v[2], enc(c[0]), enc(c[1]),
                                                         enc(c[2])))
        for t in faces:
            f.write("f %d %d %d\n" % (t[0] + 1, t[1] + 1, t[2] + 1))


def model_free_views(oracle, n_views: int, seed: int = 0, distance: float = 0.7, n_lat: int = 77,
                     width: int = 640, height: int = 480):
    """Reference views of a seeded displaced sphere (n_lat=77: 30,000 triangles)
    from cameras on a Fibonacci sphere of radius `distance` looking at the
    object (world frame = object frame). Returns (scene mesh parts, K, views
    [(rgb u8, depth f32, mask u8)], camera_to_world list), rendered by the CPU
    oracle."""
    m = syn.displaced_sphere(seed, n_lat=n_lat, n_lon=200)
    center, diameter, centered = oracle.mesh_center_diameter(m.vertices)
    normals = oracle.vertex_normals(centered, m.faces)
    colors_f = (m.colors.astype(np.float32) / np.float32(255.0)).astype(np.float32)
    K = syn.K_640
    k4 = np.array([K[0, 0], K[1, 1], K[0, 2], K[1, 2]], np.float32)
    cfg = oracle.config(input_width=width, input_height=height)
    boxes = np.array([[0.0, 0.0, float(width), float(height)]], np.float32)
    views, c2ws = [], []
    for d in syn.fibonacci_directions(n_views):
        c2w = syn.look_at_origin(d * distance)
        pose = syn.invert_pose(c2w)
        rgb_f, xyz, _ = oracle.render(centered, normals, colors_f, m.faces, pose.reshape(1, 16), boxes, k4, cfg)
        rgb = (np.clip(rgb_f[0], 0, 1) * 255.0 + 0.5).astype(np.uint8)
        depth = xyz[0, ..., 2].astype(np.float32)
        views.append((rgb, depth, (depth > 0).astype(np.uint8)))
        c2ws.append(c2w)
    parts = dict(verts=centered, normals=normals, colors_u8=m.colors, colors_f=colors_f, faces=m.faces,
                 diameter=diameter, k4=k4)
    return parts, K, views, c2ws


def render_query(oracle, parts, pose, K, width: int = 640, height: int = 480, seed: int = 0,
                 noise: float = 0.002, holes: float = 0.05):
    """One query frame of the model-free object at `pose` (object -> camera)."""
    rng = np.random.default_rng(seed)
    cfg = oracle.config(input_width=width, input_height=height)
    boxes = np.array([[0.0, 0.0, float(width), float(height)]], np.float32)
    k4 = np.array([K[0, 0], K[1, 1], K[0, 2], K[1, 2]], np.float32)
    rgb_f, xyz, _ = oracle.render(parts["verts"], parts["normals"], parts["colors_f"], parts["faces"],
                                  np.asarray(pose, np.float32).reshape(1, 16), boxes, k4, cfg)
    rgb = (np.clip(rgb_f[0], 0, 1) * 255.0 + 0.5).astype(np.uint8)
    clean = xyz[0, ..., 2].astype(np.float32)
    return rgb, syn.degrade_frame(rng, clean, noise, holes), (clean > 0).astype(np.uint8)
