"""CPU: mesh ingest of the product (fpk_load_mesh: OBJ/PLY load, normals,
centring, diameter) against the reference's loadMesh + preprocessMesh
(golden vectors in tests/golden/ref_cpu.npz, and the live reference CPU build
when it is present)."""
from __future__ import annotations

import ctypes as C
import struct
from pathlib import Path

import numpy as np
import pytest

from oracle_lib import REF_CPU_SO, RefCpu
from scene_util import write_obj

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(fpk, path, scale=1.0):
    f = fpk.lib.fpk_load_mesh
    f.restype = C.c_int
    f.argtypes = [C.c_char_p, C.c_float, C.POINTER(C.c_int), C.POINTER(C.c_int)] + [C.c_void_p] * 6
    nv, nf = C.c_int(0), C.c_int(0)
    assert f(str(path).encode(), scale, C.byref(nv), C.byref(nf), *([None] * 6)) == 0, \
        fpk.lib.fpk_last_error().decode()
    v = np.zeros((nv.value, 3), np.float32)
    n = np.zeros((nv.value, 3), np.float32)
    col = np.zeros((nv.value, 3), np.uint8)
    fc = np.zeros((nf.value, 3), np.int32)
    c = np.zeros(3, np.float32)
    d = np.zeros(1, np.float32)
    p = lambda a: a.ctypes.data  # noqa: E731
    assert f(str(path).encode(), scale, C.byref(nv), C.byref(nf), p(v), p(n), p(col), p(fc), p(c), p(d)) == 0
    return dict(vertices=v, normals=n, colors=col, faces=fc, center=c, diameter=float(d[0]))


def write_ply(path, verts, faces, colors, normals=None, binary=False):
    props = ["property float x", "property float y", "property float z"]
    if normals is not None:
        props += ["property float nx", "property float ny", "property float nz"]
    props += ["property uchar red", "property uchar green", "property uchar blue"]
    head = ["ply", f"format {'binary_little_endian' if binary else 'ascii'} 1.0",
            f"element vertex {len(verts)}", *props, f"element face {len(faces)}",
            "property list uchar int vertex_indices", "end_header"]
    with open(path, "wb") as f:
        f.write(("\n".join(head) + "\n").encode())
        for i, v in enumerate(verts):
            vals = list(v) + (list(normals[i]) if normals is not None else [])
            if binary:
                f.write(struct.pack("<" + "f" * len(vals), *vals) + bytes(colors[i].tolist()))
            else:
                f.write((" ".join("%.9g" % x for x in vals) + " %d %d %d\n" % tuple(colors[i])).encode())
        for t in faces:
            if binary:
                f.write(struct.pack("<Biii", 3, *[int(x) for x in t]))
            else:
                f.write(("3 %d %d %d\n" % tuple(int(x) for x in t)).encode())


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN / "ref_cpu.npz")


def test_obj_matches_reference_golden(fpk, golden, tmp_path):
    obj = tmp_path / "m.obj"
    write_obj(obj, golden["mesh_in_vertices"], golden["mesh_in_faces"], golden["mesh_in_colors"])
    m = load(fpk, obj)
    np.testing.assert_array_equal(m["vertices"], golden["mesh_vertices"])
    np.testing.assert_array_equal(m["normals"], golden["mesh_normals"])
    np.testing.assert_array_equal(m["colors"], golden["mesh_colors"])
    np.testing.assert_array_equal(m["faces"], golden["mesh_faces"])
    np.testing.assert_array_equal(m["center"], golden["mesh_center"])
    assert np.float32(m["diameter"]) == golden["mesh_diameter"]


@pytest.mark.parametrize("binary", [False, True])
@pytest.mark.parametrize("with_normals", [False, True])
def test_ply_matches_obj_and_reference(fpk, golden, tmp_path, binary, with_normals):
    v, f, c = golden["mesh_in_vertices"], golden["mesh_in_faces"], golden["mesh_in_colors"]
    ply = tmp_path / "m.ply"
    normals = golden["mesh_normals"] if with_normals else None
    write_ply(ply, v + np.float32(0.25), f, c, normals=normals, binary=binary)
    m = load(fpk, ply)
    np.testing.assert_array_equal(m["colors"], c)
    np.testing.assert_array_equal(m["faces"], f)
    np.testing.assert_allclose(m["center"], golden["mesh_center"] + 0.25, atol=1e-6)
    np.testing.assert_allclose(m["vertices"], golden["mesh_vertices"], atol=1e-6)
    assert abs(m["diameter"] - float(golden["mesh_diameter"])) < 1e-5
    if REF_CPU_SO.is_file():
        r = RefCpu().load_mesh(str(ply))
        for k in ("vertices", "normals", "colors", "center"):
            np.testing.assert_array_equal(m[k], r[k])
        np.testing.assert_array_equal(m["faces"], r["faces"].astype(np.int32))
        assert np.float32(m["diameter"]) == np.float32(r["diameter"])


def test_unit_scale_and_polygon_fan(fpk, tmp_path):
    obj = tmp_path / "quad.obj"
    obj.write_text("v 0 0 0\nv 1000 0 0\nv 1000 1000 0\nv 0 1000 0\nv 0 0 1000\nf 1 2 3 4\nf -5/1/1 -4 -1\n")
    m = load(fpk, obj, scale=0.001)
    np.testing.assert_array_equal(m["faces"], [[0, 1, 2], [0, 2, 3], [0, 1, 4]])
    np.testing.assert_allclose(m["center"], [0.5, 0.5, 0.5], atol=1e-7)
    assert abs(m["diameter"] - np.sqrt(3.0)) < 1e-6  # (1,1,0)-(0,0,1)
    np.testing.assert_array_equal(m["colors"], np.full((5, 3), 128, np.uint8))


def test_load_errors(fpk, tmp_path):
    bad = tmp_path / "bad.obj"
    bad.write_text("v 0 0 0\nf 0 1 2\n")
    f = fpk.lib.fpk_load_mesh
    nv, nf = C.c_int(0), C.c_int(0)
    assert f(str(bad).encode(), 1.0, C.byref(nv), C.byref(nf), *([None] * 6)) != 0
    assert "1-based" in fpk.lib.fpk_last_error().decode()
    empty = tmp_path / "empty.ply"
    empty.write_text("ply\nformat ascii 1.0\nelement vertex 0\nend_header\n")
    assert f(str(empty).encode(), 1.0, C.byref(nv), C.byref(nf), *([None] * 6)) != 0
    assert "no usable vertices" in fpk.lib.fpk_last_error().decode()
