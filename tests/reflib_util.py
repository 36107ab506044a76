"""The reference's own library (oracle/_ref/libfpref_full.so: estimator, C ABI,
pipeline kernels, rasterizer and model-free reconstruction from its unmodified
sources) for the parity tests, with torch networks behind its runner seam
(test infrastructure)."""
from __future__ import annotations

import ctypes as C
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
REF_FULL_SO = ROOT / "oracle" / "_ref" / "libfpref_full.so"


def load(refine_tensors=None, score_tensors=None, dtype=None, keep_scores=None):
    """The library with every fp_* signature declared; when weights are given,
    torch networks of that dtype (fp32 by default, TF32 off) are installed."""
    from fp_b200 import capi

    lib = C.CDLL(str(REF_FULL_SO))
    for name, (res, argt) in capi._SIGNATURES.items():
        if hasattr(lib, name):
            fn = getattr(lib, name)
            fn.restype, fn.argtypes = res, argt
    lib.refmf_reconstruct.restype = C.c_int
    out = {"lib": lib}
    if refine_tensors is not None:
        import torch

        sys.path.insert(0, str(ROOT / "oracle"))
        from fp_net_torch import TorchNets, device_tensor, install

        torch.backends.cudnn.allow_tf32 = False
        torch.backends.cuda.matmul.allow_tf32 = False
        nets = TorchNets(refine_tensors, score_tensors, dtype or torch.float32, graphs=False)
        if keep_scores is not None:
            inner = nets.score_ptrs

            def score_ptrs(r, o, s, n, stream):
                inner(r, o, s, n, stream)
                torch.cuda.ExternalStream(stream).synchronize()
                keep_scores["scores"] = device_tensor(s, (n,)).cpu().numpy()

            nets.score_ptrs = score_ptrs
        out["callbacks"] = install(lib, nets)
        out["nets"] = nets
    return out


def reconstruct(lib, views, K, c2w, stride, max_vertices, edge, depth_min=0.001, depth_max=100.0):
    """The reference's model-free mesh (host code) of views [(rgb, depth, mask)]."""
    n = len(views)
    h, w = views[0][1].shape
    keep = [(np.ascontiguousarray(r, np.uint8), np.ascontiguousarray(d, np.float32),
             np.ascontiguousarray(m, np.uint8)) for r, d, m in views]
    P8 = C.POINTER(C.c_uint8)
    PF = C.POINTER(C.c_float)
    depths = (PF * n)(*[k[1].ctypes.data_as(PF) for k in keep])
    rgbs = (P8 * n)(*[k[0].ctypes.data_as(P8) for k in keep])
    masks = (P8 * n)(*[k[2].ctypes.data_as(P8) for k in keep])
    k9 = np.ascontiguousarray(np.repeat(np.asarray(K, np.float32).reshape(1, 9), n, 0))
    m16 = np.ascontiguousarray(np.stack([np.asarray(c, np.float32).reshape(16) for c in c2w]))
    cap_v = max_vertices + 16
    cap_f = 2 * sum(v[1].size for v in views) // max(1, stride * stride) + 16
    verts = np.zeros((cap_v, 3), np.float32)
    colors = np.zeros((cap_v, 3), np.uint8)
    normals = np.zeros((cap_v, 3), np.float32)
    faces = np.zeros((cap_f, 3), np.int32)
    nv, nf = C.c_int(), C.c_int()
    err = C.create_string_buffer(512)
    rc = lib.refmf_reconstruct(n, w, h, depths, rgbs, masks, k9.ctypes.data_as(PF), m16.ctypes.data_as(PF),
                               stride, max_vertices, C.c_float(edge), C.c_float(depth_min), C.c_float(depth_max),
                               C.byref(nv), C.byref(nf), verts.ctypes.data_as(PF), colors.ctypes.data_as(P8),
                               normals.ctypes.data_as(PF), faces.ctypes.data_as(C.POINTER(C.c_int32)), cap_v, cap_f,
                               err, len(err))
    assert rc == 0, err.value.decode()
    assert nv.value <= cap_v and nf.value <= cap_f
    return verts[:nv.value], colors[:nv.value], normals[:nv.value], faces[:nf.value]
