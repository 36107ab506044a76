"""BENCHMARK / TEST INFRASTRUCTURE ONLY: RefineNet / ScoreNet as fast torch
networks, the stand-in for the reference's TensorRT engines.

The reference runs its two networks as TensorRT engines built from ONNX at the
configured precision (src/tensorrt_runner.cu:65-80, 367-407). TensorRT is not
installed here, so bench.py's reference_gpu baseline drives the reference's own
library (oracle/_ref/libfpref_full.so) with these networks behind its runner
seam: the same architecture and weight pack as oracle/fp_net_ref.py, run the
way a tuned inference engine would run it -- weights cast once to FP16/BF16,
channels-last cuDNN convolutions (autotuned), fused scaled-dot-product
attention, and each (network, batch, buffer) call replayed as a CUDA graph
after its first run. Inputs and outputs keep the runner's fp32 contract
(inputA/inputB [B,6,160,160] NCHW, trans/rot [B,3], score [B]).
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.nn.functional as F


class _DeviceArray:
    """A raw device pointer with a shape, readable by torch.as_tensor."""

    def __init__(self, ptr: int, shape: tuple, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"data": (int(ptr), False), "shape": tuple(shape), "typestr": typestr,
                                         "version": 3}


def device_tensor(ptr: int, shape: tuple) -> torch.Tensor:
    return torch.as_tensor(_DeviceArray(ptr, shape), device="cuda")


class TorchNets:
    def __init__(self, refine_tensors: dict, score_tensors: dict, dtype=torch.float16, graphs: bool = True):
        torch.backends.cudnn.benchmark = True
        self.dtype = dtype
        cast = lambda t: {k: torch.as_tensor(v).to("cuda", dtype) for k, v in t.items()}  # noqa: E731
        self.wr, self.ws = cast(refine_tensors), cast(score_tensors)
        for w in (self.wr, self.ws):
            for k in list(w):
                if w[k].ndim == 4:
                    w[k] = w[k].contiguous(memory_format=torch.channels_last)
        self.graphs = graphs
        self._graphs: dict = {}

    # -- network bodies (same layer graph as oracle/fp_net_ref.py) ------------
    @staticmethod
    def _conv(w, x, name, stride, pad, relu=True):
        y = F.conv2d(x, w[f"{name}.w"], w[f"{name}.b"], stride=stride, padding=pad)
        return F.relu(y) if relu else y

    def _res(self, w, x, name):
        y = self._conv(w, x, f"{name}.c1", 1, 1)
        y = self._conv(w, y, f"{name}.c2", 1, 1, relu=False)
        return F.relu(y + x)

    def _tokens(self, w, A, B):
        n = A.shape[0]
        x = torch.cat([A, B], 0).to(self.dtype).contiguous(memory_format=torch.channels_last)
        x = self._conv(w, x, "encA.conv1", 2, 3)
        x = self._conv(w, x, "encA.conv2", 2, 1)
        x = self._res(w, x, "encA.res1")
        x = self._res(w, x, "encA.res2")
        ab = torch.cat([x[:n], x[n:]], 1)
        ab = self._res(w, ab, "encAB.res1")
        ab = self._res(w, ab, "encAB.res2")
        ab = self._conv(w, ab, "encAB.conv", 2, 1)
        ab = self._res(w, ab, "encAB.res3")
        ab = self._res(w, ab, "encAB.res4")
        t = ab.flatten(2).transpose(1, 2)  # [n, 400, 512]
        return t + w["pos"][None, : t.shape[1]]

    @staticmethod
    def _mha(w, x, p, heads=4):
        n, L, E = x.shape
        qkv = F.linear(x, w[f"{p}.in_w"], w[f"{p}.in_b"]).view(n, L, 3, heads, E // heads)
        q, k, v = qkv.permute(2, 0, 3, 1, 4).unbind(0)
        o = F.scaled_dot_product_attention(q, k, v)
        return F.linear(o.transpose(1, 2).reshape(n, L, E), w[f"{p}.out_w"], w[f"{p}.out_b"])

    def _encoder_layer(self, w, x, p):
        x = F.layer_norm(x + self._mha(w, x, f"{p}.attn"), (x.shape[-1],), w[f"{p}.ln1.w"], w[f"{p}.ln1.b"])
        h = F.linear(F.relu(F.linear(x, w[f"{p}.ff1.w"], w[f"{p}.ff1.b"])), w[f"{p}.ff2.w"], w[f"{p}.ff2.b"])
        return F.layer_norm(x + h, (x.shape[-1],), w[f"{p}.ln2.w"], w[f"{p}.ln2.b"])

    @torch.no_grad()
    def refine(self, A, B):
        t = self._tokens(self.wr, A, B)
        out = []
        for head in ("trans", "rot"):
            y = self._encoder_layer(self.wr, t, head)
            out.append(F.linear(y, self.wr[f"{head}.out.w"], self.wr[f"{head}.out.b"]).float().mean(1))
        return out[0], out[1]

    @torch.no_grad()
    def score(self, A, B):
        t = self._tokens(self.ws, A, B)
        feat = self._mha(self.ws, t, "att").float().mean(1).to(self.dtype)
        x = self._mha(self.ws, feat[None], "att_cross")[0]
        return F.linear(x, self.ws["linear.w"], self.ws["linear.b"]).float()[:, 0]

    # -- the runner seam: device pointers in, device pointers out -------------
    def _run(self, key, body, stream_ptr):
        ext = torch.cuda.ExternalStream(stream_ptr) if stream_ptr else torch.cuda.current_stream()
        if not self.graphs:
            with torch.cuda.stream(ext):
                body()
            return
        g = self._graphs.get(key)
        if g is None:
            ext.synchronize()  # the inputs the reference kernels wrote are ready
            side = torch.cuda.Stream()
            with torch.cuda.stream(side):
                body()  # warm-up: cuDNN autotuning and workspace allocation
                body()
            side.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                body()
            self._graphs[key] = g
        with torch.cuda.stream(ext):
            g.replay()

    def refine_ptrs(self, rendered, observed, delta_t, delta_r, n, stream_ptr):
        A, B = device_tensor(rendered, (n, 6, 160, 160)), device_tensor(observed, (n, 6, 160, 160))
        dt, dr = device_tensor(delta_t, (n, 3)), device_tensor(delta_r, (n, 3))

        def body():
            t, r = self.refine(A, B)
            dt.copy_(t)
            dr.copy_(r)

        self._run(("refine", n, rendered, observed, delta_t, delta_r), body, stream_ptr)

    def score_ptrs(self, rendered, observed, scores, n, stream_ptr):
        A, B = device_tensor(rendered, (n, 6, 160, 160)), device_tensor(observed, (n, 6, 160, 160))
        s = device_tensor(scores, (n,))

        def body():
            s.copy_(self.score(A, B))

        self._run(("score", n, rendered, observed, scores), body, stream_ptr)


REFINE_CB = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p)
SCORE_CB = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p)


def install(lib: C.CDLL, nets: TorchNets):
    """Register `nets` as the network engines of the reference library `lib`
    (oracle/_ref/libfpref_full.so). Returns the callback objects, which the
    caller must keep alive while the library may call them."""
    import traceback

    def refine(r, o, dt, dr, n, stream):
        try:
            nets.refine_ptrs(r, o, dt, dr, n, stream or 0)
            return 0
        except Exception:  # a failing callback becomes the runner's error
            traceback.print_exc()
            return 1

    def score(r, o, s, n, stream):
        try:
            nets.score_ptrs(r, o, s, n, stream or 0)
            return 0
        except Exception:
            traceback.print_exc()
            return 1

    cbs = (REFINE_CB(refine), SCORE_CB(score))
    lib.refnet_set_callbacks.argtypes = [REFINE_CB, SCORE_CB]
    lib.refnet_set_callbacks.restype = None
    lib.refnet_set_callbacks(*cbs)
    return cbs
