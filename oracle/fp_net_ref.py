"""TEST INFRASTRUCTURE ONLY: torch fp32 reference of RefineNet / ScoreNet.

The parity checker for the tensor-core network kernels: the same architecture
and weight pack as the product (see foundation-pose-inference-library_b200/python/
fp_b200/weights.py), written with plain torch ops. The reference runtime runs
these networks as TensorRT engines (src/tensorrt_runner.cu:367-407); their I/O
contract is fixed there (inputs inputA/inputB [B,6,160,160] NCHW fp32, outputs
trans/rot [B,3] and score [B], tensorrt_runner.cu:123-125, config.hpp:78-82).
Only tests/ and bench.py's CPU-baseline leg may use this module.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


class NetRef:
    def __init__(self, tensors: dict, device="cpu", dtype=torch.float32):
        self.w = {k: torch.as_tensor(v).to(device=device, dtype=dtype) for k, v in tensors.items()}

    def _conv(self, x, name, stride, pad, relu=True):
        y = F.conv2d(x, self.w[f"{name}.w"], self.w[f"{name}.b"], stride=stride, padding=pad)
        return torch.relu(y) if relu else y

    def _res(self, x, name):
        y = self._conv(x, f"{name}.c1", 1, 1)
        y = self._conv(y, f"{name}.c2", 1, 1, relu=False)
        return torch.relu(y + x)

    def tokens(self, A, B):
        bs = A.shape[0]
        x = torch.cat([A, B], 0)
        x = self._conv(x, "encA.conv1", 2, 3)
        x = self._conv(x, "encA.conv2", 2, 1)
        x = self._res(x, "encA.res1")
        x = self._res(x, "encA.res2")
        ab = torch.cat([x[:bs], x[bs:]], 1)
        ab = self._res(ab, "encAB.res1")
        ab = self._res(ab, "encAB.res2")
        ab = self._conv(ab, "encAB.conv", 2, 1)
        ab = self._res(ab, "encAB.res3")
        ab = self._res(ab, "encAB.res4")
        t = ab.reshape(bs, ab.shape[1], -1).permute(0, 2, 1)
        return t + self.w["pos"][None, : t.shape[1]]

    def _mha(self, x, p, heads=4):
        # x [N, L, E]; PyTorch MultiheadAttention semantics (batch_first).
        n, L, E = x.shape
        d = E // heads
        qkv = x @ self.w[f"{p}.in_w"].T + self.w[f"{p}.in_b"]
        q, k, v = qkv.split(E, -1)
        q = q.reshape(n, L, heads, d).transpose(1, 2)
        k = k.reshape(n, L, heads, d).transpose(1, 2)
        v = v.reshape(n, L, heads, d).transpose(1, 2)
        att = torch.softmax((q @ k.transpose(-1, -2)) / (d ** 0.5), -1)
        o = (att @ v).transpose(1, 2).reshape(n, L, E)
        return o @ self.w[f"{p}.out_w"].T + self.w[f"{p}.out_b"]

    def _encoder_layer(self, x, p):
        # nn.TransformerEncoderLayer(d_model=512, nhead=4, dim_feedforward=512,
        # batch_first=True), post-norm, ReLU, eval mode.
        x = F.layer_norm(x + self._mha(x, f"{p}.attn"), (x.shape[-1],), self.w[f"{p}.ln1.w"],
                         self.w[f"{p}.ln1.b"], eps=1e-5)
        h = torch.relu(x @ self.w[f"{p}.ff1.w"].T + self.w[f"{p}.ff1.b"])
        h = h @ self.w[f"{p}.ff2.w"].T + self.w[f"{p}.ff2.b"]
        return F.layer_norm(x + h, (x.shape[-1],), self.w[f"{p}.ln2.w"], self.w[f"{p}.ln2.b"],
                            eps=1e-5)

    @torch.no_grad()
    def refine(self, A, B):
        t = self.tokens(A, B)
        out = []
        for head in ("trans", "rot"):
            y = self._encoder_layer(t, head)
            y = y @ self.w[f"{head}.out.w"].T + self.w[f"{head}.out.b"]
            out.append(y.mean(1))
        return out[0], out[1]

    @torch.no_grad()
    def score(self, A, B):
        t = self.tokens(A, B)
        feat = self._mha(t, "att").mean(1)                # [B, 512]
        x = self._mha(feat[None], "att_cross")[0]         # attention across hypotheses
        return (x @ self.w["linear.w"].T + self.w["linear.b"])[:, 0]
