"""RefineNet / ScoreNet weight packs (.fpw) for the B200 runtime.

The reference runtime loads ONNX exports of FoundationPose's two networks
(refiner_net.onnx / score_net.onnx) into TensorRT. This runtime loads the same
architectures from a flat weight pack instead: BatchNorm already folded into
the preceding convolution, fp32, little endian.

Architecture (the public FoundationPose design; the reference only fixes the
I/O contract: inputs inputA/inputB [B,6,160,160], outputs trans/rot [B,3] and
score [B]):
  encoder (shared weights for the rendered and observed crops):
    conv 7x7/2 6->64, conv 3x3/2 64->128, 2 x residual block(128)     "encA.*"
  concat(rendered, observed) -> 256 channels at 40x40, then
    2 x residual block(256), conv 3x3/2 256->512, 2 x residual(512)    "encAB.*"
  400 tokens x 512 + sinusoidal positional embedding                   "pos"
  RefineNet: two post-norm transformer encoder layers (4 heads, FF 512,
    ReLU), one per output, each followed by mean over tokens and a
    linear 512->3                                                       "trans.*", "rot.*"
  ScoreNet: self-attention over the 400 tokens, mean over tokens, then
    attention across all hypotheses and a linear 512->1                 "att.*", "att_cross.*", "linear.*"

File layout: b"FPW1", u32 version=1, u32 arch (0 refine, 1 score), u32 count,
then `count` records of 96 bytes {char name[64]; u32 ndim; u32 shape[4];
u32 pad; u64 offset}, then the tensors (fp32, 256-byte aligned offsets).
"""
from __future__ import annotations

import math
import struct
from pathlib import Path

import numpy as np

MAGIC = b"FPW1"
ARCH_IDS = {"refine": 0, "score": 1}
EMBED = 512
TOKENS = 400


def _conv_specs() -> list[tuple[str, tuple[int, ...]]]:
    s: list[tuple[str, tuple[int, ...]]] = []

    def conv(name, co, ci, k):
        s.append((f"{name}.w", (co, ci, k, k)))
        s.append((f"{name}.b", (co,)))

    conv("encA.conv1", 64, 6, 7)
    conv("encA.conv2", 128, 64, 3)
    for r in ("res1", "res2"):
        conv(f"encA.{r}.c1", 128, 128, 3)
        conv(f"encA.{r}.c2", 128, 128, 3)
    for r in ("res1", "res2"):
        conv(f"encAB.{r}.c1", 256, 256, 3)
        conv(f"encAB.{r}.c2", 256, 256, 3)
    conv("encAB.conv", 512, 256, 3)
    for r in ("res3", "res4"):
        conv(f"encAB.{r}.c1", 512, 512, 3)
        conv(f"encAB.{r}.c2", 512, 512, 3)
    s.append(("pos", (TOKENS, EMBED)))
    return s


def _mha(prefix: str) -> list[tuple[str, tuple[int, ...]]]:
    return [(f"{prefix}.in_w", (3 * EMBED, EMBED)), (f"{prefix}.in_b", (3 * EMBED,)),
            (f"{prefix}.out_w", (EMBED, EMBED)), (f"{prefix}.out_b", (EMBED,))]


def spec(arch: str) -> list[tuple[str, tuple[int, ...]]]:
    s = _conv_specs()
    if arch == "refine":
        for head in ("trans", "rot"):
            s += _mha(f"{head}.attn")
            s += [(f"{head}.ln1.w", (EMBED,)), (f"{head}.ln1.b", (EMBED,)),
                  (f"{head}.ff1.w", (EMBED, EMBED)), (f"{head}.ff1.b", (EMBED,)),
                  (f"{head}.ff2.w", (EMBED, EMBED)), (f"{head}.ff2.b", (EMBED,)),
                  (f"{head}.ln2.w", (EMBED,)), (f"{head}.ln2.b", (EMBED,)),
                  (f"{head}.out.w", (3, EMBED)), (f"{head}.out.b", (3,))]
    elif arch == "score":
        s += _mha("att") + _mha("att_cross")
        s += [("linear.w", (1, EMBED)), ("linear.b", (1,))]
    else:
        raise ValueError(f"unknown architecture {arch!r}")
    return s


def positional_embedding(tokens: int = TOKENS, dim: int = EMBED) -> np.ndarray:
    """Sinusoidal table: even channels sin(p * w_i), odd channels cos(p * w_i),
    w_i = 10000^(-2i/dim)."""
    pe = np.zeros((tokens, dim), np.float32)
    position = np.arange(tokens, dtype=np.float32)[:, None]
    div = np.exp(np.arange(0, dim, 2, dtype=np.float32) * np.float32(-math.log(10000.0) / dim))
    pe[:, 0::2] = np.sin(position * div)
    pe[:, 1::2] = np.cos(position * div)
    return pe


def random_weights(arch: str, seed: int) -> dict[str, np.ndarray]:
    """Seeded init chosen to keep activations O(1) through the whole network:
    He-uniform convolutions (BN folded as a per-channel scale in [0.5, 1]),
    the second convolution of every residual block scaled by 0.5, small
    biases, default-style uniform init for the transformer layers."""
    rng = np.random.default_rng(seed)
    out: dict[str, np.ndarray] = {}
    for name, shape in spec(arch):
        if name == "pos":
            out[name] = positional_embedding()
        elif name.endswith(".w") and len(shape) == 4:
            fan_in = shape[1] * shape[2] * shape[3]
            bound = math.sqrt(6.0 / fan_in)
            w = rng.uniform(-bound, bound, size=shape)
            w *= rng.uniform(0.5, 1.0, size=(shape[0], 1, 1, 1))  # folded BN scale
            if ".c2." in name + ".":
                w *= 0.5
            out[name] = w.astype(np.float32)
        elif name.endswith(".b") and len(shape) == 1 and any(
                name.startswith(p) for p in ("encA.", "encAB.")):
            out[name] = rng.uniform(-0.05, 0.05, size=shape).astype(np.float32)
        elif name.endswith("in_w"):
            bound = math.sqrt(6.0 / (shape[0] + shape[1]))
            out[name] = rng.uniform(-bound, bound, size=shape).astype(np.float32)
        elif name.endswith((".ln1.w", ".ln2.w")):
            out[name] = (1.0 + rng.uniform(-0.1, 0.1, size=shape)).astype(np.float32)
        elif len(shape) == 2:
            bound = 1.0 / math.sqrt(shape[1])
            out[name] = rng.uniform(-bound, bound, size=shape).astype(np.float32)
        else:
            out[name] = rng.uniform(-0.05, 0.05, size=shape).astype(np.float32)
    return out


def write_pack(path: str | Path, arch: str, tensors: dict[str, np.ndarray]) -> Path:
    path = Path(path)
    names = [n for n, _ in spec(arch)]
    missing = [n for n in names if n not in tensors]
    if missing:
        raise ValueError(f"missing tensors: {missing[:5]}")
    header = bytearray(MAGIC + struct.pack("<III", 1, ARCH_IDS[arch], len(names)))
    offset = len(header) + 96 * len(names)
    offset = (offset + 255) // 256 * 256
    records, blobs = [], []
    for n in names:
        a = np.ascontiguousarray(tensors[n], dtype="<f4")
        expect = dict(spec(arch))[n]
        if tuple(a.shape) != expect:
            raise ValueError(f"{n}: shape {a.shape} != {expect}")
        shape = list(a.shape) + [0] * (4 - a.ndim)
        records.append(struct.pack("<64sI4IIQ", n.encode(), a.ndim, *shape, 0, offset))
        blobs.append((offset, a.tobytes()))
        offset = (offset + a.nbytes + 255) // 256 * 256
    with open(path, "wb") as f:
        f.write(header)
        for r in records:
            f.write(r)
        for off, data in blobs:
            f.seek(off)
            f.write(data)
        f.truncate(offset)
    return path


def read_pack(path: str | Path) -> tuple[str, dict[str, np.ndarray]]:
    data = Path(path).read_bytes()
    if data[:4] != MAGIC:
        raise ValueError(f"{path}: not a weight pack")
    version, arch_id, count = struct.unpack_from("<III", data, 4)
    arch = {v: k for k, v in ARCH_IDS.items()}[arch_id]
    out = {}
    for i in range(count):
        rec = struct.unpack_from("<64sI4IIQ", data, 16 + 96 * i)
        name = rec[0].rstrip(b"\0").decode()
        ndim, shape, off = rec[1], rec[2:2 + rec[1]], rec[7]
        n = int(np.prod(shape)) if ndim else 1
        out[name] = np.frombuffer(data, "<f4", count=n, offset=off).reshape(shape).copy()
    return arch, out


def make_default_packs(directory: str | Path, seed: int = 0) -> tuple[Path, Path]:
    """Write seeded refine/score packs into `directory` (idempotent)."""
    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    refine = d / f"refine_seed{seed}.fpw"
    score = d / f"score_seed{seed}.fpw"
    if not refine.exists():
        write_pack(refine, "refine", random_weights("refine", seed))
    if not score.exists():
        write_pack(score, "score", random_weights("score", seed + 1))
    return refine, score
