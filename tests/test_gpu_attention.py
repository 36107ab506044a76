"""GPU tests of the tcgen05/TMEM self-attention kernel (fpk_attention) against
torch fp32 attention on the same rounded operands: 4 heads of 128 channels,
sequences of 400 tokens (RefineNet / ScoreNet) and ragged lengths.
Tolerance: 1e-2 of the output's max magnitude at fp16/bf16 (P and output
rounding) and 5e-3 at fp32 (TF32 products: 10-bit mantissas)."""
from __future__ import annotations

import math

import pytest

torch = pytest.importorskip("torch")

from fp_b200.kernels import FPK_DTYPE_BF16, FPK_DTYPE_F16, FPK_DTYPE_F32, FPK_DTYPE_F32_EXACT, attention  # noqa: E402
from kp8_util import Planar  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = "cuda"
DT = {FPK_DTYPE_BF16: torch.bfloat16, FPK_DTYPE_F16: torch.float16, FPK_DTYPE_F32: torch.float32,
      FPK_DTYPE_F32_EXACT: torch.float32}
# FPK_DTYPE_F32_EXACT (the strict-FP32 networks) runs fp32 FMA arithmetic:
# fp32 rounding of a different summation order only.
TOL = {FPK_DTYPE_BF16: 1e-2, FPK_DTYPE_F16: 1e-2, FPK_DTYPE_F32: 5e-3, FPK_DTYPE_F32_EXACT: 1e-5}


def reference(x: torch.Tensor, layers: int, heads: int, seq: int, n_seq: int) -> torch.Tensor:
    """x [n_seq*seq, layers*3*heads*128] (q | k | v per layer) -> [rows, layers*heads*128]."""
    d = heads * 128
    outs = []
    for z in range(layers):
        base = z * 3 * d
        q = x[:, base:base + d].reshape(n_seq, seq, heads, 128).transpose(1, 2)
        k = x[:, base + d:base + 2 * d].reshape(n_seq, seq, heads, 128).transpose(1, 2)
        v = x[:, base + 2 * d:base + 3 * d].reshape(n_seq, seq, heads, 128).transpose(1, 2)
        s = (q @ k.transpose(-1, -2)) / math.sqrt(128.0)
        o = torch.softmax(s, -1) @ v
        outs.append(o.transpose(1, 2).reshape(n_seq * seq, d))
    return torch.cat(outs, 1)


@pytest.mark.parametrize("dtype", [FPK_DTYPE_F16, FPK_DTYPE_BF16, FPK_DTYPE_F32, FPK_DTYPE_F32_EXACT])
@pytest.mark.parametrize("seq,n_seq,layers", [(400, 3, 2), (400, 5, 1), (77, 4, 1), (130, 2, 2)])
def test_attention_matches_torch(fpk, dtype, seq, n_seq, layers):
    torch.backends.cuda.matmul.allow_tf32 = False
    heads = 4
    d = heads * 128
    g = torch.Generator().manual_seed(seq * 31 + n_seq)
    rows = seq * n_seq
    # Logit spread large enough that the running maximum moves between key
    # blocks (exercises the lazy O rescale).
    x = torch.randn(rows, layers * 3 * d, generator=g) * 1.5
    dt = DT[dtype]
    qkv = Planar(rows, layers * 3 * d, dt).set(x.to(DEV))
    out = Planar(rows, layers * d, dt)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    attention(fpk, qkv.base, qkv.plane_stride, 3 * d, 0, d, 2 * d, out.base, out.plane_stride, d, layers,
              heads, seq, n_seq, dtype, err.data_ptr())
    torch.cuda.synchronize()
    assert err.item() == 0
    ref = reference(x.to(dt).float().to(DEV), layers, heads, seq, n_seq)
    got = out.get().float()
    scale = ref.abs().max().item()
    e = (got - ref).abs().max().item()
    assert e <= TOL[dtype] * scale, f"max err {e:.3e} vs scale {scale:.3e}"
    # Guard rows of the output stay untouched.
    assert torch.count_nonzero(out.t[:, :256]) == 0


def test_attention_rejects_bad_arguments(fpk):
    from fp_b200.kernels import FpkError

    t = torch.zeros(16, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    with pytest.raises(FpkError, match="dtype"):
        attention(fpk, t.data_ptr(), 256, 1536, 0, 512, 1024, t.data_ptr(), 256, 512, 1, 4, 400, 1, 9,
                  err.data_ptr())
    with pytest.raises(FpkError, match="aligned"):
        attention(fpk, t.data_ptr() + 4, 256, 1536, 0, 512, 1024, t.data_ptr(), 256, 512, 1, 4, 400, 1,
                  FPK_DTYPE_F16, err.data_ptr())
