"""GPU parity of RefineNet / ScoreNet (fpk_net_*, tcgen05 GEMMs + attention)
against the torch fp32 reference (oracle/fp_net_ref.py) on the same weight
pack and inputs. Bar: outputs within 1e-2 relative at FP16/BF16, 1e-3 at TF32
(fp32 activations rounded to nearest TF32 where produced, TF32 tensor-core
multiplies, fp32 accumulation) and 1e-4 at FP32 (strict: every GEMM the sum of
three TF32 products of split operands, attention in fp32 FMA arithmetic),
relative to the output's largest magnitude, per output tensor."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from fp_b200.kernels import Networks  # noqa: E402
from fp_b200.weights import make_default_packs, read_pack  # noqa: E402

sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "oracle"))
from fp_net_ref import NetRef  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = "cuda"
FP32, TF32, FP16, BF16 = 0, 1, 2, 3
# FP32 is strict (split-operand GEMMs, fp32 attention): fp32-accurate; TF32
# runs TF32 products with fp32 accumulation.
TOL = {FP32: 1e-4, TF32: 1e-3, FP16: 1e-2, BF16: 1e-2}


@pytest.fixture(scope="module")
def packs(tmp_path_factory):
    return make_default_packs(tmp_path_factory.mktemp("packs"), seed=7)


def inputs(n, seed):
    g = torch.Generator().manual_seed(seed)
    rgb = torch.rand(2, n, 3, 160, 160, generator=g)
    xyz = (torch.randn(2, n, 3, 160, 160, generator=g) * 0.5).clamp(-1.9, 1.9)
    xyz = xyz * (torch.rand(2, n, 1, 160, 160, generator=g) > 0.3)
    x = torch.cat([rgb, xyz], 2).float()
    return x[0].contiguous().to(DEV), x[1].contiguous().to(DEV)


def rel_err(got, want):
    return ((got.float() - want.float()).abs().max() / (want.float().abs().max() + 1e-6)).item()


@pytest.fixture(scope="module")
def ref_models(packs):
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    return (NetRef(read_pack(packs[0])[1], device=DEV), NetRef(read_pack(packs[1])[1], device=DEV))


@pytest.mark.parametrize("precision", [FP32, TF32, FP16, BF16])
def test_refine_matches_reference(fpk, packs, ref_models, precision):
    n = 3
    A, B = inputs(n, 1)
    net = Networks(fpk, packs[0], packs[1], precision, max_batch=8)
    trans = torch.zeros(n, 3, device=DEV)
    rot = torch.zeros(n, 3, device=DEV)
    net.refine(A.data_ptr(), B.data_ptr(), n, trans.data_ptr(), rot.data_ptr())
    torch.cuda.synchronize()
    assert net.error_flag() == 0
    rt, rr = ref_models[0].refine(A, B)
    e_t, e_r = rel_err(trans, rt), rel_err(rot, rr)
    print(f"refine precision={precision} rel err trans {e_t:.2e} rot {e_r:.2e}")
    assert e_t <= TOL[precision] and e_r <= TOL[precision]
    net.close()


@pytest.mark.parametrize("precision", [FP32, TF32, FP16, BF16])
def test_score_matches_reference(fpk, packs, ref_models, precision):
    n = 6
    A, B = inputs(n, 2)
    net = Networks(fpk, packs[0], packs[1], precision, max_batch=8)
    scores = torch.zeros(n, device=DEV)
    net.score(A.data_ptr(), B.data_ptr(), n, scores.data_ptr())
    torch.cuda.synchronize()
    assert net.error_flag() == 0
    rs = ref_models[1].score(A, B)
    e = rel_err(scores, rs)
    print(f"score precision={precision} rel err {e:.2e} argmax {scores.argmax().item()} vs {rs.argmax().item()}")
    assert e <= TOL[precision]
    net.close()


@pytest.mark.parametrize("precision", [FP16, BF16])
def test_score_matches_reference_at_252(fpk, packs, ref_models, precision):
    """ScoreNet over the full register batch: the cross-hypothesis attention
    attends across all 252 hypotheses (reference tensorrt_runner.cu:523-532
    never micro-batches ScoreNet)."""
    n = 252
    A, B = inputs(n, 4)
    net = Networks(fpk, packs[0], packs[1], precision, max_batch=n)
    scores = torch.zeros(n, device=DEV)
    net.score(A.data_ptr(), B.data_ptr(), n, scores.data_ptr())
    torch.cuda.synchronize()
    assert net.error_flag() == 0
    rs = ref_models[1].score(A, B)
    e = rel_err(scores, rs)
    print(f"score n=252 precision={precision} rel err {e:.2e} argmax {scores.argmax().item()} vs {rs.argmax().item()}")
    assert e <= TOL[precision]
    net.close()


def test_refine_batch_independence(fpk, packs):
    """RefineNet is per-hypothesis: a hypothesis gives the same output inside
    batches of any size >= 2 (deterministic kernels, no cross-sample
    reductions). Alone (the tracking pass) its layers split K across CTAs, a
    different fp32 summation order: equal to the batched result within fp32
    rounding, and bit-identical run to run."""
    A, B = inputs(4, 3)
    net = Networks(fpk, packs[0], packs[1], FP16, max_batch=8)

    def run(a, b, n):
        t = torch.zeros(n, 3, device=DEV)
        r = torch.zeros(n, 3, device=DEV)
        net.refine(a.data_ptr(), b.data_ptr(), n, t.data_ptr(), r.data_ptr())
        torch.cuda.synchronize()
        return t, r

    t4, r4 = run(A, B, 4)
    t2, r2 = run(A[1:3].contiguous(), B[1:3].contiguous(), 2)
    assert torch.equal(t4[1:3], t2) and torch.equal(r4[1:3], r2)
    A1, B1 = A[2:3].contiguous(), B[2:3].contiguous()
    t1, r1 = run(A1, B1, 1)
    t1b, r1b = run(A1, B1, 1)
    assert torch.equal(t1, t1b) and torch.equal(r1, r1b)
    assert net.error_flag() == 0
    assert rel_err(t1[0], t4[2]) <= 2e-3 and rel_err(r1[0], r4[2]) <= 2e-3
    net.close()
