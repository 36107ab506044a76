"""GPU test of the bounded-wait error path of the tcgen05 GEMM.

With the failure-injection switch `fpk_gemm_test_withhold_loads` on, the
single-CTA kernel's producer issues no operand loads, so the MMA warp's
bounded mbarrier wait for the first tile runs out (~2 s; the epilogue warps may
give up first). The kernel must record the code of the wait that ran out in
the caller's error flag, leave the output untouched, and return with nothing in
flight: the same context then runs the same GEMM correctly. No fault, trap or
hang is involved: every wait in the kernel is bounded and the flag is an
ordinary device int."""
from __future__ import annotations

import math

import pytest

torch = pytest.importorskip("torch")

from fp_b200.kernels import FPK_DTYPE_BF16, gemm  # noqa: E402
from kp8_util import Planar  # noqa: E402
from test_gpu_gemm import DEV, chunk_major, close, make_desc  # noqa: E402

pytestmark = pytest.mark.gpu

# Error codes set by gemmKernel's waits: 14 = the MMA warp's wait for an
# activation window, 17 = the epilogue's wait for a finished accumulator
# (both start waiting at once; whichever limit passes first records its code).
TIMEOUT_CODES = (14, 17)


def _case(m=1000, cin=64, cout=64):
    g = torch.Generator().manual_seed(7)
    A = torch.randn(m, cin, generator=g)
    W = torch.randn(cout, cin, generator=g) / math.sqrt(cin)
    b = torch.randn(cout, generator=g).to(DEV)
    pa = Planar(m, cin, torch.bfloat16).set(A.to(DEV))
    w = chunk_major(W.reshape(cout, 1, cin), FPK_DTYPE_BF16).to(torch.bfloat16).to(DEV)
    ref = A.to(torch.bfloat16).float().to(DEV) @ W.to(torch.bfloat16).float().to(DEV).T + b
    return pa, w, b, ref


def test_withheld_load_times_out_and_context_recovers(fpk):
    m, cin, cout = 1000, 64, 64
    pa, w, b, ref = _case(m, cin, cout)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = Planar(m, cout, torch.bfloat16)
    prev = fpk.lib.fpk_gemm_test_withhold_loads(1)
    try:
        gemm(fpk, make_desc(pa, m, cin, [0], w, cout, out, FPK_DTYPE_BF16, err, bias=b))
        torch.cuda.synchronize()  # returns: the kernel gave up on its own
    finally:
        fpk.lib.fpk_gemm_test_withhold_loads(prev)
    assert err.item() in TIMEOUT_CODES, f"error flag {err.item()}"
    assert torch.count_nonzero(out.t) == 0  # nothing was stored

    # The context is intact: the same launch now completes and is correct.
    err.zero_()
    gemm(fpk, make_desc(pa, m, cin, [0], w, cout, out, FPK_DTYPE_BF16, err, bias=b))
    torch.cuda.synchronize()
    assert err.item() == 0
    close(out.get(), ref)


def test_raised_flag_stops_later_launches_quickly(fpk):
    """A flag already raised (by an earlier timed-out layer) makes the next
    launch on the same flag give up after a few hundred polls instead of the
    full limit, so a failed network call ends promptly."""
    import time

    m, cin, cout = 1000, 64, 64
    pa, w, b, _ = _case(m, cin, cout)
    err = torch.full((1,), 99, dtype=torch.int32, device=DEV)
    out = Planar(m, cout, torch.bfloat16)
    prev = fpk.lib.fpk_gemm_test_withhold_loads(1)
    try:
        t0 = time.perf_counter()
        gemm(fpk, make_desc(pa, m, cin, [0], w, cout, out, FPK_DTYPE_BF16, err, bias=b))
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
    finally:
        fpk.lib.fpk_gemm_test_withhold_loads(prev)
    assert err.item() == 99  # the first error code is kept
    assert dt < 0.5, f"launch took {dt:.3f} s with the flag raised"
