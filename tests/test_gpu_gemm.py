"""GPU tests of the tcgen05 implicit-GEMM kernel (fpk_gemm) against torch fp32
on the same half-precision-rounded operands (fp16/bf16), or on fp32 operands
multiplied as TF32. Tolerance: 1e-2 of the output's max magnitude (fp16/bf16
output rounding or TF32 operand rounding; fp32 accumulation)."""
from __future__ import annotations

import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.nn.functional as F  # noqa: E402

from fp_b200.kernels import (FPK_DST_S2D, FPK_DST_SAME, FPK_DST_TOKENS, FPK_DTYPE_BF16,  # noqa: E402
                             FPK_DTYPE_F16, FPK_DTYPE_F32, FPK_DTYPE_F32_EXACT, GemmDesc, gemm)
from kp8_util import Planar  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = "cuda"
DT = {FPK_DTYPE_BF16: torch.bfloat16, FPK_DTYPE_F16: torch.float16, FPK_DTYPE_F32: torch.float32,
      FPK_DTYPE_F32_EXACT: torch.float32}


def make_desc(a: Planar, rows, cin, taps_off, w, cout, dst: Planar, dtype, err, bias=None,
              residual: Planar | None = None, relu=False, mode=FPK_DST_SAME, img_rows=None,
              grid_w=1, valid_h=None, valid_w=1, dst_img_rows=0, dst_grid_w=0, pos=None):
    d = GemmDesc()
    d.a, d.a_plane_stride, d.rows, d.cin = a.base, a.plane_stride, rows, cin
    d.taps = len(taps_off)
    for i, o in enumerate(taps_off):
        d.tap_off[i] = int(o)
    d.w, d.cout = w.data_ptr(), cout
    d.bias = bias.data_ptr() if bias is not None else None
    d.residual = residual.base if residual is not None else None
    d.res_plane_stride = residual.plane_stride if residual is not None else 0
    d.relu = int(relu)
    d.dst, d.dst_plane_stride, d.dst_mode = dst.base, dst.plane_stride, mode
    d.img_rows = img_rows or rows
    d.grid_w, d.valid_h, d.valid_w = grid_w, valid_h or (img_rows or rows), valid_w
    d.dst_img_rows, d.dst_grid_w, d.img_mod, d.ch_step = dst_img_rows, dst_grid_w, 1, 0
    d.pos = pos.data_ptr() if pos is not None else None
    d.dtype = dtype
    d.error_flag = err.data_ptr()
    return d


def chunk_major(w_taps: torch.Tensor, dtype=FPK_DTYPE_BF16) -> torch.Tensor:
    """[cout, taps, cin] -> [cout, K'] with k' = chunk*(taps*cw) + tap*cw + c and
    cw = the channels of one 128-byte chunk (64 for 16-bit types, 32 for fp32)."""
    cout, taps, cin = w_taps.shape
    cw = min(cin, 32 if dtype in (FPK_DTYPE_F32, FPK_DTYPE_F32_EXACT) else 64)
    return (w_taps.reshape(cout, taps, cin // cw, cw).permute(0, 2, 1, 3)
            .reshape(cout, taps * cin).contiguous())


def close(got: torch.Tensor, want: torch.Tensor, tol=1e-2):
    scale = want.abs().max().item() + 1e-6
    err = (got.float() - want.float()).abs().max().item()
    assert err <= tol * scale, f"max err {err:.3e} vs scale {scale:.3e}"


@pytest.fixture()
def err():
    return torch.zeros(1, dtype=torch.int32, device=DEV)


@pytest.fixture(params=[1, 0], ids=["pairs", "single"])
def cta_pairs(request, fpk):
    """Runs a test with CTA-pair tiles allowed (the default: layers with
    256-channel tiles, and 64- or 128-channel layers, take them when their rows
    fill every pair of SMs) and with every layer on single-CTA tiles."""
    prev = fpk.lib.fpk_gemm_set_cta_pairs(request.param)
    yield request.param
    fpk.lib.fpk_gemm_set_cta_pairs(prev)


@pytest.mark.parametrize("m,cin,cout,dtype", [(1000, 64, 64, FPK_DTYPE_BF16),
                                              (777, 128, 128, FPK_DTYPE_F16),
                                              (2000, 256, 256, FPK_DTYPE_BF16),
                                              (513, 512, 512, FPK_DTYPE_BF16),
                                              (4096, 512, 1536, FPK_DTYPE_F16),
                                              (777, 128, 128, FPK_DTYPE_F32),
                                              (777, 128, 256, FPK_DTYPE_F32_EXACT),
                                              (4096, 512, 1536, FPK_DTYPE_F32),
                                              # > 2 x 148 tiles of 128 rows: 256-row tiles with
                                              # one accumulator buffer for 1x1 layers
                                              (40000, 512, 768, FPK_DTYPE_F16),
                                              (40000, 256, 512, FPK_DTYPE_F32),
                                              # pair tiles in BF16 with a ragged last pair
                                              # tile; 128-wide windows of a 1x1 layer
                                              (37001, 256, 256, FPK_DTYPE_BF16),
                                              # 128-channel layers on 256-row tiles
                                              (40000, 256, 128, FPK_DTYPE_F16),
                                              (38000, 128, 128, FPK_DTYPE_F32),
                                              (20111, 512, 1536, FPK_DTYPE_BF16)])
def test_plain_gemm(fpk, err, cta_pairs, m, cin, cout, dtype):
    g = torch.Generator().manual_seed(m + cin)
    dt = DT[dtype]
    A = torch.randn(m, cin, generator=g)
    W = torch.randn(cout, cin, generator=g) / math.sqrt(cin)
    b = torch.randn(cout, generator=g).to(DEV)
    pa = Planar(m, cin, dt).set(A.to(DEV))
    out = Planar(m, cout, dt)
    w = chunk_major(W.reshape(cout, 1, cin), dtype).to(dt).to(DEV)
    gemm(fpk, make_desc(pa, m, cin, [0], w, cout, out, dtype, err, bias=b))
    torch.cuda.synchronize()
    assert err.item() == 0
    ref = A.to(dt).float().to(DEV) @ W.to(dt).float().to(DEV).T + b
    close(out.get(), ref)
    # Rows outside [0, m) of the destination (guard rows) were not touched.
    assert torch.count_nonzero(out.t[:, :256]) == 0


# n=24 images of 40x40 give more than 2 x 148 tiles of 128 rows, which
# selects the 256-row tiles (two accumulators per weight stage) for the
# layers of at most 128 output channels.
@pytest.mark.parametrize("cin,cout,hw,dtype,n", [(64, 128, 20, FPK_DTYPE_BF16, 3),
                                                 (128, 128, 40, FPK_DTYPE_F16, 3),
                                                 (128, 128, 40, FPK_DTYPE_F16, 24),
                                                 (64, 64, 40, FPK_DTYPE_BF16, 24),
                                                 (256, 256, 40, FPK_DTYPE_BF16, 3),
                                                 (128, 128, 40, FPK_DTYPE_F32, 24),
                                                 (256, 256, 40, FPK_DTYPE_F32, 3),
                                                 (512, 512, 20, FPK_DTYPE_BF16, 3),
                                                 # enough rows for pair tiles at 256 channels
                                                 (256, 256, 40, FPK_DTYPE_F16, 25),
                                                 (512, 512, 20, FPK_DTYPE_BF16, 64),
                                                 (256, 256, 40, FPK_DTYPE_F32, 25)])
def test_conv3x3_residual_relu(fpk, err, cta_pairs, cin, cout, hw, dtype, n):
    g = torch.Generator().manual_seed(cin * 7 + hw + n)
    dt = DT[dtype]
    H, W = hw, hw
    gw = W + 1
    img_rows = (H + 1) * gw
    rows = n * img_rows
    X = torch.randn(n, cin, H, W, generator=g)
    R = torch.randn(n, cout, H, W, generator=g)
    Wt = torch.randn(cout, cin, 3, 3, generator=g) / math.sqrt(9 * cin)
    b = torch.randn(cout, generator=g).to(DEV)

    def to_grid(t):  # [n,C,H,W] -> [rows, C] on the (H+1)x(W+1) grid, zero border row/col
        c = t.shape[1]
        z = torch.zeros(n, H + 1, W + 1, c)
        z[:, :H, :W] = t.permute(0, 2, 3, 1)
        return z.reshape(rows, c)

    pa = Planar(rows, cin, dt).set(to_grid(X).to(DEV))
    pr = Planar(rows, cout, dt).set(to_grid(R).to(DEV))
    out = Planar(rows, cout, dt)
    taps = [(ky - 1) * gw + (kx - 1) for ky in range(3) for kx in range(3)]
    w = chunk_major(Wt.permute(0, 2, 3, 1).reshape(cout, 9, cin), dtype).to(dt).to(DEV)
    gemm(fpk, make_desc(pa, rows, cin, taps, w, cout, out, dtype, err, bias=b, residual=pr,
                        relu=True, img_rows=img_rows, grid_w=gw, valid_h=H, valid_w=W))
    torch.cuda.synchronize()
    assert err.item() == 0
    ref = F.conv2d(X.to(dt).float().to(DEV), Wt.to(dt).float().to(DEV), b, padding=1)
    ref = torch.relu(ref + R.to(dt).float().to(DEV))
    got = out.get().reshape(n, H + 1, W + 1, cout)
    close(got[:, :H, :W], ref.permute(0, 2, 3, 1))
    # The zero border row/column of the output grid stays zero.
    assert torch.count_nonzero(got[:, H]) == 0 and torch.count_nonzero(got[:, :, W]) == 0


def s2d_weights(Wt: torch.Tensor, stride_taps: int, sub_offset: int) -> torch.Tensor:
    """Stride-2 conv weights [cout, cin, k, k] -> taps over space-to-depth input:
    tap (a, b) in stride_taps^2, channel (sub=(dy,dx), c) with k index 2a+dy."""
    cout, cin, k, _ = Wt.shape
    out = torch.zeros(cout, stride_taps * stride_taps, 4 * cin)
    for a in range(stride_taps):
        for bb in range(stride_taps):
            for dy in range(2):
                for dx in range(2):
                    ky, kx = 2 * a + dy, 2 * bb + dx
                    if ky < k and kx < k:
                        sub = dy * 2 + dx
                        out[:, a * stride_taps + bb, sub * cin:(sub + 1) * cin] = Wt[:, :, ky, kx]
    return out


@pytest.mark.parametrize("dtype", [FPK_DTYPE_BF16, FPK_DTYPE_F16, FPK_DTYPE_F32])
def test_s2d_stride2_conv(fpk, err, dtype):
    """1x1 layer writing space-to-depth, then a 3x3 stride-2 conv as a 2x2 conv."""
    g = torch.Generator().manual_seed(5)
    dt = DT[dtype]
    n, H2, c1, c2 = 2, 40, 64, 128
    H = H2 // 2
    gw1 = H2 + 1
    rows1 = n * (H2 + 1) * gw1
    X = torch.randn(n, c1, H2, H2, generator=g)
    W1 = torch.randn(c1, c1, generator=g) / math.sqrt(c1)
    W2 = torch.randn(c2, c1, 3, 3, generator=g) / math.sqrt(9 * c1)
    b1 = torch.zeros(c1).to(DEV)
    b2 = torch.randn(c2, generator=g).to(DEV)
    z = torch.zeros(n, H2 + 1, H2 + 1, c1)
    z[:, :H2, :H2] = X.permute(0, 2, 3, 1)
    pa = Planar(rows1, c1, dt).set(z.reshape(rows1, c1).to(DEV))
    gw2 = H + 1
    rows2 = n * (H + 1) * gw2
    t2 = Planar(rows2, 4 * c1, dt)
    w1 = chunk_major(W1.reshape(c1, 1, c1), dtype).to(dt).to(DEV)
    gemm(fpk, make_desc(pa, rows1, c1, [0], w1, c1, t2, dtype, err, bias=b1, relu=False,
                        mode=FPK_DST_S2D, img_rows=(H2 + 1) * gw1, grid_w=gw1, valid_h=H2,
                        valid_w=H2, dst_img_rows=(H + 1) * gw2, dst_grid_w=gw2))
    out = Planar(rows2, c2, dt)
    taps = [a * gw2 + bb for a in range(2) for bb in range(2)]
    w2 = chunk_major(s2d_weights(W2, 2, 1), dtype).to(dt).to(DEV)
    gemm(fpk, make_desc(t2, rows2, 4 * c1, taps, w2, c2, out, dtype, err, bias=b2, relu=True,
                        img_rows=(H + 1) * gw2, grid_w=gw2, valid_h=H, valid_w=H))
    torch.cuda.synchronize()
    assert err.item() == 0
    y = torch.einsum("nchw,dc->ndhw", X.to(dt).float(), W1.to(dt).float()).to(dt).float()
    ref = torch.relu(F.conv2d(y.to(DEV), W2.to(dt).float().to(DEV), b2, stride=2, padding=1))
    got = out.get().reshape(n, H + 1, gw2, c2)[:, :H, :H]
    close(got, ref.permute(0, 2, 3, 1))


@pytest.mark.parametrize("dtype,n", [(FPK_DTYPE_BF16, 2), (FPK_DTYPE_F16, 8), (FPK_DTYPE_F32, 8)])
def test_stem_7x7_stride2(fpk, err, cta_pairs, dtype, n):
    """7x7 stride-2 pad-3 conv over 6 channels as a 16-tap conv on the 32-channel
    space-to-depth layout the fused render+pack writes (grid 83 for 160 crops)."""
    g = torch.Generator().manual_seed(9)
    dt = DT[dtype]
    S, cin, cout = 160, 6, 64
    gs = (S + 7) // 2  # 83
    X = torch.randn(n, cin, S, S, generator=g)
    Wt = torch.randn(cout, cin, 7, 7, generator=g) / math.sqrt(49 * cin)
    b = torch.randn(cout, generator=g).to(DEV)
    # Space-to-depth input: cell (gy, gx), sub (dy, dx) holds in[2gy+dy-3, 2gx+dx-3].
    T = torch.zeros(n, gs, gs, 4, 8)
    xp = torch.zeros(n, cin, 2 * gs, 2 * gs)
    xp[:, :, 3:3 + S, 3:3 + S] = X
    for dy in range(2):
        for dx in range(2):
            T[:, :, :, dy * 2 + dx, :cin] = xp[:, :, dy::2, dx::2].permute(0, 2, 3, 1)
    rows = n * gs * gs
    pa = Planar(rows, 32, dt).set(T.reshape(rows, 32).to(DEV))
    Wp = torch.zeros(cout, cin + 2, 7, 7)
    Wp[:, :cin] = Wt
    w = chunk_major(s2d_weights(Wp, 4, 3), dtype).to(dt).to(DEV)
    out = Planar(rows, cout, dt)
    taps = [a * gs + bb for a in range(4) for bb in range(4)]
    gemm(fpk, make_desc(pa, rows, 32, taps, w, cout, out, dtype, err, bias=b, relu=True,
                        img_rows=gs * gs, grid_w=gs, valid_h=S // 2, valid_w=S // 2))
    torch.cuda.synchronize()
    assert err.item() == 0
    ref = torch.relu(F.conv2d(X.to(dt).float().to(DEV), Wt.to(dt).float().to(DEV), b, stride=2,
                              padding=3))
    got = out.get().reshape(n, gs, gs, cout)[:, :S // 2, :S // 2]
    close(got, ref.permute(0, 2, 3, 1))


@pytest.mark.parametrize("n", [3, 200])
def test_tokens_epilogue(fpk, err, cta_pairs, n):
    g = torch.Generator().manual_seed(3)
    dt = torch.bfloat16
    H, cin, cout = 20, 128, 256
    gw = H + 1
    rows = n * (H + 1) * gw
    X = torch.randn(n, H, H, cin, generator=g)
    z = torch.zeros(n, H + 1, gw, cin)
    z[:, :H, :H] = X
    Wt = torch.randn(cout, cin, generator=g) / math.sqrt(cin)
    pos = torch.randn(H * H, cout, generator=g).to(DEV)
    pa = Planar(rows, cin, dt).set(z.reshape(rows, cin).to(DEV))
    out = Planar(n * H * H, cout, dt)
    w = chunk_major(Wt.reshape(cout, 1, cin)).to(dt).to(DEV)
    gemm(fpk, make_desc(pa, rows, cin, [0], w, cout, out, FPK_DTYPE_BF16, err, relu=True,
                        mode=FPK_DST_TOKENS, img_rows=(H + 1) * gw, grid_w=gw, valid_h=H,
                        valid_w=H, pos=pos))
    torch.cuda.synchronize()
    assert err.item() == 0
    ref = torch.relu(X.reshape(n, H * H, cin).to(dt).float().to(DEV) @ Wt.to(dt).float().to(DEV).T)
    ref = ref + pos[None]
    close(out.get().reshape(n, H * H, cout), ref)


@pytest.mark.parametrize("dtype,cout,cin", [(FPK_DTYPE_F16, 256, 256), (FPK_DTYPE_BF16, 512, 256),
                                            (FPK_DTYPE_F32, 256, 256), (FPK_DTYPE_F16, 128, 128),
                                            (FPK_DTYPE_BF16, 128, 256), (FPK_DTYPE_F32, 128, 128)])
def test_pair_tiles_equal_single_tiles(fpk, err, dtype, cout, cin):
    """A 3x3 conv with enough rows for pair tiles gives the same bits on CTA
    pairs (M=256 cta_group::2 MMAs; 512-row pair tiles at 128 channels) as on
    single-CTA tiles: both accumulate every output over the same K sequence in
    fp32."""
    g = torch.Generator().manual_seed(11)
    dt = DT[dtype]
    n, H = 30, 40
    gw = H + 1
    img_rows = (H + 1) * gw
    rows = n * img_rows
    z = torch.zeros(n, H + 1, gw, cin)
    z[:, :H, :H] = torch.randn(n, H, H, cin, generator=g)
    Wt = torch.randn(cout, 9, cin, generator=g) / math.sqrt(9 * cin)
    b = torch.randn(cout, generator=g).to(DEV)
    pa = Planar(rows, cin, dt).set(z.reshape(rows, cin).to(DEV))
    w = chunk_major(Wt, dtype).to(dt).to(DEV)
    taps = [(ky - 1) * gw + (kx - 1) for ky in range(3) for kx in range(3)]
    outs = []
    pr = Planar(rows, cout, dt).set(torch.randn(rows, cout, generator=g).to(DEV))
    for pairs in (1, 0):
        prev = fpk.lib.fpk_gemm_set_cta_pairs(pairs)
        try:
            out = Planar(rows, cout, dt)
            gemm(fpk, make_desc(pa, rows, cin, taps, w, cout, out, dtype, err, bias=b, residual=pr,
                                relu=True, img_rows=img_rows, grid_w=gw, valid_h=H, valid_w=H))
            torch.cuda.synchronize()
        finally:
            fpk.lib.fpk_gemm_set_cta_pairs(prev)
        assert err.item() == 0
        outs.append(out.get())
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("rows,cin,cout,dtype,res,relu", [(100800, 512, 1536, FPK_DTYPE_F16, False, False),
                                                          (100800, 512, 512, FPK_DTYPE_F16, True, False),
                                                          (40000, 512, 512, FPK_DTYPE_BF16, False, True),
                                                          # ragged last pair tile: rows past the end clipped
                                                          (37001, 256, 256, FPK_DTYPE_BF16, True, True)])
def test_staged_stores_equal_thread_stores(fpk, err, rows, cin, cout, dtype, res, relu):
    """Dense 16-bit layers on CTA pairs leave the epilogue as bulk tensor stores
    of staged 32-column chunks: the same bits as per-thread stores, against
    torch, and nothing written outside the layer's rows (guard rows stay 0)."""
    g = torch.Generator().manual_seed(rows + cout)
    dt = DT[dtype]
    A = torch.randn(rows, cin, generator=g)
    W = torch.randn(cout, cin, generator=g) / math.sqrt(cin)
    b = torch.randn(cout, generator=g).to(DEV)
    pa = Planar(rows, cin, dt).set(A.to(DEV))
    w = chunk_major(W.reshape(cout, 1, cin), dtype).to(dt).to(DEV)
    pr = Planar(rows, cout, dt).set(torch.randn(rows, cout, generator=g).to(DEV)) if res else None
    outs = []
    for staged in (1, 0):
        prev = fpk.lib.fpk_gemm_set_tma_store(staged)
        try:
            out = Planar(rows, cout, dt)
            gemm(fpk, make_desc(pa, rows, cin, [0], w, cout, out, dtype, err, bias=b, residual=pr, relu=relu))
            torch.cuda.synchronize()
        finally:
            fpk.lib.fpk_gemm_set_tma_store(prev)
        assert err.item() == 0
        assert torch.count_nonzero(out.t[:, :256]) == 0 and torch.count_nonzero(out.t[:, 256 + rows:]) == 0
        outs.append(out.get())
    assert torch.equal(outs[0], outs[1])
    ref = A.to(dt).float().to(DEV) @ W.to(dt).float().to(DEV).T + b
    if res:
        ref = ref + pr.get().float()
    if relu:
        ref = torch.relu(ref)
    close(outs[0], ref)


# Split K (tracking one hypothesis): few output tiles, so each tile's K range
# is split over several CTAs whose fp32 partial sums a second launch adds in
# split order. Checked against torch, against the unsplit kernel, and for
# run-to-run bit identity.
@pytest.mark.parametrize("cin,cout,hw,dtype", [(256, 256, 40, FPK_DTYPE_F16), (512, 512, 20, FPK_DTYPE_BF16),
                                               (128, 128, 40, FPK_DTYPE_F16), (256, 256, 40, FPK_DTYPE_F32)])
def test_split_k_conv3x3(fpk, err, cin, cout, hw, dtype):
    g = torch.Generator().manual_seed(cin + hw)
    dt = DT[dtype]
    H = W = hw
    gw = W + 1
    img_rows = (H + 1) * gw
    X = torch.randn(1, cin, H, W, generator=g)
    R = torch.randn(1, cout, H, W, generator=g)
    Wt = torch.randn(cout, cin, 3, 3, generator=g) / math.sqrt(9 * cin)
    b = torch.randn(cout, generator=g).to(DEV)

    def to_grid(t):
        z = torch.zeros(1, H + 1, W + 1, t.shape[1])
        z[:, :H, :W] = t.permute(0, 2, 3, 1)
        return z.reshape(img_rows, t.shape[1])

    pa = Planar(img_rows, cin, dt).set(to_grid(X).to(DEV))
    pr = Planar(img_rows, cout, dt).set(to_grid(R).to(DEV))
    taps = [(ky - 1) * gw + (kx - 1) for ky in range(3) for kx in range(3)]
    w = chunk_major(Wt.permute(0, 2, 3, 1).reshape(cout, 9, cin), dtype).to(dt).to(DEV)
    ws = torch.zeros(24 << 20, dtype=torch.uint8, device=DEV)
    outs = []
    for split in (False, True, True):
        out = Planar(img_rows, cout, dt)
        d = make_desc(pa, img_rows, cin, taps, w, cout, out, dtype, err, bias=b, residual=pr, relu=True,
                      img_rows=img_rows, grid_w=gw, valid_h=H, valid_w=W)
        if split:
            d.splitk_ws, d.splitk_ws_bytes = ws.data_ptr(), ws.numel()
        gemm(fpk, d)
        torch.cuda.synchronize()
        assert err.item() == 0
        outs.append(out.get().reshape(H + 1, W + 1, cout))
    assert torch.count_nonzero(ws) > 0, "the split path did not run"
    assert torch.equal(outs[1], outs[2]), "split-K results must be identical run to run"
    ref = F.conv2d(X.to(dt).float().to(DEV), Wt.to(dt).float().to(DEV), b, padding=1)
    ref = torch.relu(ref + R.to(dt).float().to(DEV))[0].permute(1, 2, 0)
    close(outs[1][:H, :W], ref)
    close(outs[1], outs[0])
    assert torch.count_nonzero(outs[1][H]) == 0 and torch.count_nonzero(outs[1][:, W]) == 0


def test_split_k_tokens_linear(fpk, err):
    """The 400-token linears of one hypothesis (TOKENS destination with the
    positional embedding) through the split path."""
    g = torch.Generator().manual_seed(3)
    dt = torch.float16
    m, cin, cout = 400, 512, 1536
    A = torch.randn(m, cin, generator=g)
    Wm = torch.randn(cout, cin, generator=g) / math.sqrt(cin)
    b = torch.randn(cout, generator=g).to(DEV)
    pos = (torch.randn(m, cout, generator=g) * 0.1).to(DEV)
    pa = Planar(m, cin, dt).set(A.to(DEV))
    out = Planar(m, cout, dt)
    w = chunk_major(Wm.reshape(cout, 1, cin), FPK_DTYPE_F16).to(dt).to(DEV)
    ws = torch.zeros(24 << 20, dtype=torch.uint8, device=DEV)
    d = make_desc(pa, m, cin, [0], w, cout, out, FPK_DTYPE_F16, err, bias=b, mode=FPK_DST_TOKENS,
                  img_rows=m, grid_w=20, valid_h=20, valid_w=20, pos=pos)
    d.splitk_ws, d.splitk_ws_bytes = ws.data_ptr(), ws.numel()
    gemm(fpk, d)
    torch.cuda.synchronize()
    assert err.item() == 0 and torch.count_nonzero(ws) > 0
    ref = A.to(dt).float().to(DEV) @ Wm.to(dt).float().to(DEV).T + b + pos
    close(out.get(), ref)
