"""GPU parity of the per-layer kernels against the CPU oracle (KERNEL arithmetic = the
reference CUDA kernels'): every byte must match. Random stores as the reference's own unit tests
(`unit_conv1` / `unit_conv2`, kaggle/int8_pack/pack_dense8s.py:247-320); the output buffers are
pre-filled with a sentinel so a missed write shows."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from rsna_knee_efficiency_b200 import ops
from tests.helpers import dev, pixels_to_planes, planes_to_pixels, plan_tables, rand_store, split_store, tile_major

pytestmark = pytest.mark.gpu

# (block, layer) checked by the reference (pack_dense8s.py:863-864)
REF_LAYERS = [(0, 0), (0, 5), (1, 0), (1, 7), (2, 20), (3, 0), (3, 31)]


def _conv1_case(par, bi, li, c0, N, HW, f16, kind, seed):
    rng = np.random.default_rng(seed)
    cin = c0 + 32 * li
    X = rand_store(rng, (N, HW, cin), kind)
    in0, seg = split_store(X, c0)
    rows = N * HW
    out = torch.full((8 * rows * 16,), 0xA5, dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    segd = dev(seg) if li > 0 else torch.zeros(16, dtype=torch.int8, device="cuda")
    tab = par[f"L{bi}_{li}_abh"] if f16 else par[f"L{bi}_{li}_ab"]
    ops.conv1(dev(in0), segd, dev(ops.prepare_conv1_weights(par[f"L{bi}_{li}_w1"])), dev(tab),
              dev(par[f"L{bi}_{li}_gdu"]),
              out, c0 // 32, cin // 32, N, HW, f16, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    got = planes_to_pixels(out, rows)
    want = orc.conv1(X.reshape(rows, cin), par[f"L{bi}_{li}_w1"],
                     ab=None if f16 else par[f"L{bi}_{li}_ab"],
                     abh=par[f"L{bi}_{li}_abh"] if f16 else None,
                     gd=par[f"L{bi}_{li}_gdu"], mode=orc.KERNEL)
    return got, want


@pytest.mark.parametrize("bi,li", REF_LAYERS)
@pytest.mark.parametrize("f16", [True, False])
def test_conv1_ref_layers_512(bi, li, f16):
    _, plan, par = plan_tables(512)
    b = plan.blocks[bi]
    got, want = _conv1_case(par, bi, li, b.c0, 2, b.h * b.w, f16, "uniform", 100 * bi + li)
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("N,HW", [(3, 100), (1, 7), (5, 256), (2, 4)])
def test_conv1_ragged_rows(N, HW):
    """Row counts that are not multiples of the 128-row tile and tiles straddling images."""
    _, plan, par = plan_tables(512)
    got, want = _conv1_case(par, 1, 3, plan.blocks[1].c0, N, HW, True, "relu", 7 * N + HW)
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("bi,li,N,HW", [(0, 5, 2, 16384), (2, 20, 3, 1024), (3, 31, 2, 256), (1, 3, 3, 100),
                                         (1, 3, 1, 7)])
def test_conv1_tile_major_store(bi, li, N, HW):
    """The tile-major block store ([tiles][tile_groups][128][32]) gives the oracle's bytes too,
    including a partial last tile and a CTA pair whose second CTA has no rows."""
    _, plan, par = plan_tables(512)
    c0 = plan.blocks[bi].c0
    cin = c0 + 32 * li
    G, Gt = cin // 32, cin // 32 + 3
    rows = N * HW
    X = rand_store(np.random.default_rng(11 * bi + li), (N, HW, cin), "uniform").reshape(rows, cin)
    tm = tile_major(X.reshape(N, HW, cin), Gt)
    out = torch.full((8 * rows * 16,), 0xA5, dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.conv1(dev(tm), None, dev(ops.prepare_conv1_weights(par[f"L{bi}_{li}_w1"])), dev(par[f"L{bi}_{li}_abh"]),
              dev(par[f"L{bi}_{li}_gdu"]), out, 0, G, N, HW, True, err=err, tile_groups=Gt)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    want = orc.conv1(X, par[f"L{bi}_{li}_w1"], ab=None, abh=par[f"L{bi}_{li}_abh"], gd=par[f"L{bi}_{li}_gdu"],
                     mode=orc.KERNEL)
    np.testing.assert_array_equal(planes_to_pixels(out, rows), want)


@pytest.mark.parametrize("N,HW", [(1, 7), (3, 100), (2, 256)])
def test_conv1_pairs_ragged_rows(N, HW):
    """A layer whose weights only fit half per CTA (block 4, layer 32: 51 K groups) runs on CTA
    pairs: 256-row tiles, including a pair whose second CTA has no rows."""
    _, plan, par = plan_tables(512)
    got, want = _conv1_case(par, 3, 31, plan.blocks[3].c0, N, HW, True, "relu", 5 * N + HW)
    np.testing.assert_array_equal(got, want)


def _conv2_case(par, bi, li, N, H, W, seed):
    rng = np.random.default_rng(seed)
    V = rng.integers(0, 80, size=(N, H, W, 128), dtype=np.int64).astype(np.uint8)
    rows = N * H * W
    out = torch.full((rows * 32,), 0x5A, dtype=torch.int8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.conv2(dev(pixels_to_planes(V.reshape(rows, 128))),
              dev(ops.prepare_conv2_weights(par[f"L{bi}_{li}_w2k"])),
              dev(par[f"L{bi}_{li}_c2u"]), out, N, H, W, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    got = out.view(N, H, W, 32).cpu().numpy()
    want = orc.conv2(V, par[f"L{bi}_{li}_w2k"], par[f"L{bi}_{li}_c2u"], orc.KERNEL)
    return got, want


@pytest.mark.parametrize("bi,li", [(0, 0), (1, 7), (2, 20), (3, 31)])
def test_conv2_ref_layers_512(bi, li):
    _, plan, par = plan_tables(512)
    b = plan.blocks[bi]
    got, want = _conv2_case(par, bi, li, 2, b.h, b.w, 7 + 100 * bi + li)
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("N,H,W", [(1, 16, 16), (3, 8, 8), (2, 2, 2), (1, 5, 72), (2, 9, 9), (1, 3, 128)])
def test_conv2_small_and_ragged(N, H, W):
    _, _, par = plan_tables(512)
    got, want = _conv2_case(par, 1, 2, N, H, W, N * 1000 + H * 10 + W)
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("N,H,W", [(1, 1, 128), (3, 5, 128), (2, 100, 128), (300, 4, 128), (10, 128, 128)])
def test_conv2_one_row_tiles(N, H, W):
    """W = 128 (tiles of one image row, the block-1 geometry): one-row images (both vertical taps in
    the zero padding), images of a few rows, and more tiles than CTAs so that CTAs take several
    tiles across image boundaries."""
    _, _, par = plan_tables(512)
    got, want = _conv2_case(par, 1, 2, N, H, W, N * 1000 + H * 10 + W)
    np.testing.assert_array_equal(got, want)


def _trans_case(par, plan, bi, N, H, W, f16, kind, seed):
    rng = np.random.default_rng(seed)
    b = plan.blocks[bi]
    c0, ctot = b.c0, b.c_tot
    X = rand_store(rng, (N, H * W, ctot), kind)
    in0, seg = split_store(X, c0)
    cout = ctot // 2
    out = torch.full((N * cout * (H // 2) * (W // 2),), 0x33, dtype=torch.int8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    tab = par[f"T{bi}_abh"] if f16 else par[f"T{bi}_ab"]
    ops.trans(dev(in0), dev(seg), dev(ops.prepare_trans_weights(par[f"T{bi}_w"])), dev(tab),
              dev(par[f"T{bi}_gd"]), out, c0 // 32, ctot // 32, N, H, W, f16, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    # next block's group-major in0 [G0n][N][HW/4][32] -> channel-last [N, H/2, W/2, cout]
    got = out.view(cout // 32, N, (H // 2) * (W // 2), 32).permute(1, 2, 0, 3).reshape(
        N, H // 2, W // 2, cout).cpu().numpy()
    want = orc.trans(X.reshape(N, H, W, ctot), par[f"T{bi}_w"],
                     ab=None if f16 else par[f"T{bi}_ab"], abh=par[f"T{bi}_abh"] if f16 else None,
                     gd=par[f"T{bi}_gd"], mode=orc.KERNEL)
    return got, want


@pytest.mark.parametrize("bi", [0, 1, 2])
@pytest.mark.parametrize("f16", [True, False])
def test_trans_512(bi, f16):
    _, plan, par = plan_tables(512)
    b = plan.blocks[bi]
    got, want = _trans_case(par, plan, bi, 2, b.h, b.w, f16, "uniform", 900 + bi)
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("bi,N,H,W", [(0, 3, 6, 10), (2, 2, 4, 4), (1, 1, 2, 2), (2, 5, 8, 6)])
def test_trans_small_and_ragged(bi, N, H, W):
    _, plan, par = plan_tables(512)
    got, want = _trans_case(par, plan, bi, N, H, W, True, "relu", 31 * bi + N + H + W)
    np.testing.assert_array_equal(got, want)


def _stem_case(par, x, flip, u8_planes):
    N, _, H, W = x.shape
    PH, PW = H // 4, W // 4
    out = torch.full((2 * N * PH * PW * 32,), 0x11, dtype=torch.int8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    flags = None if flip is None else dev(np.asarray(flip, np.int32))
    w8u, kc = dev(ops.prepare_stem_weights(par["S_w8"])), dev(par["S_kc"])
    if u8_planes:
        src = np.zeros((N, 4), np.int32)
        src[:, :3] = np.arange(3 * N).reshape(N, 3)
        ops.stem(dev(x.reshape(3 * N, H, W)), w8u, kc, out, N, H, W, src=dev(src), flags=flags, err=err)
    else:
        ops.stem(dev(x), w8u, kc, out, N, H, W, flags=flags, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    # group-major [2][N][PH*PW][32] -> channel-last [N, PH, PW, 64]
    got = out.view(2, N, PH * PW, 32).permute(1, 2, 0, 3).reshape(N, PH, PW, 64).cpu().numpy()
    want = orc.stem(x, par["S_w8f"], par["S_kc"], flip=flip, mode=orc.KERNEL)
    return got, want


@pytest.mark.parametrize("u8_planes", [True, False])
@pytest.mark.parametrize("flip", [None, [1, 0, 1]])
def test_stem_512(u8_planes, flip):
    from rsna_knee_efficiency_b200 import synth
    _, _, par = plan_tables(512)
    t = synth.triplets(synth.volume(5))[[0, 11, 23]]
    x = t if u8_planes else (t.astype(np.float32) / 255.0).astype(np.float16)
    got, want = _stem_case(par, x, flip, u8_planes)
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("H,W", [(64, 64), (32, 96), (128, 128), (16, 24)])
def test_stem_small_and_fp16_off_grid(H, W):
    """Small images, and fp16 pixels that are not k/255 (zoomed / interpolated windows)."""
    _, _, par = plan_tables(512)
    rng = np.random.default_rng(H * W)
    x = rng.uniform(-0.05, 1.05, size=(2, 3, H, W)).astype(np.float16)
    got, want = _stem_case(par, x, [0, 1], False)
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("N,HW", [(3, 256), (2, 4), (5, 16)])
def test_head(N, HW):
    _, plan, par = plan_tables(512)
    from rsna_knee_efficiency_b200 import densenet
    b = plan.blocks[3]
    rng = np.random.default_rng(N + HW)
    X = rand_store(rng, (N, HW, b.c_tot), "uniform")
    in0, seg = split_store(X, b.c0)
    head = densenet.random_head(3)
    hw = head.fc.weight.detach().numpy().astype(np.float32)
    hb = head.fc.bias.detach().numpy().astype(np.float32)
    feat = torch.zeros((N, b.c_tot), dtype=torch.float32, device="cuda")
    logits = torch.zeros((N, 4), dtype=torch.float32, device="cuda")
    per_view = 1 if N % 2 else 2
    views = torch.zeros((N // per_view, 4), dtype=torch.float32, device="cuda")
    tickets = torch.zeros(N // per_view, dtype=torch.int32, device="cuda")
    for _ in range(2):                                   # tickets must come back zeroed
        ops.head(dev(in0), dev(seg), dev(par["F_ab"]), b.c0 // 32, b.c_tot // 32, N, HW, feat=feat,
                 hw=dev(hw), hb=dev(hb), logits=logits, view_logits=views, tickets=tickets,
                 per_view=per_view)
    torch.cuda.synchronize()
    want_f = orc.final(X, par["F_ab"], orc.KERNEL)
    np.testing.assert_array_equal(feat.cpu().numpy(), want_f)        # bit-exact features
    want_l = orc.head(want_f, hw, hb)
    np.testing.assert_allclose(logits.cpu().numpy(), want_l, rtol=0, atol=1e-5)
    np.testing.assert_allclose(views.cpu().numpy(), want_l.reshape(-1, per_view, 4).mean(1), rtol=0, atol=1e-5)
    assert int(tickets.abs().sum().item()) == 0
