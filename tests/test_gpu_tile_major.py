"""The tile-major block store on the GPU: every kernel that writes or reads it (stem, conv2, the
transition on both sides, pooling + head) against the CPU oracle's bytes, at the reference's 512 px
block shapes and at small / ragged shapes (partial last tiles, tiles that straddle images, spans
that do not start on a tile). The store is [ceil(N HW / 128)][Gt][128][32]: 128 consecutive pixels
per tile, all Gt groups of a tile contiguous; bytes outside the groups a kernel writes must stay
untouched."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from rsna_knee_efficiency_b200 import densenet, ops
from tests.helpers import dev, from_tile_major, pixels_to_planes, plan_tables, rand_store, tile_major

pytestmark = pytest.mark.gpu

SENTINEL = 0x5A


def _store(rows: int, Gt: int) -> torch.Tensor:
    return torch.full((-(-rows // 128) * Gt * 4096,), SENTINEL, dtype=torch.int8, device="cuda")


def _untouched(t: np.ndarray, rows: int, keep) -> None:
    """Every byte of groups outside `keep`, and of rows past the last pixel, still holds the sentinel."""
    flat = t.transpose(0, 2, 1, 3).reshape(-1, t.shape[1], 32)
    other = [g for g in range(t.shape[1]) if g not in set(keep)]
    if other:
        assert (flat[:rows, other] == SENTINEL).all()
    assert (flat[rows:] == SENTINEL).all()


@pytest.mark.parametrize("bi,li,N,H,W", [(0, 0, 2, 128, 128), (1, 7, 2, 64, 64), (2, 20, 3, 32, 32),
                                         (3, 31, 2, 16, 16), (1, 2, 3, 5, 72), (1, 2, 2, 9, 9)])
def test_conv2_writes_its_group(bi, li, N, H, W):
    _, _, par = plan_tables(512)
    rng = np.random.default_rng(40 + bi + li + H)
    V = rng.integers(0, 80, size=(N, H, W, 128), dtype=np.int64).astype(np.uint8)
    rows, Gt, grp = N * H * W, 9, 5
    out = _store(rows, Gt)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.conv2(dev(pixels_to_planes(V.reshape(rows, 128))), dev(ops.prepare_conv2_weights(par[f"L{bi}_{li}_w2k"])),
              dev(par[f"L{bi}_{li}_c2u"]), out, N, H, W, err=err, tile_groups=Gt, group=grp)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    t = out.view(-1, Gt, 128, 32).cpu().numpy()
    want = orc.conv2(V, par[f"L{bi}_{li}_w2k"], par[f"L{bi}_{li}_c2u"], orc.KERNEL).reshape(rows, 32)
    np.testing.assert_array_equal(from_tile_major(t, rows, [grp]), want)
    _untouched(t, rows, [grp])


@pytest.mark.parametrize("bi,N,H,W", [(0, 2, 128, 128), (1, 2, 64, 64), (2, 2, 32, 32), (0, 3, 6, 10),
                                      (2, 2, 4, 4), (1, 1, 2, 2), (2, 5, 8, 6)])
@pytest.mark.parametrize("f16", [True, False])
def test_transition_reads_and_writes_tile_major(bi, N, H, W, f16):
    _, plan, par = plan_tables(512)
    b = plan.blocks[bi]
    c0, ctot = b.c0, b.c_tot
    cout = ctot // 2
    X = rand_store(np.random.default_rng(60 + bi + N + H + W), (N, H * W, ctot), "relu")
    Gt_in, Gt_out = ctot // 32 + 2, cout // 32 + 3          # wider stores than the groups in use
    rows_out = N * (H // 2) * (W // 2)
    out = _store(rows_out, Gt_out)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    tab = par[f"T{bi}_abh"] if f16 else par[f"T{bi}_ab"]
    ops.trans(dev(tile_major(X, Gt_in)), None, dev(ops.prepare_trans_weights(par[f"T{bi}_w"])), dev(tab),
              dev(par[f"T{bi}_gd"]), out, c0 // 32, ctot // 32, N, H, W, f16, err=err,
              tile_groups=Gt_in, out_tile_groups=Gt_out)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    t = out.view(-1, Gt_out, 128, 32).cpu().numpy()
    want = orc.trans(X.reshape(N, H, W, ctot), par[f"T{bi}_w"], ab=None if f16 else tab,
                     abh=tab if f16 else None, gd=par[f"T{bi}_gd"], mode=orc.KERNEL).reshape(rows_out, cout)
    np.testing.assert_array_equal(from_tile_major(t, rows_out, range(cout // 32)), want)
    _untouched(t, rows_out, range(cout // 32))


@pytest.mark.parametrize("img,N,flip", [(512, 3, [1, 0, 1]), (64, 2, None), (96, 3, [0, 1, 1])])
def test_stem_writes_groups_0_and_1(img, N, flip):
    from rsna_knee_efficiency_b200 import synth
    _, _, par = plan_tables(512)
    x = synth.triplets(synth.volume(8, H=img, W=img))[:N]
    PH = img // 4
    rows, Gt = N * PH * PH, 8
    out = _store(rows, Gt)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    src = np.zeros((N, 4), np.int32)
    src[:, :3] = np.arange(3 * N).reshape(N, 3)
    ops.stem(dev(x.reshape(3 * N, img, img)), dev(ops.prepare_stem_weights(par["S_w8"])), dev(par["S_kc"]), out,
             N, img, img, src=dev(src), flags=None if flip is None else dev(np.asarray(flip, np.int32)), err=err,
             tile_groups=Gt)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    t = out.view(-1, Gt, 128, 32).cpu().numpy()
    want = orc.stem(x, par["S_w8f"], par["S_kc"], flip=flip, mode=orc.KERNEL).reshape(rows, 64)
    np.testing.assert_array_equal(from_tile_major(t, rows, [0, 1]), want)
    _untouched(t, rows, [0, 1])


@pytest.mark.parametrize("N,HW", [(3, 256), (2, 4), (5, 16), (3, 100)])
def test_head_reads_tile_major(N, HW):
    _, plan, par = plan_tables(512)
    b = plan.blocks[3]
    X = rand_store(np.random.default_rng(N * HW), (N, HW, b.c_tot), "uniform")
    head = densenet.random_head(5)
    hw = head.fc.weight.detach().numpy().astype(np.float32)
    hb = head.fc.bias.detach().numpy().astype(np.float32)
    feat = torch.zeros((N, b.c_tot), dtype=torch.float32, device="cuda")
    logits = torch.zeros((N, 4), dtype=torch.float32, device="cuda")
    views = torch.zeros((1, 4), dtype=torch.float32, device="cuda")
    tickets = torch.zeros(1, dtype=torch.int32, device="cuda")
    G = b.c_tot // 32
    ops.head(dev(tile_major(X, G + 1)), None, dev(par["F_ab"]), b.c0 // 32, G, N, HW, feat=feat, hw=dev(hw),
             hb=dev(hb), logits=logits, view_logits=views, tickets=tickets, per_view=N, tile_groups=G + 1)
    torch.cuda.synchronize()
    want_f = orc.final(X, par["F_ab"], orc.KERNEL)
    np.testing.assert_array_equal(feat.cpu().numpy(), want_f)
    want_l = orc.head(want_f, hw, hb)
    np.testing.assert_allclose(logits.cpu().numpy(), want_l, rtol=0, atol=1e-5)
    np.testing.assert_allclose(views.cpu().numpy()[0], want_l.mean(0), rtol=0, atol=1e-5)
