"""Parity against the reference's OWN CUDA kernels on the B200: `src/knee/dense8s_kernels.cu`
compiled here unmodified for sm_100 (`make -C oracle ref` -> oracle/_ref/, launched by
oracle/refcu.py with the reference's argument structs and launch geometry). Each of this
repository's kernels runs on the same inputs and must give the same bytes (conv1 u8 bottleneck,
conv2 int8 slot, transition int8 next-block input, stem int8 block input) and the same fp32
features (final_q) as the reference kernel it replaces. This pins the oracle's KERNEL mode to the
reference's compiled arithmetic as well (the same cases are compared with it).

Skipped when oracle/_ref/ was not built (the reference tree is needed to build it)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from oracle import refcu
from rsna_knee_efficiency_b200 import ops
from tests.helpers import dev, planes_to_pixels, pixels_to_planes, plan_tables, rand_store, split_store

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not refcu.available(), reason="oracle/_ref not built (make -C oracle ref)")]

PAD = 1 << 16          # slack after every buffer a reference kernel reads (its tail loads)


@pytest.fixture(scope="module")
def ref():
    return refcu.RefKernels(0)


def _buf(a: np.ndarray) -> torch.Tensor:
    """Device copy of `a` with PAD zero bytes after it (returned view: exactly `a`)."""
    flat = np.ascontiguousarray(a).reshape(-1).view(np.uint8)
    t = torch.zeros(flat.size + PAD, dtype=torch.uint8, device="cuda")
    t[:flat.size].copy_(torch.from_numpy(flat))
    return t[:flat.size].view(torch.from_numpy(np.ascontiguousarray(a).reshape(-1)[:1]).dtype)


def _out(nbytes: int, fill: int, dtype=torch.uint8) -> torch.Tensor:
    return torch.full((nbytes + PAD,), fill, dtype=torch.uint8, device="cuda")[:nbytes].view(dtype)


def _ref_in0(X: np.ndarray, c0: int) -> np.ndarray:
    """Channel-last store [N, HW, c] -> the reference's block input [N][G0][HW][32]."""
    N, HW, _ = X.shape
    return np.ascontiguousarray(X[..., :c0].reshape(N, HW, c0 // 32, 32).transpose(0, 2, 1, 3))


# (block, layer): the layers the reference's own checks use (pack_dense8s.py:863-864)
LAYERS = [(0, 0), (0, 5), (1, 7), (2, 20), (3, 31)]


@pytest.mark.parametrize("bi,li", LAYERS)
@pytest.mark.parametrize("kind", ["w64_pl", "u128"])
def test_conv1_vs_reference_kernel(ref, bi, li, kind):
    _, plan, par = plan_tables(512)
    b = plan.blocks[bi]
    N, HW, c0 = 2, b.h * b.w, b.c0
    cin = c0 + 32 * li
    rows = N * HW
    f16 = kind == "w64_pl"
    X = rand_store(np.random.default_rng(10 * bi + li), (N, HW, cin), "relu")
    tab = par[f"L{bi}_{li}_abh"] if f16 else par[f"L{bi}_{li}_ab"]
    _, seg = split_store(X, c0)
    segd = _buf(seg) if li > 0 else _buf(np.zeros(16, np.int8))
    # the reference kernel
    rout = _out(rows * 128, 0xA5)
    ref.conv1(_buf(_ref_in0(X, c0)), segd, _buf(par[f"L{bi}_{li}_w1"]), _buf(tab), _buf(par[f"L{bi}_{li}_gdu"]),
              rout, c0 // 32, cin // 32, N, HW, b.w, kind)
    # ours
    in0, _ = split_store(X, c0)
    out = _out(rows * 128, 0x5A)
    ops.conv1(dev(in0), segd, dev(ops.prepare_conv1_weights(par[f"L{bi}_{li}_w1"])), dev(tab),
              dev(par[f"L{bi}_{li}_gdu"]), out, c0 // 32, cin // 32, N, HW, f16)
    torch.cuda.synchronize()
    if f16:    # planar [4][rows][32]
        want = rout.view(4, rows, 32).permute(1, 0, 2).reshape(rows, 128).cpu().numpy()
    else:      # [rows][128]
        want = rout.view(rows, 128).cpu().numpy()
    got = planes_to_pixels(out, rows)
    np.testing.assert_array_equal(got, want)
    np.testing.assert_array_equal(orc.conv1(X.reshape(rows, cin), par[f"L{bi}_{li}_w1"],
                                            ab=None if f16 else tab, abh=tab if f16 else None,
                                            gd=par[f"L{bi}_{li}_gdu"], mode=orc.KERNEL), want)


@pytest.mark.parametrize("bi,li,kern", [(0, 0, "t8x32_pl"), (1, 7, "t16x16_pl"), (1, 3, "t8x32_pl"),
                                        (2, 20, "t16x16_pl"), (3, 31, "t16x16_pl")])
def test_conv2_vs_reference_kernel(ref, bi, li, kern):
    _, plan, par = plan_tables(512)
    b = plan.blocks[bi]
    N, H, W = 2, b.h, b.w
    rows = N * H * W
    rng = np.random.default_rng(70 + bi + li)
    V = rng.integers(0, 256, size=(rows, 128), dtype=np.int64).astype(np.uint8)
    V[rng.random(size=V.shape) < 0.4] = 0
    rout = _out(rows * 32, 0x11, torch.int8)
    ref.conv2(_buf(np.ascontiguousarray(V.reshape(rows, 4, 32).transpose(1, 0, 2))),
              _buf(par[f"L{bi}_{li}_w2k"]), _buf(par[f"L{bi}_{li}_c2u"]), rout, N, H, W, kern)
    out = _out(rows * 32, 0x22, torch.int8)
    ops.conv2(dev(pixels_to_planes(V)), dev(ops.prepare_conv2_weights(par[f"L{bi}_{li}_w2k"])),
              dev(par[f"L{bi}_{li}_c2u"]), out, N, H, W)
    torch.cuda.synchronize()
    want = rout.cpu().numpy()
    np.testing.assert_array_equal(out.cpu().numpy(), want)
    np.testing.assert_array_equal(
        orc.conv2(V.reshape(N, H, W, 128), par[f"L{bi}_{li}_w2k"], par[f"L{bi}_{li}_c2u"], orc.KERNEL).reshape(-1),
        want)


@pytest.mark.parametrize("bi", [0, 1, 2])
def test_transition_vs_reference_integer_kernel(ref, bi):
    """Our transition with the fp32 prologue against the reference's integer-form `trans_q128`."""
    _, plan, par = plan_tables(512)
    b = plan.blocks[bi]
    N, H, W, c0, ctot = 2, b.h, b.w, b.c0, b.c_tot
    cout = ctot // 2
    X = rand_store(np.random.default_rng(300 + bi), (N, H * W, ctot), "relu")
    in0, seg = split_store(X, c0)
    n_out = N * cout * (H // 2) * (W // 2)
    rout = _out(n_out, 0x33, torch.int8)
    ref.trans_q128(_buf(_ref_in0(X, c0)), _buf(seg), _buf(par[f"T{bi}_w"]), _buf(par[f"T{bi}_ab"]),
                   _buf(par[f"T{bi}_gd"]), rout, c0 // 32, ctot // 32, N, H, W)
    out = _out(n_out, 0x44, torch.int8)
    ops.trans(dev(in0), dev(seg), dev(ops.prepare_trans_weights(par[f"T{bi}_w"])), dev(par[f"T{bi}_ab"]),
              dev(par[f"T{bi}_gd"]), out, c0 // 32, ctot // 32, N, H, W, False)
    torch.cuda.synchronize()
    hw4 = (H // 2) * (W // 2)
    want = rout.view(N, cout // 32, hw4, 32).cpu().numpy()                 # [N][G0n][HW/4][32]
    got = out.view(cout // 32, N, hw4, 32).permute(1, 0, 2, 3).cpu().numpy()  # group-major -> [N][G][..]
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("bi", [0, 1, 2])
@pytest.mark.parametrize("kind", ["w0", "w1"])
def test_transition_vs_shipped_wide_kernels(ref, bi, kind):
    """The shipped 512-px packs select the wide transitions `trans_w0` / `trans_w1` (fp16 prologue,
    2x2 mean before the 1x1 conv on fp16 tensor cores with fp32 accumulation). This repository
    computes the exact integer form instead; on the same random store the two must meet the
    reference's own gate for a transition kernel against the exact formula (max diff <= 1,
    mismatch < 1e-3: kaggle/int8_pack/pack_dense8s.py:819-843, `unit_trans` :370-385)."""
    _, plan, par = plan_tables(512)
    b = plan.blocks[bi]
    N, H, W, c0, ctot = 2, b.h, b.w, b.c0, b.c_tot
    cout = ctot // 2
    if cout % {"w0": 128, "w1": 256}[kind]:
        pytest.skip(f"trans_{kind} needs c_out a multiple of {128 if kind == 'w0' else 256} (c_out {cout})")
    X = rand_store(np.random.default_rng(500 + bi), (N, H * W, ctot), "relu")
    in0, seg = split_store(X, c0)
    n_out = N * cout * (H // 2) * (W // 2)
    rout = _out(n_out, 0x33, torch.int8)
    ref.trans_w(kind, _buf(_ref_in0(X, c0)), _buf(seg), _buf(par[f"T{bi}_wh"]), _buf(par[f"T{bi}_abh"]),
                _buf(par[f"T{bi}_gdf"]), rout, c0 // 32, ctot // 32, N, H, W)
    out = _out(n_out, 0x44, torch.int8)
    ops.trans(dev(in0), dev(seg), dev(ops.prepare_trans_weights(par[f"T{bi}_w"])), dev(par[f"T{bi}_abh"]),
              dev(par[f"T{bi}_gd"]), out, c0 // 32, ctot // 32, N, H, W, True)
    torch.cuda.synchronize()
    hw4 = (H // 2) * (W // 2)
    want = rout.view(N, cout // 32, hw4, 32).cpu().numpy().astype(np.int32)
    got = out.view(cout // 32, N, hw4, 32).permute(1, 0, 2, 3).cpu().numpy().astype(np.int32)
    d = np.abs(got - want)
    print(f"transition {bi} vs trans_{kind}: max diff {int(d.max())}, mismatch {float((d > 0).mean()):.2e}")
    assert d.max() <= 1 and (d > 0).mean() < 1e-3


def test_stem_vs_reference_kernel(ref):
    """stem_i8 tiles 9 x 9 pooled pixels, so it runs at 288 px (72 = 8 x 9), the reference's
    training size; fp16 windows that are exact k/255 and some that are not."""
    _, _, par = plan_tables(512)
    from rsna_knee_efficiency_b200 import synth
    img, N = 288, 3
    t = synth.triplets(synth.volume(12, H=img, W=img))[[1, 9, 20]]
    x = (t.astype(np.float32) / 255.0).astype(np.float16)
    x[2] = np.random.default_rng(5).uniform(-0.05, 1.05, size=x[2].shape).astype(np.float16)
    PH = img // 4
    rout = _out(N * 2 * PH * PH * 32, 0x66, torch.int8)
    ref.stem_i8(_buf(x), _buf(par["S_w8"]), _buf(par["S_kc"]), rout, N, img, img)
    out = _out(N * 2 * PH * PH * 32, 0x77, torch.int8)
    ops.stem(dev(x), dev(ops.prepare_stem_weights(par["S_w8"])), dev(par["S_kc"]), out, N, img, img)
    torch.cuda.synchronize()
    want = rout.view(N, 2, PH * PH, 32).cpu().numpy()
    got = out.view(2, N, PH * PH, 32).permute(1, 0, 2, 3).cpu().numpy()
    np.testing.assert_array_equal(got, want)
    np.testing.assert_array_equal(
        orc.stem(x, par["S_w8f"], par["S_kc"], mode=orc.KERNEL),
        want.transpose(0, 2, 1, 3).reshape(N, PH, PH, 64))


@pytest.mark.parametrize("HW", [256, 16])
def test_final_vs_reference_kernel(ref, HW):
    _, plan, par = plan_tables(512)
    b = plan.blocks[3]
    N, c0, ctot = 3, b.c0, b.c_tot
    X = rand_store(np.random.default_rng(HW), (N, HW, ctot), "relu")
    in0, seg = split_store(X, c0)
    rf = torch.zeros((N, ctot), dtype=torch.float32, device="cuda")
    ref.final_q(_buf(_ref_in0(X, c0)), c0 // 32, _buf(seg), N, HW, _buf(par["F_ab"]), rf, ctot)
    feat = torch.zeros((N, ctot), dtype=torch.float32, device="cuda")
    ops.head(dev(in0), dev(seg), dev(par["F_ab"]), c0 // 32, ctot // 32, N, HW, feat=feat)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(feat.cpu().numpy(), rf.cpu().numpy())
