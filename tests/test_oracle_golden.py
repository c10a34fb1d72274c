"""The CPU oracle and the host-side tables, pinned against golden vectors produced by the
reference itself (tests/golden/make_golden.py ran the reference's calibrate, make_plan,
kernel_params and emulate)."""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from rsna_knee_efficiency_b200 import densenet, quant, synth
from tests.golden_util import CASES, HASHED_CASES, golden_case, golden_input, oracle_meta, table_hash

VSEED = {"img64_f16": 7, "img64_f32": 8, "img64_flip": 9, "img128_f16": 10, "img512_f16": 11}


@pytest.mark.parametrize("name", CASES + HASHED_CASES)
def test_tables_bit_identical_to_reference(name):
    z, meta, plan, par = golden_case(name)
    ref = {k[4:]: bytes(v).decode() for k, v in z.items() if k.startswith("tab_")}
    assert set(ref) == set(par)
    bad = [k for k in par if table_hash(par[k]) != ref[k]]
    assert bad == []


@pytest.mark.parametrize("name", CASES + HASHED_CASES)
def test_calibration_matches_reference(name):
    z, meta, _, _ = golden_case(name)
    cal_ref = json.loads(bytes(z["cal"]).decode())
    m = densenet.random_init(densenet.DenseNet169(), meta["model_seed"])
    batches = [torch.from_numpy(b) for b in synth.calibration_batches(2, 2, meta["img"], seed=500 + VSEED[name])]
    cal = quant.calibrate(m, batches)
    assert set(cal) == set(cal_ref)
    for k in cal_ref:
        np.testing.assert_array_equal(np.asarray(cal[k], np.float64), np.asarray(cal_ref[k], np.float64))


def _stores(trace, plan):
    return [np.concatenate([trace[(bi, j)] for j in range(len(b.layers) + 1)], 1)
            for bi, b in enumerate(plan.blocks)]


@pytest.mark.parametrize("name", CASES)
def test_oracle_emulate_mode_bit_exact(name):
    """EMULATE mode reproduces the reference's emulate(): every store byte and the features."""
    z, meta, plan, par = golden_case(name)
    tr = {}
    f = orc.forward(par, oracle_meta(plan, meta["f16"]), z["x"], flip=1 if meta["flip"] else None,
                    mode=orc.EMULATE, trace=tr)
    for bi, got in enumerate(_stores(tr, plan)):
        np.testing.assert_array_equal(got, z[f"store_{bi}"])
    np.testing.assert_allclose(f, z["feat"], rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("name", CASES)
def test_oracle_kernel_mode_per_layer_gate(name):
    """KERNEL mode (the reference CUDA kernels' fp32 arithmetic) against emulate, layer by layer on
    the reference's own stores: the reference's gate (pack_dense8s.py:835), max_diff <= 1 and a
    mismatch fraction < 1e-3 (< 4e-3 on the 2 x 2 maps of the 64 px cases)."""
    z, meta, plan, par = golden_case(name)
    limit = 4e-3 if meta["img"] == 64 else 1e-3
    for bi, b in enumerate(plan.blocks):
        X = z[f"store_{bi}"].transpose(0, 2, 3, 1).copy()
        for li in range(len(b.layers)):
            cin = b.c0 + 32 * li
            kw = {"abh": par[f"L{bi}_{li}_abh"]} if meta["f16"] else {"ab": par[f"L{bi}_{li}_ab"]}
            v = orc.conv1(X[..., :cin], par[f"L{bi}_{li}_w1"], gd=par[f"L{bi}_{li}_gdu"], mode=orc.KERNEL, **kw)
            s = orc.conv2(v, par[f"L{bi}_{li}_w2k"], par[f"L{bi}_{li}_c2u"], orc.KERNEL)
            d = np.abs(s.astype(int) - X[..., cin:cin + 32].astype(int))
            assert d.max() <= 1 and (d > 0).mean() < limit, (bi, li, d.max(), (d > 0).mean())
        if b.ta is not None:
            kw = {"abh": par[f"T{bi}_abh"]} if meta["f16"] else {"ab": par[f"T{bi}_ab"]}
            q = orc.trans(X, par[f"T{bi}_w"], gd=par[f"T{bi}_gd"], mode=orc.KERNEL, **kw)
            want = z[f"store_{bi + 1}"][:, :b.c_tot // 2].transpose(0, 2, 3, 1)
            d = np.abs(q.astype(int) - want.astype(int))
            assert d.max() <= 1 and (d > 0).mean() < limit


def test_oracle_stem_kernel_mode_matches_emulate_formula():
    """stem: the kernel's single fmaf rounding against emulate's float64-then-fp32 rounding, on the
    128 px fixture: the reference gate allows max_diff <= 2 for the stem (pack_dense8s.py:837)."""
    z, meta, plan, par = golden_case("img128_f16")
    q = orc.stem(z["x"], par["S_w8f"], par["S_kc"], mode=orc.KERNEL)
    want = z["store_0"][:, :64].transpose(0, 2, 3, 1)
    d = np.abs(q.astype(int) - want.astype(int))
    assert d.max() <= 2 and (d > 0).mean() < 1e-3


@pytest.mark.parametrize("name", HASHED_CASES)
def test_oracle_emulate_mode_bit_exact_512(name):
    """At 512 px (the north star's resolution) EMULATE mode reproduces the reference's emulate():
    the sha256 of every block store of each image (emulate's trace) and the features, on the first
    and the last image of the fixture's 24-triplet view."""
    z, meta, plan, par = golden_case(name)
    pick = [0, len(z["feat"]) - 1]
    tr = {}
    f = orc.forward(par, oracle_meta(plan, meta["f16"]), golden_input(name)[pick], flip=1 if meta["flip"] else None,
                    mode=orc.EMULATE, trace=tr)
    for bi, got in enumerate(_stores(tr, plan)):
        for k, i in enumerate(pick):
            want = bytes(z[f"storehash_{bi}"][i]).decode()
            assert table_hash(np.ascontiguousarray(got[k])) == want, f"block {bi} image {i}"
    np.testing.assert_allclose(f, z["feat"][pick], rtol=1e-6, atol=1e-7)
