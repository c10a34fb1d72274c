"""The study path on the GPU: two seeds, two windows per study, 24 slice triplets per window (with
and without flip TTA), study logits = mean over seeds of the slice-mean logits of the head -- checked
against the oracle's features of every image pushed through the fp64 head on the host, and the
sharded host loop (`run_shard`) against one call."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from rsna_knee_efficiency_b200 import densenet, infer, pack as packmod, quant, synth

pytestmark = pytest.mark.gpu

IMG, SLICES = 64, 26


def _packs(n):
    out = []
    for seed in (42, 43):
        torch.manual_seed(0)
        m = densenet.random_init(densenet.DenseNet169(), seed)
        cal = quant.calibrate(m, [torch.from_numpy(b) for b in synth.calibration_batches(2, 2, IMG, seed=1000 + seed)],
                              method="pct", pct=99.99)
        plan = quant.make_plan(m, cal, IMG)
        head = densenet.random_head(seed)
        out.append((packmod.make_pack(plan, n, head), plan, head))
    return out


@pytest.mark.parametrize("design,flip_tta", [("parx", False), ("parx", True), ("scale", False)])
def test_study_logits_match_oracle(design, flip_tta):
    """Seed k reads the windows `member_windows(design, 0, 2, 24, seed=k)` of both crop windows
    ("parx": alternate positions of every slot; "scale": all of slot k)."""
    studies = 2
    per_view = (SLICES - 2) * (2 if flip_tta else 1)
    packs = _packs(studies * per_view)
    runner = infer.StudyRunner([p for p, _, _ in packs], 0, studies, SLICES, flip_tta, design=design)
    vols = infer.make_volumes(studies, img=IMG, slices=SLICES, seed=77)
    got = runner.run(torch.from_numpy(vols).cuda()).cpu().numpy()
    for e in runner.encoders:
        e.check()
    planes = vols.reshape(-1, IMG, IMG)
    want = np.zeros((studies, 4))
    for k, (p, plan, head) in enumerate(packs):
        par = quant.kernel_params(plan)
        hw, hb = head.fc.weight.detach().double().numpy(), head.fc.bias.detach().double().numpy()
        src, flags, _ = infer.plane_table(design, k, studies, SLICES, 2, flip_tta)
        assert runner.per_view[k] == per_view
        for s in range(studies):
            rows = slice(s * per_view, (s + 1) * per_view)
            x = planes[src[rows, :3]]
            f = orc.forward(par, packmod.pack_meta(plan, len(x)), x, flip=flags[rows], mode=orc.KERNEL)
            np.testing.assert_array_equal(runner.encoders[k].out[rows].cpu().numpy(), f)
            want[s] += (f.astype(np.float64) @ hw.T + hb).mean(0) / len(packs)
    np.testing.assert_allclose(got, want, atol=1e-5)


def test_run_shard_matches_single_call():
    studies = 2
    packs = _packs(studies * (SLICES - 2))
    runner = infer.StudyRunner([p for p, _, _ in packs], 0, studies, SLICES)
    vols = infer.make_volumes(5, img=IMG, slices=SLICES, seed=91)
    host = torch.from_numpy(vols).pin_memory()
    all5 = infer.run_shard(runner, host)
    assert all5.shape == (5, 4)
    one = runner.run(torch.from_numpy(vols[:, 2:4]).cuda()).cpu()
    torch.testing.assert_close(all5[2:4], one, rtol=0, atol=0)
    second = infer.run_shard(runner, host, rank=1, world=2)          # studies 3, 4
    torch.testing.assert_close(second, all5[3:], rtol=0, atol=0)
