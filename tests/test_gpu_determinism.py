"""Repeatability on the GPU: the same studies encoded in back-to-back calls (no host synchronisation
between them) give bit-identical features and study logits. A kernel that read accumulator
registers before its asynchronous TMEM load had landed, or a buffer before its producer had
finished, shows up here as calls that disagree."""
from __future__ import annotations

import torch
import pytest

from rsna_knee_efficiency_b200 import infer
from tests.test_gpu_study import SLICES, IMG, _packs

pytestmark = pytest.mark.gpu


def test_back_to_back_calls_are_bit_identical():
    studies = 8
    packs = _packs(studies * (SLICES - 2))
    runner = infer.StudyRunner([p for p, _, _ in packs], 0, studies, SLICES)
    vols = torch.from_numpy(infer.make_volumes(studies, img=IMG, slices=SLICES, seed=5)).cuda()
    logits, feats = [], []
    for _ in range(12):
        logits.append(runner.run(vols).clone())
        feats.append([e.out.clone() for e in runner.encoders])
    torch.cuda.synchronize()
    for k in range(1, len(logits)):
        for e in range(len(runner.encoders)):
            diff = (feats[k][e] != feats[0][e]).any(dim=1).nonzero().flatten().tolist()
            assert not diff, (f"call {k} seed {e}: features of images {diff[:16]} (of {len(diff)}) differ "
                              f"from call 0")
        assert torch.equal(logits[k], logits[0]), f"call {k} study logits differ from call 0"
