"""Generates tests/golden/ref_pack_64.npz: a pack written by the REFERENCE's own
`knee.dense8s.save_pack(..., conv2="ours", stem="i8")` (src/knee/dense8s.py:833-844), for a small
3-block DenseNet (6 / 4 / 1 dense layers, growth 32; the reference's `DenseNet(3, "avg", (6, 4, 1))`)
at 64 px with 2 images per pass, so the fixture stays under a megabyte.

Run here (the reference is importable on CPU; the GPU box only reads the committed file):

    PYTHONPATH=<reference>/src python tests/golden/make_ref_pack.py

Kernel choices: the conv1 of block 1 as "w64_pl" with the planar conv2 "t16x16_pl" and transition 1 as
"w0" (the shipped 512-px kinds: fp16 prologue tables `*_abh`), everything else the reference's
defaults (conv1 "64", conv2 "q3w4", transition "q128": fp32 prologue tables `*_ab`), so one pack
exercises both prologues.
"""
from __future__ import annotations

from pathlib import Path

import torch

from knee import dense8s                       # the reference
from knee.models.densenet import DenseNet      # the reference

HERE = Path(__file__).resolve().parent


def main() -> None:
    torch.manual_seed(2026)
    m = DenseNet(3, "avg", (6, 4, 1))
    with torch.no_grad():                      # non-trivial BatchNorm statistics
        for mod in m.modules():
            if isinstance(mod, torch.nn.BatchNorm2d):
                mod.running_mean.normal_(0, 0.1)
                mod.running_var.uniform_(0.5, 1.5)
                mod.weight.normal_(1, 0.1)
                mod.bias.normal_(0, 0.1)
    m.eval()
    g = torch.Generator().manual_seed(7)
    cal = dense8s.calibrate(m, [torch.rand(2, 3, 64, 64, generator=g) for _ in range(2)])
    plan = dense8s.make_plan(m, cal, 64)
    bm = {f"b0l{li}": "w64_pl" for li in range(6)}
    dense8s.save_pack(HERE / "ref_pack_64.npz", plan, 2, {}, conv2="ours", stem="i8", stem_int8=True,
                      bm=bm, tbm={"t0": "w0"}, c2cfg={16: [16, 16, "t16x16_pl"]})
    print((HERE / "ref_pack_64.npz").stat().st_size, "bytes")


if __name__ == "__main__":
    main()
