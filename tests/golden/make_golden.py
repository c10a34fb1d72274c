"""Generates the golden fixtures of tests/golden/ by running the REFERENCE's own code.

Run here (the reference is importable on CPU; it is not present on the GPU box, which only reads
the committed .npz files):

    PYTHONPATH=<reference>/src python tests/golden/make_golden.py [<reference>/src]

For each case it builds a DenseNet169 with this repository's seeded `random_init` (same state_dict
names as the reference's `knee.models.densenet.DenseNet169`, so the weights load into it
unchanged), then calls the reference's `dense8s.calibrate`, `make_plan`, `kernel_params` and
`emulate(quant=True, dtype=float64, conv2="ours", stem="i8", f16_layers=...)` with `trace`, and
stores:
  * `x`: the uint8 input [N, 3, img, img] (emulate gets x / 255 as float64);
  * `cal`: the calibration ranges (JSON);
  * `tab_<name>`: sha256 of every kernel table, so that this repository's `kernel_params` can be
    checked bit for bit without committing megabytes of weights;
  * `store_<b>`: the whole block store after block b, int8 [N, c_tot, h, w] (emulate's trace);
  * `feat`: the emulated features [N, 1664] float32.
The 512-px case (the north star's resolution: one whole view, the 24 triplets of a volume) keeps
only `storehash_<b>` (sha256 of each image's store bytes) and `xhash` instead of the stores and the
input (which the test regenerates from the seeded synthetic volume), so the fixture stays small.
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
REF = Path(sys.argv[1]) if len(sys.argv) > 1 else None
if REF is not None:
    sys.path.insert(0, str(REF))

from knee import dense8s                                     # noqa: E402  (the reference)
from knee.models.densenet import DenseNet169 as RefDenseNet  # noqa: E402

from rsna_knee_efficiency_b200 import densenet, synth        # noqa: E402

CASES = {
    # name: (img, images, model seed, volume seed, fp16 prologue everywhere, flip)
    "img64_f16": (64, 3, 42, 7, True, False),
    "img64_f32": (64, 2, 43, 8, False, False),
    "img64_flip": (64, 2, 42, 9, True, True),
    "img128_f16": (128, 2, 44, 10, True, False),
}
HASHED = {
    # name: (img, images, model seed, volume seed, fp16 prologue everywhere, flip)
    "img512_f16": (512, 24, 45, 11, True, False),     # one whole view: the 24 triplets of a volume
}


def input_images(img: int, n: int, vseed: int) -> np.ndarray:
    """The case's uint8 images [n, 3, img, img]: n slice triplets spread over a seeded volume."""
    t = synth.triplets(synth.volume(vseed, H=img, W=img))
    return np.ascontiguousarray(t[np.linspace(0, len(t) - 1, n).round().astype(int)])


def table_hash(a: np.ndarray) -> str:
    a = np.ascontiguousarray(a)
    h = hashlib.sha256(a.tobytes())
    h.update(str(a.dtype).encode() + str(a.shape).encode())
    return h.hexdigest()


@torch.no_grad()
def make(name: str, img: int, n: int, mseed: int, vseed: int, f16: bool, flip: bool, hashed: bool = False) -> None:
    mine = densenet.random_init(densenet.DenseNet169(), mseed)
    ref = RefDenseNet()
    ref.load_state_dict(mine.state_dict())
    ref.eval()
    cal_x = [torch.from_numpy(b) for b in synth.calibration_batches(2, 2, img, seed=500 + vseed)]
    cal = dense8s.calibrate(ref, cal_x)
    plan = dense8s.make_plan(ref, cal, img)
    par = dense8s.kernel_params(plan)
    x = input_images(img, n, vseed)
    xin = torch.from_numpy(x).double() / 255.0
    if flip:
        xin = torch.flip(xin, [-1])
    f16l = set()
    if f16:
        f16l = {(bi, li) for bi, b in enumerate(plan.blocks) for li in range(len(b.layers))}
        f16l |= {("t", bi) for bi, b in enumerate(plan.blocks) if b.ta is not None}
    trace: dict = {}
    feat = dense8s.emulate(plan, xin, quant=True, dtype=torch.float64, par=par, trace=trace,
                           conv2="ours", stem="i8", f16_layers=f16l)
    arrays = {"x": x, "cal": np.frombuffer(json.dumps(cal).encode(), np.uint8),
              "feat": feat.numpy().astype(np.float32),
              "meta": np.frombuffer(json.dumps({"img": img, "f16": f16, "flip": flip,
                                                "model_seed": mseed}).encode(), np.uint8)}
    for k, v in par.items():
        arrays[f"tab_{k}"] = np.frombuffer(table_hash(v).encode(), np.uint8)
    for bi, b in enumerate(plan.blocks):
        segs = [trace[(bi, j)] for j in range(len(b.layers) + 1)]
        store = np.ascontiguousarray(torch.cat(segs, 1).round().to(torch.int8).numpy())
        if hashed:                       # one hash per image, [N][64] sha256 hex digits
            arrays[f"storehash_{bi}"] = np.stack([np.frombuffer(table_hash(store[i]).encode(), np.uint8)
                                                  for i in range(n)])
        else:
            arrays[f"store_{bi}"] = store
    if hashed:
        arrays["xhash"] = np.frombuffer(table_hash(x).encode(), np.uint8)
        arrays["xspec"] = np.frombuffer(json.dumps({"n": n, "vseed": vseed}).encode(), np.uint8)
        del arrays["x"]
    np.savez_compressed(HERE / f"{name}.npz", **arrays)
    print(name, {k: v.shape for k, v in arrays.items() if k.startswith(("store", "feat", "x"))})


if __name__ == "__main__":
    torch.manual_seed(0)
    only = sys.argv[2:]                  # optional case names
    for name, args in CASES.items():
        if not only or name in only:
            make(name, *args)
    for name, args in HASHED.items():
        if not only or name in only:
            make(name, *args, hashed=True)
