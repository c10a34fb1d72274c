"""Loading of the golden fixtures (tests/golden/*.npz, made by tests/golden/make_golden.py from the
reference's own calibrate / make_plan / kernel_params / emulate)."""
from __future__ import annotations

import functools
import hashlib
import json
from pathlib import Path

import numpy as np

from rsna_knee_efficiency_b200 import densenet, quant

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = ["img64_f16", "img64_f32", "img64_flip", "img128_f16"]
HASHED_CASES = ["img512_f16"]          # stores kept as sha256 only; the input is regenerated


def table_hash(a: np.ndarray) -> str:
    a = np.ascontiguousarray(a)
    h = hashlib.sha256(a.tobytes())
    h.update(str(a.dtype).encode() + str(a.shape).encode())
    return h.hexdigest()


@functools.lru_cache(maxsize=8)
def golden_case(name: str):
    """(fixture arrays, meta, plan, tables) with the plan rebuilt by this repository's make_plan
    from the fixture's calibration and the seeded model."""
    z = dict(np.load(GOLDEN / f"{name}.npz"))
    meta = json.loads(bytes(z["meta"]).decode())
    cal = json.loads(bytes(z["cal"]).decode())
    model = densenet.random_init(densenet.DenseNet169(), meta["model_seed"])
    plan = quant.make_plan(model, cal, meta["img"])
    return z, meta, plan, quant.kernel_params(plan)


def golden_input(name: str) -> np.ndarray:
    """The case's uint8 input [N, 3, img, img]: stored, or (hashed cases) regenerated from the seeded
    synthetic volume exactly as tests/golden/make_golden.py drew it, and checked against its hash."""
    from rsna_knee_efficiency_b200 import synth
    z, meta, _, _ = golden_case(name)
    if "x" in z:
        return z["x"]
    spec = json.loads(bytes(z["xspec"]).decode())
    t = synth.triplets(synth.volume(spec["vseed"], H=meta["img"], W=meta["img"]))
    x = np.ascontiguousarray(t[np.linspace(0, len(t) - 1, spec["n"]).round().astype(int)])
    if table_hash(x) != bytes(z["xhash"]).decode():
        raise AssertionError(f"{name}: the regenerated input differs from the one the reference saw")
    return x


def oracle_meta(plan, f16: bool) -> dict:
    """Pack-like meta for oracle.forward: fp16 prologues everywhere (the shipped kernel choice) or
    fp32 ones."""
    return {"blocks": [{"c0": b.c0, "h": b.h, "w": b.w, "L": len(b.layers), "trans": b.ta is not None,
                        "bm": ["w64_pl" if f16 else "u128"] * len(b.layers),
                        "tbm": "w0" if f16 else "q128"} for b in plan.blocks]}
