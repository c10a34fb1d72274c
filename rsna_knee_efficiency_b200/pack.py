"""INT8 packs in the reference's `.npz` format (src/knee/dense8s.py:810-867, src/knee/dense8.py:597-604).

A pack holds `meta` (JSON as uint8 bytes), optional `cubin` / `eng_*` entries (never used here: no
NVRTC, no TensorRT) and the kernel tables as `par_<name>`. Packs written by the reference load here
and the other way round; this repository adds the optional head tables `par_H_w`, `par_H_b` and
`meta["n_out"]`.
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np

from . import quant

PACK_FORMAT = 1
KIND = "dense8s"
CSRC = Path(__file__).resolve().parent / "csrc"

# conv1 / transition kernel names of the reference whose prologue is the fp16 one (`C1_F16`,
# `TRANS_F16H`, src/knee/dense8s.py:105-106, :798): they select the `*_abh` tables.
C1_F16 = {"h128h", "u128h", "u256h", "w4f", "u128hp", "u256hp", "u128hs", "u256hs", "u256hps",
          "p128", "u64hs", "u256hs_pl", "w64", "w64_pl"}
TRANS_F16H = {"hh", "f16h", "w0", "w1"}


def kernels_sha() -> str:
    """Identity of this repository's kernel sources (the reference keys packs on its .cu's sha)."""
    h = hashlib.sha1()
    for p in sorted(CSRC.glob("*")):
        h.update(p.name.encode() + p.read_bytes())
    return h.hexdigest()[:12]


def pack_meta(plan: quant.SPlan, n: int, conv1: str = "w64_pl", trans: str = "w0",
              n_out: int = 0) -> dict:
    """The reference's meta layout (src/knee/dense8s.py:810-831) for our kernels: conv2 "ours"
    (u8 bottleneck), INT8 stem "i8". `conv1` / `trans` name the prologue the pack was built for:
    the reference's fp16 kinds ("w64_pl", "w0", ...) or fp32 ones ("u128", "q128")."""
    blocks = []
    for b in plan.blocks:
        blocks.append({"c0": b.c0, "h": b.h, "w": b.w, "L": len(b.layers), "trans": b.ta is not None,
                       "bm": [conv1] * len(b.layers), "c2": [16, 16, "t16x16_pl"],
                       "tbm": trans, "fused": None})
    return {"format": PACK_FORMAT, "kind": KIND, "n": int(n), "img": plan.img, "in_ch": plan.in_ch,
            "kernels_sha": kernels_sha(), "n_features": plan.n_features, "stem_c": int(plan.w0.shape[0]),
            "conv2_int8": True, "stem_int8": True, "conv2": "ours", "stem": "i8", "blocks": blocks,
            "engines": [], "n_out": int(n_out)}


def pack_params(plan: quant.SPlan, head=None) -> dict:
    """The tables a pack carries (the reference's `pack_params(conv2="ours")`, dense8s.py:847-859:
    the TensorRT conv2 tables are left out), plus the head when given."""
    par = quant.kernel_params(plan)
    par = {k: v for k, v in par.items() if not (k.startswith("L") and k.endswith(("_gd", "_c2")))}
    if head is not None:
        par.update(quant.head_params(head))
    return par


def save_pack(path, plan: quant.SPlan, n: int, head=None, extra: dict | None = None,
              conv1: str = "w64_pl", trans: str = "w0") -> None:
    n_out = 0 if head is None else int(head.fc.weight.shape[0])
    meta = pack_meta(plan, n, conv1, trans, n_out) | (extra or {})
    arrays = {"meta": np.frombuffer(json.dumps(meta).encode(), np.uint8)}
    arrays |= {f"par_{k}": v for k, v in pack_params(plan, head).items()}
    with open(path, "wb") as fh:
        np.savez(fh, **arrays)


def make_pack(plan: quant.SPlan, n: int, head=None, conv1: str = "w64_pl", trans: str = "w0") -> dict:
    """The in-memory pack (the dict `load_pack` returns) without a file round trip."""
    n_out = 0 if head is None else int(head.fc.weight.shape[0])
    return {"meta": pack_meta(plan, n, conv1, trans, n_out), "engines": {},
            "par": pack_params(plan, head), "cubin": None}


def load_pack(path) -> dict:
    with np.load(path) as z:
        meta = json.loads(bytes(z["meta"]).decode())
        engines = {k[4:]: z[k].tobytes() for k in z.files if k.startswith("eng_")}
        par = {k[4:]: np.array(z[k]) for k in z.files if k.startswith("par_")}
        cubin = z["cubin"].tobytes() if "cubin" in z.files else None
    return {"meta": meta, "engines": engines, "par": par, "cubin": cubin}


def is_pack(pack) -> bool:
    return isinstance(pack, dict) and pack.get("meta", {}).get("kind") == KIND


def f16_layers(meta: dict) -> set:
    """(b, l) and ("t", b) that use the fp16 prologue (the reference's `f16_layers_meta`)."""
    out = {(bi, li) for bi, b in enumerate(meta["blocks"]) for li, k in enumerate(b["bm"])
           if str(k) in C1_F16 or b.get("fused")}
    return out | {("t", bi) for bi, b in enumerate(meta["blocks"]) if b.get("tbm") in TRANS_F16H}
