"""TEST INFRASTRUCTURE ONLY -- ctypes front-end of the CPU oracle (`oracle/dn8_oracle.c`).

Only tests/, `__graft_entry__.smoke()` and bench.py's CPU-baseline leg use this module, as the
checker; the product package never imports it. It chains the C operators into the reference's
whole-network INT8 pipeline (`dense8s.emulate`, `src/knee/dense8s.py:549-622`) using the pack
tables (`kernel_params` names), in one of two arithmetic modes:
  KERNEL  -- the reference CUDA kernels' fp32 arithmetic (bit-exact target of the GPU kernels);
  EMULATE -- the reference's float64 emulation (pinned against tests/golden/ fixtures made by the
             reference itself).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "libdn8oracle.so"
KERNEL, EMULATE = 0, 1

# conv1 / transition kernel kinds of the reference that use the fp16 prologue table (`*_abh`):
# `C1_F16` and `TRANS_F16H` (src/knee/dense8s.py:105-106, :798)
C1_F16 = {"h128h", "u128h", "u256h", "w4f", "u128hp", "u256hp", "u128hs", "u256hs", "u256hps",
          "p128", "u64hs", "u256hs_pl", "w64", "w64_pl"}
TRANS_F16H = {"hh", "f16h", "w0", "w1"}

_lib = None


def build() -> Path:
    """Compiles the oracle (make) if the library is missing or older than its source."""
    src = HERE / "dn8_oracle.c"
    if not LIB.exists() or LIB.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(str(LIB))
        P = ctypes.c_void_p
        I, L = ctypes.c_int, ctypes.c_long
        _lib.orc_conv1.argtypes = [P, L, I, P, P, P, P, I, P, P]
        _lib.orc_conv2.argtypes = [P, I, I, I, P, P, I, P, P]
        _lib.orc_trans.argtypes = [P, I, I, I, I, P, P, P, P, I, P]
        _lib.orc_final.argtypes = [P, I, I, I, P, I, P]
        _lib.orc_stem.argtypes = [P, I, P, I, I, I, P, P, I, P]
        _lib.orc_head.argtypes = [P, I, I, P, P, I, P]
        for f in ("orc_conv1", "orc_conv2", "orc_trans", "orc_final", "orc_stem", "orc_head"):
            getattr(_lib, f).restype = None
    return _lib


def _p(a):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def set_threads(n: int | None) -> None:
    if n:
        os.environ["OMP_NUM_THREADS"] = str(n)


# --- operators (channel-last arrays) --------------------------------------------------------
def conv1(X, w1c, ab=None, abh=None, gd=None, mode=KERNEL, want_acc=False):
    """X int8 [..., cin] -> u8 [..., 128] (and int32 accumulators)."""
    X = _c(X, np.int8)
    cin = X.shape[-1]
    P = X.size // cin
    out = np.empty(X.shape[:-1] + (128,), np.uint8)
    acc = np.empty(X.shape[:-1] + (128,), np.int32) if want_acc else None
    lib().orc_conv1(_p(X), P, cin, _p(_c(w1c, np.int8)),
                    _p(None if ab is None else _c(ab, np.float32)),
                    _p(None if abh is None else _c(abh, np.int16).view(np.uint16)),
                    _p(_c(gd, np.float32)), mode, _p(out), _p(acc))
    return (out, acc) if want_acc else out


def conv2(V, w2k, sc, mode=KERNEL, want_acc=False):
    """V u8 [N, H, W, 128] -> int8 [N, H, W, 32]."""
    V = _c(V, np.uint8)
    N, H, W, _ = V.shape
    out = np.empty((N, H, W, 32), np.int8)
    acc = np.empty((N, H, W, 32), np.int32) if want_acc else None
    lib().orc_conv2(_p(V), N, H, W, _p(_c(w2k, np.int8)), _p(_c(sc, np.float32)), mode,
                    _p(out), _p(acc))
    return (out, acc) if want_acc else out


def trans(X, wc, ab=None, abh=None, gd=None, mode=KERNEL):
    """X int8 [N, H, W, C] -> int8 [N, H/2, W/2, C/2]."""
    X = _c(X, np.int8)
    N, H, W, C = X.shape
    out = np.empty((N, H // 2, W // 2, C // 2), np.int8)
    lib().orc_trans(_p(X), N, H, W, C, _p(_c(wc, np.int8)),
                    _p(None if ab is None else _c(ab, np.float32)),
                    _p(None if abh is None else _c(abh, np.int16).view(np.uint16)),
                    _p(_c(gd, np.float32)), mode, _p(out))
    return out


def final(X, fab, mode=KERNEL):
    """X int8 [N, HW, C] -> float32 [N, C]."""
    X = _c(X, np.int8)
    N, HW, C = X.shape
    out = np.empty((N, C), np.float32)
    lib().orc_final(_p(X), N, HW, C, _p(_c(fab, np.float32)), mode, _p(out))
    return out


def stem(x, w8f, kc, flip=None, mode=KERNEL):
    """x [N, 3, H, W] uint8 (u = byte) or float16 (u = rint(255 sat(x))) -> int8 [N, H/4, W/4, 64]."""
    in_u8 = x.dtype == np.uint8
    x = _c(x, np.uint8 if in_u8 else np.float16)
    N, _, H, W = x.shape
    fl = None if flip is None else _c(np.broadcast_to(np.asarray(flip, np.int32), (N,)), np.int32)
    out = np.empty((N, H // 4, W // 4, 64), np.int8)
    lib().orc_stem(_p(x if in_u8 else x.view(np.uint16)), int(in_u8), _p(fl), N, H, W,
                   _p(_c(w8f, np.float32)), _p(_c(kc, np.float32)), mode, _p(out))
    return out


def head(f, hw, hb):
    f = _c(f, np.float32)
    N, C = f.shape
    n_out = hw.shape[0]
    out = np.empty((N, n_out), np.float32)
    lib().orc_head(_p(f), N, C, _p(_c(hw, np.float32)), _p(_c(hb, np.float32)), n_out, _p(out))
    return out


# --- whole network --------------------------------------------------------------------------
def f16_layers(meta: dict) -> set:
    """(b, l) and ("t", b) that use the fp16 prologue, from the pack's kernel choices
    (the reference's `f16_layers_meta`, src/knee/dense8s.py:1654-1659)."""
    out = {(bi, li) for bi, b in enumerate(meta["blocks"]) for li, k in enumerate(b["bm"])
           if str(k) in C1_F16 or b.get("fused")}
    return out | {("t", bi) for bi, b in enumerate(meta["blocks"]) if b.get("tbm") in TRANS_F16H}


def forward(par: dict, meta: dict, x, flip=None, mode=KERNEL, trace: dict | None = None,
            f16: set | None = None):
    """The INT8 encoder on the CPU: x [N, 3, img, img] (uint8 or float16) -> features [N, C]
    float32. `trace` receives {(block, j): int8 [N, c, H, W]} (j = 0 block input, j >= 1 output
    of layer j-1), like the reference's `Dense8SEncoder.trace`.
    """
    f16 = f16_layers(meta) if f16 is None else f16
    q = stem(x, par["S_w8f"], par["S_kc"], flip, mode)              # [N, h, w, 64]
    N = q.shape[0]
    for bi, b in enumerate(meta["blocks"]):
        H, W, c0, L = b["h"], b["w"], b["c0"], b["L"]
        ctot = c0 + 32 * L
        X = np.zeros((N, H, W, ctot), np.int8)
        X[..., :c0] = q
        if trace is not None:
            trace[(bi, 0)] = np.ascontiguousarray(q.transpose(0, 3, 1, 2))
        for li in range(L):
            cin = c0 + 32 * li
            fp16 = (bi, li) in f16
            v = conv1(X[..., :cin], par[f"L{bi}_{li}_w1"],
                      ab=None if fp16 else par[f"L{bi}_{li}_ab"],
                      abh=par[f"L{bi}_{li}_abh"] if fp16 else None,
                      gd=par[f"L{bi}_{li}_gdu"], mode=mode)
            seg = conv2(v, par[f"L{bi}_{li}_w2k"], par[f"L{bi}_{li}_c2u"], mode)
            X[..., cin:cin + 32] = seg
            if trace is not None:
                trace[(bi, li + 1)] = np.ascontiguousarray(seg.transpose(0, 3, 1, 2))
        if b["trans"]:
            fp16 = ("t", bi) in f16
            q = trans(X, par[f"T{bi}_w"], ab=None if fp16 else par[f"T{bi}_ab"],
                      abh=par[f"T{bi}_abh"] if fp16 else None, gd=par[f"T{bi}_gd"], mode=mode)
        else:
            return final(X.reshape(N, H * W, ctot), par["F_ab"], mode)
    raise RuntimeError("pack without a final block")
