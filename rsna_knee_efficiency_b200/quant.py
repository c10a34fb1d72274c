"""Post-training INT8 quantisation of DenseNet169: calibration, plan and kernel tables.

This is the host half of the reference's `knee.dense8s` (`src/knee/dense8s.py:272-541`) and of the
helpers it takes from `knee.dense8` (`src/knee/dense8.py:176-189`). The tables must come out
bit-identical to the reference's (same float64 expression order, then one cast), because a pack
built by the reference has to load here and give the same integers; the function and field names
follow the reference so that pack-building scripts run unchanged.

Quantisation, per conv input:
  * block store: q = rint(x / sigma_c), sigma_c = amax_c / 127 (per channel, int8);
  * conv1 / transition input: u8 = relu(bn(x)) / s, s = amax / 255 (per tensor);
  * conv2 input: u8 bottleneck, s2u = amax / 255;
  * weights: int8 per output channel, scale max|w| / 127.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

QU = 255                 # u8 inputs of the kernels
QS = 127                 # store / int8 range
GROUP = 32               # channels per store group (= growth rate)
GROWTH = 32
BOTTLENECK = 128


# --- helpers (reference `src/knee/dense8.py:176-189`) ---------------------------------------
def _affine(bn) -> tuple[np.ndarray, np.ndarray]:
    """BatchNorm (eval) as a per-channel affine y = s x + t, float64."""
    s = bn.weight.detach().double() / torch.sqrt(bn.running_var.detach().double() + bn.eps)
    t = bn.bias.detach().double() - bn.running_mean.detach().double() * s
    return s.numpy(), t.numpy()


def _wq(w: torch.Tensor) -> tuple[np.ndarray, np.ndarray]:
    """Symmetric int8 per output channel: scale = max|w| / 127 (float32 arithmetic), q = rint(w / scale)."""
    w = w.detach().float()
    scale = w.abs().flatten(1).amax(1).clamp_min(1e-12) / QS
    inv = (1.0 / scale).view(-1, *[1] * (w.dim() - 1))
    q = torch.round(w * inv).clamp(-128, 127)
    return q.to(torch.int8).numpy(), scale.numpy().astype(np.float32)


def _sig(v, floor: float = 1e-6) -> np.ndarray:
    return np.maximum(np.asarray(v, dtype=np.float64), floor) / QS


# --- calibration (reference `src/knee/dense8s.py:272-318`) ----------------------------------
class _TopK:
    """Running 99.99th-percentile estimate of |x| (exact over the union of the batches): keeps the
    k largest values seen, k = ceil((1 - q) * n_seen).
    """

    def __init__(self, q: float, per_channel: bool) -> None:
        self.q, self.per_channel = q, per_channel
        self.vals: torch.Tensor | None = None      # (C, k) or (k,)
        self.n = 0

    def add(self, y: torch.Tensor) -> None:
        a = y.detach().float().abs()
        if self.per_channel:
            a = a.transpose(0, 1).reshape(a.shape[1], -1)
            self.n += a.shape[1]
        else:
            a = a.reshape(-1)
            self.n += a.numel()
        k = max(1, int(np.ceil((1.0 - self.q) * self.n)))
        cat = a if self.vals is None else torch.cat([self.vals, a], -1)
        k = min(k, cat.shape[-1])
        self.vals = torch.topk(cat, k, dim=-1).values

    def value(self):
        v = self.vals[..., -1]
        return v.cpu().double().numpy().tolist() if self.per_channel else float(v)


@torch.no_grad()
def calibrate(encoder, batches, method: str = "max", pct: float = 99.99) -> dict:
    """Activation ranges of the fp32 `encoder` over `batches` (tensors (N, in, H, W) on its device).

    Keys as the reference's: `seg0.{b}` and `conv2.{b}.{l}` are per-channel |x| ranges of every
    store segment (block input, conv2 output), `in1.{b}.{l}`, `in2.{b}.{l}`, `tin.{b}` the
    per-tensor ranges of the conv inputs. `method="max"` is the reference's maximum;
    `method="pct"` the `pct`-th percentile of |x| over the union of all batches.
    """
    f = encoder.features
    use_max = method == "max"
    if not use_max and method != "pct":
        raise ValueError(f"calibrate: method {method!r}, expected 'max' or 'pct'")
    q = pct / 100.0
    chan: dict = {}
    tens: dict = {}
    hooks = []

    def chan_hook(key):
        def hook(_m, _i, y):
            if use_max:
                v = y.detach().float().abs().amax(dim=(0, 2, 3))
                chan[key] = v if key not in chan else torch.maximum(chan[key], v)
            else:
                chan.setdefault(key, _TopK(q, True)).add(y)
        return hook

    def in_hook(key):
        def hook(_m, inp):
            x = inp[0]
            if use_max:
                tens[key] = max(tens.get(key, 0.0), float(x.detach().float().abs().max()))
            else:
                tens.setdefault(key, _TopK(q, False)).add(x)
        return hook

    hooks.append(f.pool0.register_forward_hook(chan_hook("seg0.0")))
    b = 0
    while hasattr(f, f"denseblock{b + 1}"):
        for li, layer in enumerate(getattr(f, f"denseblock{b + 1}").values()):
            hooks.append(layer.conv2.register_forward_hook(chan_hook(f"conv2.{b}.{li}")))
            hooks.append(layer.conv1.register_forward_pre_hook(in_hook(f"in1.{b}.{li}")))
            hooks.append(layer.conv2.register_forward_pre_hook(in_hook(f"in2.{b}.{li}")))
        if hasattr(f, f"transition{b + 1}"):
            tr = getattr(f, f"transition{b + 1}")
            hooks.append(tr.conv.register_forward_pre_hook(in_hook(f"tin.{b}")))
            hooks.append(tr.pool.register_forward_hook(chan_hook(f"seg0.{b + 1}")))
        b += 1
    try:
        for x in batches:
            encoder(x)
    finally:
        for h in hooks:
            h.remove()
    if use_max:
        out: dict = {k: v.cpu().numpy().astype(np.float64).tolist() for k, v in chan.items()}
        out.update(tens)
    else:
        out = {k: v.value() for k, v in chan.items()}
        out.update({k: v.value() for k, v in tens.items()})
    return out


# --- plan (reference `src/knee/dense8s.py:322-433`) ------------------------------------------
@dataclass
class SLayer:
    c_in: int
    a1: np.ndarray              # norm1 affine [c_in], float64
    b1: np.ndarray
    s1: float                   # u8 scale of the conv1 input
    w1: np.ndarray              # int8 [128, c_in], sign of norm2 folded in
    w1s: np.ndarray             # [128] > 0: weight scale * |a2|
    bias1: np.ndarray           # [128] = shift of norm2
    s2: float                   # int8 scale of the conv2 input (s2u = s2 * 127 / 255)
    w2: np.ndarray              # int8 [32, 128, 3, 3]
    w2s: np.ndarray             # [32]
    sig: np.ndarray             # [32] store scale of the output


@dataclass
class SBlock:
    c0: int
    h: int
    w: int
    sig0: np.ndarray
    layers: list
    ta: np.ndarray | None = None
    tb: np.ndarray | None = None
    ts: float | None = None
    tw: np.ndarray | None = None
    tws: np.ndarray | None = None

    @property
    def c_tot(self) -> int:
        return self.c0 + GROWTH * len(self.layers)

    @property
    def sig_all(self) -> np.ndarray:
        return np.concatenate([self.sig0] + [L.sig for L in self.layers])


@dataclass
class SPlan:
    img: int
    in_ch: int
    w0: np.ndarray              # stem, norm0 folded, float32 [64, in_ch, 7, 7]
    b0: np.ndarray
    blocks: list = field(default_factory=list)
    a5: np.ndarray | None = None
    b5: np.ndarray | None = None

    @property
    def n_features(self) -> int:
        return self.blocks[-1].c_tot


def make_plan(encoder, cal: dict, img: int) -> SPlan:
    """Integer weights, scales and affines of `encoder` (eval, BatchNorms not folded) for the
    ranges `cal` from `calibrate`, at input side `img`.
    """
    f = encoder.features
    a0, b0 = _affine(f.norm0)
    w0 = f.conv0.weight.detach().double().numpy() * a0[:, None, None, None]
    plan = SPlan(img=img, in_ch=int(f.conv0.weight.shape[1]), w0=w0.astype(np.float32),
                 b0=b0.astype(np.float32))
    h = w = img // 4
    c = int(f.conv0.weight.shape[0])
    sig0 = _sig(cal["seg0.0"])
    k = 1
    while hasattr(f, f"denseblock{k}"):
        bi = k - 1
        layers = []
        for li, layer in enumerate(getattr(f, f"denseblock{k}").values()):
            if not hasattr(layer.norm2, "running_var"):
                raise ValueError(f"denseblock{k}.denselayer{li + 1}: norm2 already folded")
            a1, b1 = _affine(layer.norm1)
            a2, b2 = _affine(layer.norm2)
            q1, s1w = _wq(layer.conv1.weight)
            sign = np.where(a2 < 0, -1, 1).astype(np.int8)
            mag = np.abs(a2)
            dead = mag < 1e-30
            q1 = (q1 * sign[:, None, None, None]).astype(np.int8)
            q1[dead] = 0
            w1s = np.where(dead, s1w, s1w * mag)
            q2, s2w = _wq(layer.conv2.weight)
            layers.append(SLayer(
                c_in=c + GROWTH * li, a1=a1, b1=b1,
                s1=max(float(cal[f"in1.{bi}.{li}"]), 1e-12) / QU,
                w1=q1.reshape(BOTTLENECK, -1), w1s=w1s.astype(np.float64),
                bias1=b2.astype(np.float64),
                s2=max(float(cal[f"in2.{bi}.{li}"]), 1e-12) / QS, w2=q2,
                w2s=s2w.astype(np.float64), sig=_sig(cal[f"conv2.{bi}.{li}"])))
        blk = SBlock(c0=c, h=h, w=w, sig0=sig0, layers=layers)
        c = blk.c_tot
        if hasattr(f, f"transition{k}"):
            tr = getattr(f, f"transition{k}")
            blk.ta, blk.tb = _affine(tr.norm)
            tq, tsw = _wq(tr.conv.weight)
            blk.ts = max(float(cal[f"tin.{bi}"]), 1e-12) / QU
            blk.tw, blk.tws = tq.reshape(tq.shape[0], -1), tsw.astype(np.float64)
            sig0 = _sig(cal[f"seg0.{bi + 1}"])
            c //= 2
            h //= 2
            w //= 2
        plan.blocks.append(blk)
        k += 1
    plan.a5, plan.b5 = _affine(f.norm5)
    return plan


# --- kernel tables (reference `src/knee/dense8s.py:436-541`) --------------------------------
def _chunked(w: np.ndarray) -> np.ndarray:
    """[cout, cin] -> [cin // 32, cout, 32]."""
    cout, cin = w.shape
    return np.ascontiguousarray(w.reshape(cout, cin // GROUP, GROUP).transpose(1, 0, 2))


def _abh(ab: np.ndarray) -> np.ndarray:
    """Prologue table [c, 2] float32 -> [c // 2, 4] fp16 bits: (A_2p, A_2p+1, B_2p, B_2p+1)."""
    h = ab.astype(np.float16)
    return np.ascontiguousarray(np.stack([h[0::2, 0], h[1::2, 0], h[0::2, 1], h[1::2, 1]],
                                         1)).view(np.int16)


def _abh_ab(abh: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """(A, B) per channel as float64 from an `_abh` table."""
    h = np.ascontiguousarray(abh).view(np.float16).astype(np.float64)
    return h[:, :2].reshape(-1), h[:, 2:].reshape(-1)


def stem_weights16(w: np.ndarray) -> np.ndarray:
    """[64, 3, 7, 7] -> [64, 168] fp16, k = (ch * 7 + ky) * 8 + kx', kx' = kx + 1 (kx' = 0 zero)."""
    cout, cin, kh, kw = w.shape
    out = np.zeros((cout, cin, kh, kw + 1), np.float32)
    out[..., 1:] = w
    return np.ascontiguousarray(out.reshape(cout, -1).astype(np.float16))


def stem_weights8(w8: np.ndarray) -> np.ndarray:
    """int8 [64, 3, 7, 7] -> [64, 176]: k as in `stem_weights16`, 8 trailing zeros."""
    cout, cin, kh, kw = w8.shape
    out = np.zeros((cout, cin, kh, kw + 1), np.int8)
    out[..., 1:] = w8
    flat = out.reshape(cout, -1)
    pad = np.zeros((cout, 176 - flat.shape[1]), np.int8)
    return np.ascontiguousarray(np.concatenate([flat, pad], 1))


def kernel_params(plan: SPlan) -> dict:
    """The kernel tables, with the reference's names and formulas:
    `L{b}_{l}_ab/_abh` conv1 prologue, `_gd/_gdu` conv1 epilogue (int8 / u8 bottleneck), `_w1`
    [G, 128, 32], `_c2` / `_c2u` conv2 scale, `_w2k` [4, 9, 32, 32]; `T{b}_ab/_abh/_gd/_w/_wh/_gdf`
    transition; `F_ab` norm5 with sigma folded; stem `S_w0, S_b0, S_w16, S_bias, S_inv` (floating
    stems) and `S_w8, S_w8f, S_kc` (INT8 stem: q = rint(clamp(acc k + c, 0, 127))).
    """
    out: dict = {}
    for bi, blk in enumerate(plan.blocks):
        sig = blk.sig_all
        for li, L in enumerate(blk.layers):
            s = sig[:L.c_in]
            out[f"L{bi}_{li}_ab"] = np.stack([L.a1 * s / (QU * L.s1),
                                              L.b1 / (QU * L.s1)], 1).astype(np.float32)
            out[f"L{bi}_{li}_abh"] = _abh(out[f"L{bi}_{li}_ab"])
            out[f"L{bi}_{li}_gd"] = np.stack([L.w1s * L.s1 / (QS * L.s2),
                                              L.bias1 / (QS * L.s2)], 1).astype(np.float32)
            out[f"L{bi}_{li}_w1"] = _chunked(L.w1)
            out[f"L{bi}_{li}_c2"] = (L.w2s / L.sig).astype(np.float32)
            s2u = L.s2 * QS / QU
            out[f"L{bi}_{li}_gdu"] = np.stack([L.w1s * L.s1 / (QU * s2u),
                                               L.bias1 / (QU * s2u)], 1).astype(np.float32)
            w2 = L.w2.reshape(GROWTH, 4, GROUP, 9)                 # [o, c, i, tap]
            out[f"L{bi}_{li}_w2k"] = np.ascontiguousarray(w2.transpose(1, 3, 0, 2))
            out[f"L{bi}_{li}_c2u"] = (s2u * L.w2s / L.sig).astype(np.float32)
        if blk.ta is not None:
            nxt = plan.blocks[bi + 1].sig0
            out[f"T{bi}_ab"] = np.stack([blk.ta * sig / (QU * blk.ts),
                                         blk.tb / (QU * blk.ts)], 1).astype(np.float32)
            out[f"T{bi}_gd"] = np.stack([0.25 * blk.ts * blk.tws / nxt,
                                         np.zeros_like(nxt)], 1).astype(np.float32)
            out[f"T{bi}_w"] = _chunked(blk.tw)
            out[f"T{bi}_abh"] = _abh(out[f"T{bi}_ab"])
            out[f"T{bi}_wh"] = _chunked(blk.tw).astype(np.float16)
            out[f"T{bi}_gdf"] = np.stack([blk.ts * blk.tws / nxt, np.zeros_like(nxt)],
                                         1).astype(np.float32)
    last = plan.blocks[-1]
    out["F_ab"] = np.stack([plan.a5 * last.sig_all, plan.b5], 1).astype(np.float32)
    s0 = plan.blocks[0].sig0
    out["S_w0"] = (plan.w0.astype(np.float64) / s0[:, None, None, None]).astype(np.float32)
    out["S_b0"] = (plan.b0.astype(np.float64) / s0).astype(np.float32)
    out["S_w16"] = stem_weights16(plan.w0)
    out["S_bias"] = plan.b0.astype(np.float32)
    out["S_inv"] = (1.0 / s0).astype(np.float32)
    w0 = plan.w0.astype(np.float64)
    sw = np.maximum(np.abs(w0).reshape(w0.shape[0], -1).max(1), 1e-12) / QS
    w8 = np.clip(np.rint(w0 / sw[:, None, None, None]), -QS, QS)
    out["S_w8"] = stem_weights8(w8)
    out["S_w8f"] = w8.astype(np.float32)
    out["S_kc"] = np.concatenate([sw / (QU * s0), plan.b0 / s0]).astype(np.float32)
    return out


def head_params(head) -> dict:
    """The linear head as pack tables: `H_w` [n_out, C] float32, `H_b` [n_out] float32."""
    return {"H_w": head.fc.weight.detach().float().numpy().copy(),
            "H_b": head.fc.bias.detach().float().numpy().copy()}
