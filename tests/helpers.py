"""Shared helpers of the tests: seeded plans / tables, random stores in the reference's layouts."""
from __future__ import annotations

import functools

import numpy as np
import torch

from rsna_knee_efficiency_b200 import densenet, quant, synth


@functools.lru_cache(maxsize=4)
def plan_tables(img: int, seed: int = 42):
    """(model, plan, par) for a seeded random DenseNet169 calibrated on synthetic batches."""
    torch.manual_seed(0)
    m = densenet.random_init(densenet.DenseNet169(), seed)
    batches = [torch.from_numpy(b) for b in synth.calibration_batches(2, 2, img, seed=1000 + seed)]
    cal = quant.calibrate(m, batches)
    plan = quant.make_plan(m, cal, img)
    return m, plan, quant.kernel_params(plan)


def rand_store(rng: np.random.Generator, shape, kind: str = "uniform") -> np.ndarray:
    """int8 store bytes: 'uniform' = randint(-127, 128) (the reference's unit tests,
    kaggle/int8_pack/pack_dense8s.py:233-243); 'relu' = half zeros, the rest |N(0, 40)| clipped to
    127 (a requantised ReLU distribution)."""
    if kind == "uniform":
        return rng.integers(-127, 128, size=shape, dtype=np.int64).astype(np.int8)
    v = np.minimum(np.abs(rng.normal(0, 40, size=shape)), 127).round()
    v[rng.random(size=shape) < 0.5] = 0
    return v.astype(np.int8)


def split_store(X: np.ndarray, c0: int):
    """Channel-last store X [N, HW, c] -> (in0 [G0, N, HW, 32] group-major, seg [L, N, HW, 32])."""
    N, HW, c = X.shape
    in0 = X[..., :c0].reshape(N, HW, c0 // 32, 32).transpose(2, 0, 1, 3)
    L = (c - c0) // 32
    seg = X[..., c0:].reshape(N, HW, L, 32).transpose(2, 0, 1, 3)
    return np.ascontiguousarray(in0), np.ascontiguousarray(seg)


def planes_to_pixels(out: torch.Tensor, rows: int) -> np.ndarray:
    """Bottleneck planes [8, rows, 16] -> [rows, 128]."""
    return out.view(8, rows, 16).permute(1, 0, 2).reshape(rows, 128).cpu().numpy()


def pixels_to_planes(v: np.ndarray) -> np.ndarray:
    """[rows, 128] -> [8, rows, 16]."""
    rows = v.shape[0]
    return np.ascontiguousarray(v.reshape(rows, 8, 16).transpose(1, 0, 2))


def dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _flip(a: np.ndarray) -> np.ndarray:
    """int8 q <-> its offset-binary byte q + 128 (the same bit flip both ways)."""
    return (a.view(np.uint8) ^ np.uint8(0x80)).view(np.int8)


def tile_major(X: np.ndarray, Gt: int | None = None) -> np.ndarray:
    """Channel-last store X [N, HW, c] (c = 32 G) of signed q -> the tile-major block store
    [ceil(N HW / 128), Gt, 128, 32], whose bytes are q + 128 (offset binary; groups G .. Gt - 1 and
    the rows past the last pixel zero bytes)."""
    N, HW, c = X.shape
    G = c // 32
    Gt = G if Gt is None else Gt
    rows = N * HW
    nt = -(-rows // 128)
    t = np.zeros((nt * 128, Gt, 32), np.int8)
    t[:rows, :G] = _flip(np.ascontiguousarray(X.reshape(rows, G, 32)))
    return np.ascontiguousarray(t.reshape(nt, 128, Gt, 32).transpose(0, 2, 1, 3))


def from_tile_major(t: np.ndarray, rows: int, groups) -> np.ndarray:
    """Tile-major [T, Gt, 128, 32] (bytes q + 128) -> channel-last signed q [rows, 32 len(groups)] of
    the given groups."""
    flat = t.transpose(0, 2, 1, 3).reshape(-1, t.shape[1], 32)[:rows]
    return _flip(np.ascontiguousarray(flat[:, list(groups)].reshape(rows, -1)))
