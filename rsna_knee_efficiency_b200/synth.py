"""Seeded synthetic knee-MRI stand-ins (the competition DICOMs are not available).

A study volume is uint8 [S, H, W] (S = 26 slices of 512 x 512): a Rayleigh(sigma = 20) background
plus 6 Gaussian ellipsoid blobs (peak 80-220, in-plane radius 20-120 px, 2-8 slices deep), rounded
and clipped to 0-255. The encoder reads slice triplets (three adjacent slices, stride 1: 24 images
from 26 slices), the reference's `make_windows(vol, stride=1, depth=3)`
(src/knee/models/baseline.py:154-165).
"""
from __future__ import annotations

import numpy as np

N_SLICES = 26
DEPTH = 3


def volume(seed: int, S: int = N_SLICES, H: int = 512, W: int = 512) -> np.ndarray:
    rng = np.random.default_rng(seed)
    v = rng.rayleigh(20.0, size=(S, H, W))
    z, y, x = np.arange(S, dtype=np.float64), np.arange(H, dtype=np.float64), \
        np.arange(W, dtype=np.float64)
    for _ in range(6):
        cz, cy, cx = rng.uniform(0, S), rng.uniform(0, H), rng.uniform(0, W)
        rz = rng.uniform(2, 8)
        ry, rx = rng.uniform(20, 120) * H / 512, rng.uniform(20, 120) * W / 512
        peak = rng.uniform(80, 220)
        ez = np.exp(-0.5 * ((z - cz) / rz) ** 2)
        ey = np.exp(-0.5 * ((y - cy) / ry) ** 2)
        ex = np.exp(-0.5 * ((x - cx) / rx) ** 2)
        v += peak * ez[:, None, None] * ey[None, :, None] * ex[None, None, :]
    return np.clip(np.rint(v), 0, 255).astype(np.uint8)


def triplet_index(n_slices: int = N_SLICES, depth: int = DEPTH) -> np.ndarray:
    """[n_win, depth] slice indices of the stride-1 windows."""
    n_win = n_slices - depth + 1
    return np.arange(n_win)[:, None] + np.arange(depth)[None, :]


def triplets(vol: np.ndarray, depth: int = DEPTH) -> np.ndarray:
    """uint8 [S, H, W] -> uint8 [S - depth + 1, depth, H, W]."""
    return np.ascontiguousarray(vol[triplet_index(vol.shape[0], depth)])


def calibration_batches(n_batches: int = 8, per_batch: int = 4, img: int = 512, seed: int = 1000):
    """`n_batches` seeded float32 batches (per_batch, 3, img, img) in [0, 1], each from a fresh
    synthetic volume (triplets spread over the slices)."""
    out = []
    for b in range(n_batches):
        t = triplets(volume(seed + b, H=img, W=img))
        idx = np.linspace(0, len(t) - 1, per_batch).round().astype(int)
        out.append((t[idx].astype(np.float32) / 255.0))
    return out
