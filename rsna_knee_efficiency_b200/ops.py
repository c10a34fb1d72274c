"""Kernel-level operators on torch CUDA tensors (the reference's per-kernel launches, through the
C ABI of include/dn8.h). Layouts:
  store  in0 [N, G0, HW, 32] int8, seg [L, N, HW, 32] int8 (the reference's block store);
  bottleneck u8 as 8 planes of 16 channels [8, N*HW, 16];
  conv2 output: the store slot [N, HW, 32] int8.
"""
from __future__ import annotations

import torch

from . import _native as nat


def _ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def _stream(stream) -> int | None:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def conv1(in0: torch.Tensor, seg: torch.Tensor, w1: torch.Tensor, ab: torch.Tensor,
          gd: torch.Tensor, out: torch.Tensor, G0: int, G: int, N: int, HW: int,
          prologue_f16: bool, err: torch.Tensor | None = None, stream=None) -> None:
    a = nat.Conv1Args(_ptr(in0), _ptr(seg), _ptr(w1), _ptr(ab), _ptr(gd), _ptr(out), _ptr(err),
                      G0, G, N, HW, int(bool(prologue_f16)))
    nat.check(nat.lib().dn8_conv1(a, _stream(stream)), "dn8_conv1")


def conv2(x: torch.Tensor, w2k: torch.Tensor, sc: torch.Tensor, out: torch.Tensor, N: int, H: int,
          W: int, err: torch.Tensor | None = None, stream=None) -> None:
    a = nat.Conv2Args(_ptr(x), _ptr(w2k), _ptr(sc), _ptr(out), _ptr(err), N, H, W)
    nat.check(nat.lib().dn8_conv2(a, _stream(stream)), "dn8_conv2")
