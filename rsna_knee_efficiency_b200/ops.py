"""Kernel-level operators on torch CUDA tensors (the reference's per-kernel launches, through the
C ABI of include/dn8.h). Layouts:
  store  group-major in0 [G0, N, HW, 32] int8 and seg [L, N, HW, 32] int8, or (tile_groups = Gt > 0)
         the tile-major block store [ceil(N*HW/128), Gt, 128, 32] int8 holding every group;
  bottleneck u8 as 8 planes of 16 channels [8, N*HW, 16];
  conv2 output: the store slot [N, HW, 32] int8, or group `group` of a tile-major store.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _native as nat


def _ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def _stream(stream) -> int | None:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def conv1(in0: torch.Tensor, seg: torch.Tensor | None, w1: torch.Tensor, ab: torch.Tensor,
          gd: torch.Tensor, out: torch.Tensor, G0: int, G: int, N: int, HW: int,
          prologue_f16: bool, err: torch.Tensor | None = None, stream=None, tile_groups: int = 0) -> None:
    """tile_groups = 0: in0 / seg are group-major planes; > 0: in0 is a tile-major block store."""
    a = nat.Conv1Args(_ptr(in0), _ptr(seg), _ptr(w1), _ptr(ab), _ptr(gd), _ptr(out), _ptr(err),
                      G0, G, N, HW, int(bool(prologue_f16)), int(tile_groups))
    nat.check(nat.lib().dn8_conv1(a, _stream(stream)), "dn8_conv1")


def conv2(x: torch.Tensor, w2k: torch.Tensor, sc: torch.Tensor, out: torch.Tensor, N: int, H: int,
          W: int, err: torch.Tensor | None = None, stream=None, tile_groups: int = 0, group: int = 0) -> None:
    a = nat.Conv2Args(_ptr(x), _ptr(w2k), _ptr(sc), _ptr(out), _ptr(err), N, H, W, tile_groups, group)
    nat.check(nat.lib().dn8_conv2(a, _stream(stream)), "dn8_conv2")


def trans(in0: torch.Tensor, seg: torch.Tensor, tw: torch.Tensor, ab: torch.Tensor, gd: torch.Tensor,
          out: torch.Tensor, G0: int, G: int, N: int, H: int, W: int, prologue_f16: bool,
          err: torch.Tensor | None = None, stream=None, tile_groups: int = 0, out_tile_groups: int = 0) -> None:
    a = nat.TransArgs(_ptr(in0), _ptr(seg), _ptr(tw), _ptr(ab), _ptr(gd), _ptr(out), _ptr(err),
                      G0, G, N, H, W, int(bool(prologue_f16)), tile_groups, out_tile_groups)
    nat.check(nat.lib().dn8_trans(a, _stream(stream)), "dn8_trans")


def stem(x: torch.Tensor, w8u: torch.Tensor, kc: torch.Tensor, out: torch.Tensor, N: int, H: int,
         W: int, src: torch.Tensor | None = None, flags: torch.Tensor | None = None,
         err: torch.Tensor | None = None, stream=None, tile_groups: int = 0) -> None:
    """x: fp16 [N, 3, H, W] windows, or uint8 planes [P, H, W] with `src` int32 [N, 4]."""
    x_u8 = x.dtype == torch.uint8
    a = nat.StemArgs(_ptr(x), _ptr(src), _ptr(flags), _ptr(w8u), _ptr(kc), _ptr(out), _ptr(err),
                     N, H, W, int(x_u8), 0, tile_groups)
    nat.check(nat.lib().dn8_stem(a, _stream(stream)), "dn8_stem")


def head(in0: torch.Tensor, seg: torch.Tensor, fab: torch.Tensor, G0: int, G: int, N: int, HW: int,
         feat: torch.Tensor | None = None, hw: torch.Tensor | None = None, hb: torch.Tensor | None = None,
         logits: torch.Tensor | None = None, view_logits: torch.Tensor | None = None,
         tickets: torch.Tensor | None = None, per_view: int = 0, stream=None, tile_groups: int = 0) -> None:
    n_out = 0 if hw is None else hw.shape[0]
    a = nat.HeadArgs(_ptr(in0), _ptr(seg), _ptr(fab), _ptr(feat), _ptr(hw), _ptr(hb), _ptr(logits),
                     _ptr(view_logits), _ptr(tickets), G0, G, N, HW, n_out, per_view, 0, tile_groups)
    nat.check(nat.lib().dn8_head(a, _stream(stream)), "dn8_head")


def zoom(planes: torch.Tensor, src: torch.Tensor, out: torch.Tensor, N: int, H: int, W: int,
         scale: float, tx: float = 0.0, ty: float = 0.0, flags: torch.Tensor | None = None,
         err: torch.Tensor | None = None, stream=None) -> None:
    """Zoomed / shifted fp16 windows [N, 3, H, W] from uint8 planes [P, H, W] (src int32 [N, 4])."""
    a = nat.ZoomArgs(_ptr(planes), _ptr(src), _ptr(flags), _ptr(out), _ptr(err), N, H, W, scale, tx, ty)
    nat.check(nat.lib().dn8_zoom(a, _stream(stream)), "dn8_zoom")


def head_noalloc(in0: torch.Tensor, seg: torch.Tensor, fab: torch.Tensor, G0: int, G: int, N: int, HW: int,
                 feat: torch.Tensor | None = None, hw: torch.Tensor | None = None, hb: torch.Tensor | None = None,
                 logits: torch.Tensor | None = None, view_logits: torch.Tensor | None = None,
                 per_view: int = 0, stream=None) -> None:
    """`head` with the library's built-in per-view counters instead of a ticket array (no device
    allocation by the caller): at most DN8_HEAD_SCRATCH_VIEWS views per call, calls in order."""
    n_out = 0 if hw is None else hw.shape[0]
    a = nat.HeadArgs(_ptr(in0), _ptr(seg), _ptr(fab), _ptr(feat), _ptr(hw), _ptr(hb), _ptr(logits),
                     _ptr(view_logits), None, G0, G, N, HW, n_out, per_view, 0)
    nat.check(nat.lib().dn8_head_noalloc(a, _stream(stream)), "dn8_head_noalloc")


# --- weight preparation (numpy in, numpy out) ----------------------------------------------
def prepare_stem_weights(w8: np.ndarray) -> np.ndarray:
    """`S_w8` [64, 176] int8 -> the stem operand table (14336 bytes)."""
    w8 = np.ascontiguousarray(w8, dtype=np.int8)
    out = np.empty(14336, np.uint8)
    nat.check(nat.lib().dn8_prepare_stem_weights(w8.ctypes.data, out.ctypes.data),
              "dn8_prepare_stem_weights")
    return out


def prepare_conv1_weights(w1: np.ndarray) -> np.ndarray:
    """`L*_w1` [G, 128, 32] int8 -> the UMMA-ready table (G * 4096 bytes)."""
    w1 = np.ascontiguousarray(w1, dtype=np.int8)
    out = np.empty(w1.shape[0] * 4096, np.uint8)
    nat.check(nat.lib().dn8_prepare_conv1_weights(w1.ctypes.data, w1.shape[0], out.ctypes.data),
              "dn8_prepare_conv1_weights")
    return out


def prepare_trans_weights(tw: np.ndarray) -> np.ndarray:
    """`T*_w` [G, c_out, 32] int8 -> the UMMA-ready table (G * c_out * 32 bytes)."""
    tw = np.ascontiguousarray(tw, dtype=np.int8)
    out = np.empty(tw.size, np.uint8)
    nat.check(nat.lib().dn8_prepare_trans_weights(tw.ctypes.data, tw.shape[0], tw.shape[1],
                                                  out.ctypes.data), "dn8_prepare_trans_weights")
    return out


def prepare_conv2_weights(w2k: np.ndarray) -> np.ndarray:
    """`L*_w2k` [4, 9, 32, 32] int8 -> the conv2 operand table (36864 bytes)."""
    w2k = np.ascontiguousarray(w2k, dtype=np.int8)
    out = np.empty(36864, np.uint8)
    nat.check(nat.lib().dn8_prepare_conv2_weights(w2k.ctypes.data, out.ctypes.data),
              "dn8_prepare_conv2_weights")
    return out
