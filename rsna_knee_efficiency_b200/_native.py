"""ctypes binding of libdn8b200.so (include/dn8.h). No fallback: if the library or a GPU is missing,
every entry point raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libdn8b200.so")
IN_TREE = LIB_PATH
DN8_OK, DN8_EINVAL, DN8_ECUDA, DN8_EDEVICE = 0, 1, 2, 3
DN8_HEAD_SCRATCH_VIEWS = 4096
P, I32 = ctypes.c_void_p, ctypes.c_int32


class Conv1Args(ctypes.Structure):
    _fields_ = [("in0", P), ("seg", P), ("w", P), ("ab", P), ("gd", P), ("out", P), ("err", P),
                ("G0", I32), ("G", I32), ("N", I32), ("HW", I32), ("prologue_f16", I32), ("tile_groups", I32)]


class Conv2Args(ctypes.Structure):
    _fields_ = [("x", P), ("w", P), ("sc", P), ("out", P), ("err", P),
                ("N", I32), ("H", I32), ("W", I32), ("tile_groups", I32), ("group", I32)]


class TransArgs(ctypes.Structure):
    _fields_ = [("in0", P), ("seg", P), ("w", P), ("ab", P), ("gd", P), ("out", P), ("err", P),
                ("G0", I32), ("G", I32), ("N", I32), ("H", I32), ("W", I32), ("prologue_f16", I32),
                ("tile_groups", I32), ("out_tile_groups", I32)]


class StemArgs(ctypes.Structure):
    _fields_ = [("x", P), ("src", P), ("flags", P), ("w", P), ("kc", P), ("out", P), ("err", P),
                ("N", I32), ("H", I32), ("W", I32), ("x_u8", I32), ("n_alloc", I32), ("tile_groups", I32)]


class HeadArgs(ctypes.Structure):
    _fields_ = [("in0", P), ("seg", P), ("fab", P), ("feat", P), ("hw", P), ("hb", P),
                ("logits", P), ("view_logits", P), ("tickets", P),
                ("G0", I32), ("G", I32), ("N", I32), ("HW", I32), ("n_out", I32), ("per_view", I32),
                ("n_alloc", I32), ("tile_groups", I32)]


class ZoomArgs(ctypes.Structure):
    _fields_ = [("planes", P), ("src", P), ("flags", P), ("out", P), ("err", P),
                ("N", I32), ("H", I32), ("W", I32), ("scale", ctypes.c_double), ("tx", ctypes.c_double),
                ("ty", ctypes.c_double)]


class Table(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("data", P), ("nbytes", ctypes.c_int64)]


class PackDesc(ctypes.Structure):
    _fields_ = [("n", I32), ("img", I32), ("in_ch", I32), ("n_blocks", I32),
                ("c0", I32 * 4), ("h", I32 * 4), ("w", I32 * 4), ("L", I32 * 4), ("trans", I32 * 4),
                ("trans_f16", I32 * 4), ("c1_f16", P * 4), ("n_out", I32),
                ("tables", ctypes.POINTER(Table)), ("n_tables", I32)]


class Input(ctypes.Structure):
    _fields_ = [("x", P), ("src", P), ("flags", P), ("x_u8", I32)]


class LaunchInfo(ctypes.Structure):
    _fields_ = [("kind", I32), ("block", I32), ("layer", I32), ("ms", ctypes.c_float)]


KIND_NAMES = {0: "stem", 1: "conv1", 2: "conv2", 3: "trans", 4: "head"}
K_STEM, K_CONV1, K_CONV2, K_TRANS, K_HEAD = 0, 1, 2, 3, 4

EXPORTS = {
    "dn8_conv1": ([ctypes.POINTER(Conv1Args), P], ctypes.c_int),
    "dn8_conv2": ([ctypes.POINTER(Conv2Args), P], ctypes.c_int),
    "dn8_trans": ([ctypes.POINTER(TransArgs), P], ctypes.c_int),
    "dn8_stem": ([ctypes.POINTER(StemArgs), P], ctypes.c_int),
    "dn8_head": ([ctypes.POINTER(HeadArgs), P], ctypes.c_int),
    "dn8_head_noalloc": ([ctypes.POINTER(HeadArgs), P], ctypes.c_int),
    "dn8_zoom": ([ctypes.POINTER(ZoomArgs), P], ctypes.c_int),
    "dn8_prepare_stem_weights": ([P, P], ctypes.c_int),
    "dn8_prepare_conv1_weights": ([P, I32, P], ctypes.c_int),
    "dn8_prepare_trans_weights": ([P, I32, I32, P], ctypes.c_int),
    "dn8_prepare_conv2_weights": ([P, P], ctypes.c_int),
    "dn8_engine_create": ([ctypes.POINTER(PackDesc), ctypes.c_int, ctypes.POINTER(P)], ctypes.c_int),
    "dn8_engine_destroy": ([P], None),
    "dn8_engine_forward": ([P, ctypes.POINTER(Input), I32, P, P, P, I32, P], ctypes.c_int),
    "dn8_engine_check": ([P, P], ctypes.c_int),
    "dn8_engine_profile": ([P, ctypes.POINTER(Input), I32, P, ctypes.POINTER(LaunchInfo), I32,
                            ctypes.POINTER(I32), P], ctypes.c_int),
    "dn8_engine_store": ([P, I32, I32, P, P], ctypes.c_int),
    "dn8_engine_forward_to": ([P, ctypes.POINTER(Input), I32, I32, P], ctypes.c_int),
    "dn8_engine_launch": ([P, I32, I32, I32, P], ctypes.c_int),
    "dn8_engine_error": ([P], ctypes.c_char_p),
    "dn8_engine_device_bytes": ([P], ctypes.c_int64),
    "dn8_test_inject_wait_fault": ([I32, ctypes.c_int64], ctypes.c_int),
    "dn8_last_error": ([], ctypes.c_char_p),
    "dn8_device_sms": ([ctypes.c_int], ctypes.c_int),
}

_lib = None


def lib():
    """The loaded library (built in-tree by `build.py`); raises if it is missing."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with "
                               "`python -m rsna_knee_efficiency_b200.build` (no CPU fallback)")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (args, res) in EXPORTS.items():
            if LIB_PATH != IN_TREE and not hasattr(handle, name):
                continue                 # another build (bench.py --lib) may predate newer entry points
            fn = getattr(handle, name)
            fn.argtypes, fn.restype = args, res
        _lib = handle
    return _lib


class Dn8Error(RuntimeError):
    pass


def check(status: int, what: str, engine=None) -> None:
    if status == DN8_OK:
        return
    src = lib().dn8_engine_error(engine) if engine else lib().dn8_last_error()
    msg = src.decode(errors="replace")
    if status == DN8_EINVAL:
        raise ValueError(f"{what}: {msg}")
    raise Dn8Error(f"{what} (status {status}): {msg}")
