"""The C-ABI boundary without a GPU: libdn8b200.so loads, exports exactly the functions that
include/dn8.h declares, the ctypes structures match the header's C layout (compiled here with gcc),
and the host-only weight preparation functions produce the shared-memory operand layouts they
document (restated in numpy), with EINVAL on bad arguments."""
from __future__ import annotations

import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from rsna_knee_efficiency_b200 import _native as nat

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "dn8.h"


def _declared() -> set[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return set(re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(dn8_\w+)\s*\(", text, flags=re.M))


def test_library_loads_and_exports_every_declared_function():
    declared = _declared()
    assert len(declared) >= 19
    assert declared == set(nat.EXPORTS), declared ^ set(nat.EXPORTS)
    lib = nat.lib()
    for name in declared:
        assert getattr(lib, name) is not None
    nm = shutil.which("nm")
    if nm:
        out = subprocess.run([nm, "-D", "--defined-only", str(nat.LIB_PATH)], capture_output=True, text=True).stdout
        exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln and ln.split()[-1].startswith("dn8_")}
        assert exported == declared, exported ^ declared


STRUCTS = {
    "dn8_conv1_args": nat.Conv1Args, "dn8_conv2_args": nat.Conv2Args, "dn8_trans_args": nat.TransArgs,
    "dn8_stem_args": nat.StemArgs, "dn8_head_args": nat.HeadArgs, "dn8_table": nat.Table,
    "dn8_pack_desc": nat.PackDesc, "dn8_input": nat.Input, "dn8_launch_info": nat.LaunchInfo,
}


def test_struct_layouts_match_header(tmp_path):
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "dn8.h"', "int main(void) {"]
    for cname, py in STRUCTS.items():
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for f, _ in py._fields_:
            lines.append(f'printf("{cname} {f} %zu\\n", offsetof({cname}, {f}));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run([gcc, "-I", str(HEADER.parent), str(src), "-o", str(exe)], check=True)
    got = {}
    for ln in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.splitlines():
        s, f, v = ln.split()
        got[(s, f)] = int(v)
    for cname, py in STRUCTS.items():
        assert got[(cname, "size")] == ctypes.sizeof(py), cname
        for f, _ in py._fields_:
            assert got[(cname, f)] == getattr(py, f).offset, (cname, f)


def _swz32(tile: np.ndarray) -> np.ndarray:
    """Rows of 32 bytes: the two 16-byte halves swap in rows r with (r >> 2) & 1 (32-byte swizzle
    of the tensor cores' shared-memory operand layout)."""
    rows = tile.shape[0]
    out = tile.reshape(rows, 2, 16).copy()
    sw = ((np.arange(rows) >> 2) & 1).astype(bool)
    out[sw] = out[sw][:, ::-1]
    return out.reshape(rows, 32)


def _call(fn, *arrays_and_ints):
    args = [a.ctypes.data if isinstance(a, np.ndarray) else a for a in arrays_and_ints]
    return fn(*args)


def test_prepare_conv1_weights():
    rng = np.random.default_rng(1)
    G = 5
    w1 = rng.integers(-127, 128, size=(G, 128, 32), dtype=np.int64).astype(np.int8)
    out = np.zeros(G * 4096, np.uint8)
    assert _call(nat.lib().dn8_prepare_conv1_weights, w1, G, out) == nat.DN8_OK
    want = np.concatenate([_swz32(w1[g]).view(np.uint8).reshape(-1) for g in range(G)])
    np.testing.assert_array_equal(out, want)
    assert nat.lib().dn8_prepare_conv1_weights(w1.ctypes.data, 0, out.ctypes.data) == nat.DN8_EINVAL
    assert b"bad arguments" in nat.lib().dn8_last_error()


@pytest.mark.parametrize("G,cout", [(8, 128), (12, 384), (40, 640), (16, 256)])
def test_prepare_trans_weights(G, cout):
    rng = np.random.default_rng(G)
    tw = rng.integers(-127, 128, size=(G, cout, 32), dtype=np.int64).astype(np.int8)
    out = np.zeros(G * cout * 32, np.uint8)
    assert _call(nat.lib().dn8_prepare_trans_weights, tw, G, cout, out) == nat.DN8_OK
    # chunks of 256 output channels, the last one 128 when c_out is an odd multiple of 128
    nc = 256 if cout >= 256 else 128
    parts = [_swz32(tw[g, c * nc:min(cout, (c + 1) * nc)]) for c in range(-(-cout // nc)) for g in range(G)]
    np.testing.assert_array_equal(out, np.concatenate(parts).view(np.uint8).reshape(-1))
    assert _call(nat.lib().dn8_prepare_trans_weights, tw, G, 96, out) == nat.DN8_EINVAL


def test_prepare_conv2_weights():
    rng = np.random.default_rng(2)
    w2k = rng.integers(-127, 128, size=(4, 9, 32, 32), dtype=np.int64).astype(np.int8)
    out = np.zeros(36864, np.uint8)
    assert _call(nat.lib().dn8_prepare_conv2_weights, w2k, out) == nat.DN8_OK
    # [dy][cblk][half][dx * 32 + o][16]
    want = w2k.reshape(4, 3, 3, 32, 2, 16).transpose(1, 0, 4, 2, 3, 5).reshape(-1).view(np.uint8)
    np.testing.assert_array_equal(out, want)


def test_prepare_stem_weights():
    rng = np.random.default_rng(3)
    w8 = rng.integers(-127, 128, size=(64, 176), dtype=np.int64).astype(np.int8)
    out = np.zeros(14336, np.uint8)
    assert _call(nat.lib().dn8_prepare_stem_weights, w8, out) == nat.DN8_OK
    # one K step per kernel row ky: [ch 0 kx' 0..7 | ch 1 | ch 2 | 8 zeros] of S_w8's (ch, ky) slots
    slots = w8[:, :168].reshape(64, 3, 7, 8)
    steps = np.zeros((7, 64, 32), np.int8)
    steps[:, :, :24] = slots.transpose(2, 0, 1, 3).reshape(7, 64, 24)
    want = np.concatenate([_swz32(steps[ky]) for ky in range(7)])
    np.testing.assert_array_equal(out, want.view(np.uint8).reshape(-1))


def test_kernel_entry_points_reject_bad_geometry_without_launching():
    """Argument validation runs before any CUDA call (so it is checked here, with no GPU)."""
    lib = nat.lib()
    a = nat.Conv2Args()
    a.N, a.H, a.W = 1, 8, 200                     # W > 128
    assert lib.dn8_conv2(ctypes.byref(a), None) == nat.DN8_EINVAL
    t = nat.TransArgs()
    t.G0, t.G, t.N, t.H, t.W = 2, 12, 1, 8, 8     # c_out 192: not a multiple of 128
    assert lib.dn8_trans(ctypes.byref(t), None) == nat.DN8_EINVAL
    s = nat.StemArgs()
    s.N, s.H, s.W = 1, 64, 1024                   # W > 512
    assert lib.dn8_stem(ctypes.byref(s), None) == nat.DN8_EINVAL
    assert lib.dn8_conv1(None, None) == nat.DN8_EINVAL
    assert lib.dn8_last_error()
    c = nat.Conv1Args()
    c.G0, c.G, c.N, c.HW = 2, 71, 1, 64           # 71 K groups: the weights fit no launch shape
    assert lib.dn8_conv1(ctypes.byref(c), None) == nat.DN8_EINVAL
    assert b"exceed" in lib.dn8_last_error()
    c.G, c.tile_groups = 8, 6                     # a tile-major store must hold all G groups
    assert lib.dn8_conv1(ctypes.byref(c), None) == nat.DN8_EINVAL


def test_head_scratch_constant_matches_header(tmp_path):
    """The Python binding's copy of DN8_HEAD_SCRATCH_VIEWS is the header's value."""
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    src = tmp_path / "views.c"
    src.write_text('#include <stdio.h>\n#include "dn8.h"\n'
                   'int main(void) { printf("%d\\n", DN8_HEAD_SCRATCH_VIEWS); return 0; }\n')
    exe = tmp_path / "views"
    subprocess.run([gcc, "-I", str(HEADER.parent), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    assert int(out) == nat.DN8_HEAD_SCRATCH_VIEWS


@pytest.mark.parametrize("entry", ["dn8_head", "dn8_head_noalloc"])
def test_head_rejects_view_logits_without_a_head(entry):
    """view_logits with no head weights would never be written: refused before any CUDA call."""
    lib = nat.lib()
    fake = 1 << 20                                            # 16-byte aligned, never used
    tickets = fake if entry == "dn8_head" else None
    a = nat.HeadArgs(fake, fake, fake, None, None, None, None, fake, tickets, 20, 52, 6, 256, 0, 3, 0)
    assert getattr(lib, entry)(ctypes.byref(a), None) == nat.DN8_EINVAL
    assert b"need the head" in lib.dn8_last_error()


def test_zoom_rejects_bad_arguments_without_launching():
    lib = nat.lib()
    fake = 1 << 20
    a = nat.ZoomArgs(fake, fake, None, fake, None, 2, 64, 72, 1.1, 0.0, 0.0)       # W % 16 != 0
    assert lib.dn8_zoom(ctypes.byref(a), None) == nat.DN8_EINVAL
    a.W, a.scale = 64, 0.2                                                          # scale < 0.25
    assert lib.dn8_zoom(ctypes.byref(a), None) == nat.DN8_EINVAL
    assert b"dn8_zoom" in lib.dn8_last_error()
