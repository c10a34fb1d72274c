"""TEST INFRASTRUCTURE ONLY -- the reference's own CUDA kernels on the GPU, as a checker.

`oracle/_ref/dense8s_kernels.cubin` is the reference's `src/knee/dense8s_kernels.cu` compiled here,
unmodified, by `make -C oracle ref` (nvcc -cubin -arch=sm_100 -std=c++14, the options of the
reference's NVRTC build, src/knee/cudart.py:223-253). This module loads it through the CUDA driver
API (into the current context, which torch owns) and launches single kernels with the reference's
argument structs and launch geometry (src/knee/dense8s.py:1205-1290, :1330-1385). Only tests/ (as
the byte checker) and bench.py's reference arm (`--impl reference --layers`, which times these
kernels beside the BASELINE config 1 shapes) use it; the product never does.

Layouts are the reference's: block input [N][G0][HW][32], layer segments [L][N][HW][32], planar u8
bottleneck [4][N*HW][32], stem output = block 1's input [N][2][HW][32].
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import torch

CUBIN = Path(__file__).resolve().parent / "_ref" / "dense8s_kernels.cubin"
_U64, _I = ctypes.c_uint64, ctypes.c_int


class KArg(ctypes.Structure):
    """`struct KArg` (src/knee/dense8s_kernels.cu:147-158), passed by value."""
    _fields_ = [("in0", _U64), ("seg", _U64), ("w", _U64), ("ab", _U64), ("gd", _U64), ("out", _U64),
                ("G0", _I), ("G", _I), ("N", _I), ("HW", _I), ("W", _I), ("rows", _I), ("cout", _I),
                ("G0n", _I)]


class C2Arg(ctypes.Structure):
    """`struct C2Arg` (src/knee/dense8s_kernels.cu:1936-1942), passed by value."""
    _fields_ = [("x", _U64), ("w", _U64), ("sc", _U64), ("out", _U64), ("N", _I), ("H", _I), ("W", _I),
                ("TH", _I), ("TW", _I), ("txn", _I)]


# shared-memory sizes of the launches (src/knee/dense8s.py:60-66, :127-132, :221-262)
def gemm_shared(bm: int, mode: int, groups: int) -> int:
    stage = (bm // 4 if mode == 1 else bm) * 144
    return max(2 * (bm * 32 + 128 * 32), stage) + groups * 32 * 8


def c2t_shared(th: int, tw: int) -> int:
    plane = -(-(th + 2) * (tw + 2) * 16 // 128) * 128 + 64
    return 36864 + 4 * plane + 128


def trans_w_shared(bm: int, bn: int, groups: int) -> int:
    """`trans_w_body<bm, bn>` (src/knee/dense8s.py:221-225)."""
    return max(2 * (bm + bn) * 64, bm * (bn + 16)) + groups * 16 * 8


STEM_I8_SMEM = -(-(64 * 176 + 512 + 5696 + 3 * 43 * 44) // 16) * 16 + 361 * 68
STEM_TP = 9


def available() -> bool:
    return CUBIN.exists()


class RefKernels:
    def __init__(self, dev: int = 0):
        torch.cuda.set_device(dev)
        torch.zeros(1, device=f"cuda:{dev}")               # the primary context is current
        self.cu = ctypes.CDLL("libcuda.so.1")
        self.cu.cuLaunchKernel.argtypes = [ctypes.c_void_p] + [ctypes.c_uint] * 7 + \
            [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        data = CUBIN.read_bytes()
        self._image = ctypes.create_string_buffer(data, len(data))
        self.mod = ctypes.c_void_p()
        self._ok(self.cu.cuModuleLoadData(ctypes.byref(self.mod), self._image), "cuModuleLoadData")
        self.sms = torch.cuda.get_device_properties(dev).multi_processor_count
        self._fn: dict = {}

    def _ok(self, rc: int, what: str) -> None:
        if rc != 0:
            raise RuntimeError(f"{what}: CUresult {rc}")

    def fn(self, name: str, smem: int):
        f = self._fn.get(name)
        if f is None:
            f = ctypes.c_void_p()
            self._ok(self.cu.cuModuleGetFunction(ctypes.byref(f), self.mod, name.encode()), name)
            self._fn[name] = f
        if smem > 48 * 1024:
            self._ok(self.cu.cuFuncSetAttribute(f, 8, ctypes.c_int(smem)), f"{name} max shared")
        return f

    def launch(self, name: str, grid, block, args: list, smem: int, stream=None) -> None:
        f = self.fn(name, smem)
        grid = tuple(grid) + (1,) * (3 - len(grid))
        block = tuple(block) + (1,) * (3 - len(block))
        holders = [a if isinstance(a, ctypes.Structure | ctypes._SimpleCData) else ctypes.c_uint64(a)
                   for a in args]
        params = (ctypes.c_void_p * len(holders))(*[ctypes.cast(ctypes.pointer(h), ctypes.c_void_p)
                                                    for h in holders])
        st = (stream or torch.cuda.current_stream()).cuda_stream
        self._ok(self.cu.cuLaunchKernel(f, *grid, *block, smem, ctypes.c_void_p(st), params, None), name)

    # -- the reference's launches ---------------------------------------------------------------
    def conv1(self, in0, seg, w1, ab, gd, out, G0, G, N, HW, W, kind="w64_pl"):
        """conv1 `kind`: "w64_pl" (fp16 prologue, planar out) or "u128" (fp32 prologue, NHWC128 out)."""
        rows = N * HW
        a = KArg(in0.data_ptr(), seg.data_ptr(), w1.data_ptr(), ab.data_ptr(), gd.data_ptr(), out.data_ptr(),
                 G0, G, N, HW, W, rows, 128, 0)
        if kind == "w64_pl":
            self.launch("conv1_w64_pl", (-(-rows // 256),), (256,), [a], gemm_shared(256, 2, G))
        elif kind == "u128":
            self.launch("conv1_u128", (-(-rows // 128),), (256,), [a], gemm_shared(128, 2, G))
        else:
            raise ValueError(kind)

    def conv2(self, x, w2k, sc, out, N, H, W, kern="t16x16_pl"):
        """`conv2_t16x16_pl` or `conv2_t8x32_pl` (the reference's kernels for the u8 bottleneck at
        512 px: t8x32 in block 1, t16x16 elsewhere, dense8s.py:1118-1124)."""
        th, tw = {"t16x16_pl": (16, 16), "t8x32_pl": (8, 32)}[kern]
        if H % th or W % tw:
            raise ValueError(f"conv2 {kern}: {H}x{W}")
        txn, tyn = W // tw, H // th
        a = C2Arg(x.data_ptr(), w2k.data_ptr(), sc.data_ptr(), out.data_ptr(), N, H, W, th, tw, txn)
        self.launch(f"conv2_{kern}", (min(self.sms, txn * tyn * N),), (256,), [a], c2t_shared(th, tw))
        return kern

    def trans_q128(self, in0, seg, tw, ab, gd, out, G0, G, N, H, W):
        hw, cout = H * W, G * 16
        rows = N * hw
        a = KArg(in0.data_ptr(), seg.data_ptr(), tw.data_ptr(), ab.data_ptr(), gd.data_ptr(), out.data_ptr(),
                 G0, G, N, hw, W, rows, cout, cout // 32)
        self.launch("trans_q128", (cout // 128, -(-rows // 128)), (256,), [a], gemm_shared(128, 1, G))

    def trans_w(self, kind, in0, seg, twh, abh, gdf, out, G0, G, N, H, W):
        """The shipped wide transitions `trans_w0` / `trans_w1` (fp16 prologue, 2x2 mean before the
        1x1 conv on fp16 tensor cores with fp32 accumulation; src/knee/dense8s_kernels.cu:3077-3268),
        launched as `_trans_item` does (src/knee/dense8s.py:1242-1272): tables T*_wh, T*_abh, T*_gdf;
        out = the next block's input in the reference layout [N][c_out/32][H*W/4][32]."""
        bm, bn = {"w0": (256, 128), "w1": (128, 256)}[kind]
        hw, cout = H * W, G * 16
        if cout % bn:
            raise ValueError(f"trans_{kind}: c_out {cout} not a multiple of {bn}")
        rows = N * hw
        a = KArg(in0.data_ptr(), seg.data_ptr(), twh.data_ptr(), abh.data_ptr(), gdf.data_ptr(), out.data_ptr(),
                 G0, G, N, hw, W, rows, cout, cout // 32)
        self.launch(f"trans_{kind}", (cout // bn, -(-(rows // 4) // bm)), (512,), [a], trans_w_shared(bm, bn, G))

    def stem_i8(self, x, w8, kc, out, N, H, W):
        if (H // 4) % STEM_TP or (W // 4) % STEM_TP or H != W:
            raise ValueError("stem_i8 tiles 9 x 9 pooled pixels: square images with H / 4 % 9 == 0")
        tiles = N * (H // 4 // STEM_TP) ** 2
        self.launch("stem_i8", (min(self.sms, tiles),), (256,),
                    [x.data_ptr(), w8.data_ptr(), kc.data_ptr(), out.data_ptr(), _I(N), _I(H), _I(W)],
                    STEM_I8_SMEM)

    def final_q(self, in0, G0, seg, N, HW, fab, out, ctot):
        self.launch("final_q", (N, ctot // 32), (128,),
                    [in0.data_ptr(), _I(G0), seg.data_ptr(), _I(N), _I(HW), fab.data_ptr(), out.data_ptr(),
                     _I(ctot)], 0)
