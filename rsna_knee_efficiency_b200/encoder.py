"""`Dense8SEncoder`: the drop-in for the reference's runner of the same name
(src/knee/dense8s.py:944-1651), over the native engine of libdn8b200.so.

Same constructor (pack dict as `load_pack` returns, GPU index, images per call, max_inflight),
same call contract: `enc(x)` with x (N, 3, img, img) fp16/float on cuda:dev returns a VIEW of the
encoder's own buffer `out[:N]` (N, n_features) float32, valid until the next call; the work runs
on a private stream that waits on the caller's stream, and the caller's stream waits on it before
returning. `capture(n)` records CUDA graphs, `graph_in_buf(n)` exposes the static input buffer the
reference's inference loop fills in place; the diagnostics `store(b, j)` (one store segment),
`trace(x)` (every block's store and the features), `profile` (device ms of every launch of a pass)
and `time_layers(reps)` (every conv1 / conv2 / transition timed alone) are the reference's. Errors:
a bad pack or geometry raises ValueError (as the reference), CUDA failures RuntimeError.

Beyond the reference: `encode_u8` feeds the uint8 volume planes straight into the stem (gather +
normalise + optional horizontal flip fused) and returns the head's logits and per-view means.
"""
from __future__ import annotations

import collections
import ctypes
import time

import numpy as np
import torch

from . import _native as nat
from .pack import C1_F16, KIND, PACK_FORMAT, TRANS_F16H


class Dense8SEncoder:
    def __init__(self, pack: dict, dev: int, n_total: int, max_inflight: int | None = None) -> None:
        meta = pack["meta"]
        if meta.get("kind") != KIND or meta.get("format") != PACK_FORMAT:
            raise ValueError(f"package {meta.get('kind')} format {meta.get('format')}, "
                             f"expected {KIND} {PACK_FORMAT}")
        if meta.get("conv2", "trt") != "ours":
            raise ValueError("package built for the TensorRT conv2 (no L*_gdu / L*_w2k tables): "
                             "rebuild it with conv2='ours'")
        t0 = time.perf_counter()
        self.meta, self.dev = meta, dev
        self.nb = int(meta["n"])
        self.n_out = -(-n_total // self.nb) * self.nb
        self.max_inflight = max_inflight
        self.inflight: collections.deque = collections.deque()
        self.graphs: dict = {}
        self.calls = {"graph": 0, "plain": 0}
        blocks = meta["blocks"]
        if len(blocks) > 4:
            raise ValueError(f"{len(blocks)} blocks: at most 4")
        par = pack["par"]
        self.n_head = int(meta.get("n_out", 0)) if "H_w" in par else 0
        self._keep = []                                  # host arrays referenced by the descriptor
        tabs = []
        for name, arr in par.items():
            a = np.ascontiguousarray(arr)
            self._keep.append(a)
            tabs.append(nat.Table(name.encode(), a.ctypes.data, a.nbytes))
        table_arr = (nat.Table * len(tabs))(*tabs)
        self._keep.append(table_arr)
        d = nat.PackDesc()
        d.n, d.img, d.in_ch, d.n_blocks = self.nb, int(meta["img"]), int(meta["in_ch"]), len(blocks)
        for b, blk in enumerate(blocks):
            d.c0[b], d.h[b], d.w[b], d.L[b] = blk["c0"], blk["h"], blk["w"], blk["L"]
            d.trans[b] = int(bool(blk["trans"]))
            d.trans_f16[b] = int(blk.get("tbm") in TRANS_F16H)
            f16 = np.array([str(k) in C1_F16 or bool(blk.get("fused")) for k in blk["bm"]], np.int8)
            self._keep.append(f16)
            d.c1_f16[b] = f16.ctypes.data
        d.n_out = self.n_head
        d.tables, d.n_tables = table_arr, len(tabs)
        handle = ctypes.c_void_p()
        nat.check(nat.lib().dn8_engine_create(ctypes.byref(d), dev, ctypes.byref(handle)),
                  "dn8_engine_create")
        self._h = handle
        self.n_features = int(meta["n_features"])
        self.in_shape = (self.nb, int(meta["in_ch"]), int(meta["img"]), int(meta["img"]))
        self.in_dtype = torch.float16
        with torch.cuda.device(dev):
            self.stream = torch.cuda.Stream(dev)
            self.out = torch.empty((self.n_out, self.n_features), dtype=torch.float32, device=f"cuda:{dev}")
            self._pad = None
        self.load_s = time.perf_counter() - t0
        self.device_mb = round(nat.lib().dn8_engine_device_bytes(self._h) / 2**20, 1)

    # -- lifetime --
    def close(self) -> None:
        if getattr(self, "_h", None):
            torch.cuda.synchronize(self.dev)
            self.graphs.clear()
            nat.lib().dn8_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- core --
    def _forward(self, inp: nat.Input, n: int, feat_ptr, logits_ptr=None, views_ptr=None, per_view=0):
        nat.check(nat.lib().dn8_engine_forward(self._h, ctypes.byref(inp), n, feat_ptr, logits_ptr,
                                               views_ptr, per_view, self.stream.cuda_stream),
                  "dn8_engine_forward", self._h)

    def _throttle(self) -> None:
        if self.max_inflight:
            while len(self.inflight) >= self.max_inflight:
                self.inflight.popleft().synchronize()

    def _mark(self) -> None:
        if self.max_inflight:
            ev = torch.cuda.Event(blocking=True)
            ev.record(self.stream)
            self.inflight.append(ev)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        n = x.shape[0]
        if x.dim() != 4 or tuple(x.shape[1:]) != self.in_shape[1:]:
            raise ValueError(f"input {tuple(x.shape)}, expected (N, {', '.join(map(str, self.in_shape[1:]))})")
        if n > self.out.shape[0]:
            raise ValueError(f"{n} images, the encoder was built for {self.out.shape[0]}")
        cur = torch.cuda.current_stream(self.dev)
        self.stream.wait_stream(cur)
        with torch.cuda.stream(self.stream):
            gs = self._graph_for(n)
            if gs is not None:
                graphs, buf = gs
                if x.data_ptr() != buf.data_ptr():
                    buf[:n].copy_(x)
                for g in graphs:
                    self._throttle()
                    g.replay()
                    self._mark()
                self.calls["graph"] += 1
            else:
                xh = x.to(self.in_dtype, memory_format=torch.contiguous_format)
                self._throttle()
                self._forward(nat.Input(xh.data_ptr(), None, None, 0), n, self.out.data_ptr())
                self._mark()
                self._last_input = xh                    # alive until the stream has consumed it
                self.calls["plain"] += 1
        cur.wait_stream(self.stream)
        return self.out[:n]

    def encode_u8(self, planes: torch.Tensor, src: torch.Tensor, flags: torch.Tensor | None = None,
                  logits: torch.Tensor | None = None, views: torch.Tensor | None = None,
                  per_view: int = 0) -> torch.Tensor:
        """Encode n = len(src) images gathered from uint8 planes [P, img, img] (src int32 [n, 4] =
        plane of each channel, flags int32 [n] bit 0 = horizontal flip). Fills `logits` [n, n_out]
        and `views` [n / per_view, n_out] when given. Returns out[:n] (features)."""
        cur = torch.cuda.current_stream(self.dev)
        self.stream.wait_stream(cur)
        out = self.enqueue_u8(planes, src, flags, logits, views, per_view)
        cur.wait_stream(self.stream)
        return out

    def enqueue_u8(self, planes: torch.Tensor, src: torch.Tensor, flags: torch.Tensor | None = None,
                   logits: torch.Tensor | None = None, views: torch.Tensor | None = None,
                   per_view: int = 0) -> torch.Tensor:
        """`encode_u8` without the stream hand-offs: the pass is enqueued on the encoder's own
        stream (`self.stream`) only. The caller makes that stream wait for the inputs and waits on it
        before reading the outputs; this lets several encoders (the seeds of a study batch) run
        their passes concurrently."""
        n = src.shape[0]
        if planes.dtype != torch.uint8 or src.dtype != torch.int32:
            raise ValueError("encode_u8: uint8 planes and int32 plane table expected")
        with torch.cuda.stream(self.stream):
            inp = nat.Input(planes.data_ptr(), src.data_ptr(), None if flags is None else flags.data_ptr(), 1)
            self._forward(inp, n, self.out.data_ptr(), None if logits is None else logits.data_ptr(),
                          None if views is None else views.data_ptr(), per_view)
        return self.out[:n]

    def encode(self, x: torch.Tensor, logits: torch.Tensor | None = None, views: torch.Tensor | None = None,
               per_view: int = 0) -> torch.Tensor:
        """`encode_u8` for fp16 windows x (N, 3, img, img) on cuda:dev (e.g. the zoomed view of
        `ops.zoom`): features out[:N], and the head's logits / per-view means when given."""
        n = x.shape[0]
        if x.dtype != torch.float16 or tuple(x.shape[1:]) != self.in_shape[1:]:
            raise ValueError(f"encode: fp16 (N, {', '.join(map(str, self.in_shape[1:]))}) expected")
        x = x.contiguous()
        cur = torch.cuda.current_stream(self.dev)
        self.stream.wait_stream(cur)
        with torch.cuda.stream(self.stream):
            self._forward(nat.Input(x.data_ptr(), None, None, 0), n, self.out.data_ptr(),
                          None if logits is None else logits.data_ptr(),
                          None if views is None else views.data_ptr(), per_view)
            self._last_input = x
        cur.wait_stream(self.stream)
        return self.out[:n]

    def check(self) -> None:
        """Raises if a kernel gave up a bounded wait since the last check (synchronises)."""
        nat.check(nat.lib().dn8_engine_check(self._h, self.stream.cuda_stream), "dn8_engine_check", self._h)

    # -- graphs (the reference's `capture` / `graph_in_buf`, dense8s.py:1410-1444) --
    def capture(self, n: int) -> float:
        n = -(-n // self.nb) * self.nb
        if n > self.out.shape[0]:
            raise ValueError(f"graph for {n} images: the engine does {self.nb} per pass, "
                             f"the output holds {self.out.shape[0]}")
        t = time.perf_counter()
        with torch.cuda.device(self.dev):
            buf = torch.zeros((n, *self.in_shape[1:]), dtype=self.in_dtype, device=f"cuda:{self.dev}")
            with torch.cuda.stream(self.stream):
                self._forward(nat.Input(buf.data_ptr(), None, None, 0), self.nb, self.out.data_ptr())
            self.stream.synchronize()
            graphs = []
            for i in range(n // self.nb):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=self.stream, capture_error_mode="thread_local"):
                    chunk = buf[i * self.nb:(i + 1) * self.nb]
                    self._forward(nat.Input(chunk.data_ptr(), None, None, 0), self.nb,
                                  self.out[i * self.nb].data_ptr())
                graphs.append(g)
            self.stream.synchronize()
        self.graphs[n] = (graphs, buf)
        return time.perf_counter() - t

    def _graph_for(self, n: int):
        gs = self.graphs.get(n)
        if gs is None:
            k = -(-n // self.nb)
            for m, (g, buf) in sorted(self.graphs.items()):
                if m >= k * self.nb:
                    return g[:k], buf
        return gs

    def graph_in_buf(self, n: int) -> torch.Tensor | None:
        gs = self._graph_for(n)
        return None if gs is None else gs[1][:n]

    # -- diagnostics --
    def store(self, bi: int, j: int) -> torch.Tensor:
        """Store segment (bi, j) of the last pass as float (nb, c, h, w) of integers (j = 0 block input,
        j >= 1 output of layer j-1). Only the last two blocks survive a pass (alternating arenas)."""
        b = self.meta["blocks"][bi]
        hw = b["h"] * b["w"]
        g0 = b["c0"] // 32
        groups = g0 if j == 0 else 1
        buf = torch.empty(groups * self.nb * hw * 32, dtype=torch.int8, device=f"cuda:{self.dev}")
        nat.check(nat.lib().dn8_engine_store(self._h, bi, j, buf.data_ptr(), self.stream.cuda_stream),
                  "dn8_engine_store", self._h)
        self.stream.synchronize()
        t = buf.view(groups, self.nb, hw, 32).permute(1, 0, 3, 2).reshape(self.nb, groups * 32, b["h"], b["w"])
        return t.float()

    @torch.no_grad()
    def trace(self, x: torch.Tensor) -> tuple[dict, torch.Tensor]:
        """One pass over the first `nb` images of x (N, 3, img, img) with every block's store: returns
        ({(block, j): float (nb, c, h, w)}, features (nb, n_features)) like the reference's `trace`
        (src/knee/dense8s.py:1509-1546; j = 0 the block input, j >= 1 the output of layer j - 1). The
        blocks alternate between two arenas, so the stores are read after partial passes that stop
        after blocks 1, 3, ... (passes are deterministic) and the features from a full pass."""
        xh = x[:self.nb].to(self.in_dtype).contiguous()
        n = xh.shape[0]
        f = torch.zeros((self.nb, self.n_features), dtype=torch.float32, device=f"cuda:{self.dev}")
        inp = nat.Input(xh.data_ptr(), None, None, 0)
        blocks = self.meta["blocks"]
        out: dict = {}
        self.stream.wait_stream(torch.cuda.current_stream(self.dev))
        for last in range(len(blocks)):
            if last % 2 == 0 and last != len(blocks) - 1:
                continue
            nat.check(nat.lib().dn8_engine_forward_to(self._h, ctypes.byref(inp), n, last, self.stream.cuda_stream),
                      "dn8_engine_forward_to", self._h)
            for bi in (last - 1, last):                  # store() synchronises the encoder's stream
                if bi >= 0 and (bi, 0) not in out:
                    for j in range(blocks[bi]["L"] + 1):
                        out[(bi, j)] = self.store(bi, j)[:n]
        with torch.cuda.stream(self.stream):
            self._forward(inp, n, f.data_ptr())
        self.stream.synchronize()
        self.check()
        return out, f[:n]

    def _time(self, fn, reps: int = 20) -> float:
        """ms per call of `fn` (launches on the encoder's stream): a CUDA graph of `reps` calls,
        replayed once as warm-up and once under events (the reference's `_time`,
        src/knee/dense8s.py:1565-1581)."""
        with torch.cuda.device(self.dev), torch.cuda.stream(self.stream):
            fn()
            self.stream.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=self.stream, capture_error_mode="thread_local"):
                for _ in range(reps):
                    fn()
            g.replay()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(self.stream)
            g.replay()
            e1.record(self.stream)
            self.stream.synchronize()
        return e0.elapsed_time(e1) / reps

    def time_layers(self, reps: int = 20) -> dict:
        """ms of every conv1, conv2 and transition of a pass, each launched `reps` times back to back
        on the current store (the reference's `time_layers`, src/knee/dense8s.py:1583-1596): keys
        "c1 b{block}l{layer}", "c2 b{block}l{layer}", "t{block}"."""
        out: dict = {}
        lib = nat.lib()

        def launcher(kind, b, l):
            def fn():
                nat.check(lib.dn8_engine_launch(self._h, kind, b, l, self.stream.cuda_stream),
                          "dn8_engine_launch", self._h)
            return fn

        for bi, b in enumerate(self.meta["blocks"]):
            for li in range(b["L"]):
                out[f"c1 b{bi}l{li}"] = round(self._time(launcher(nat.K_CONV1, bi, li), reps), 4)
                out[f"c2 b{bi}l{li}"] = round(self._time(launcher(nat.K_CONV2, bi, li), reps), 4)
            if b["trans"]:
                out[f"t{bi}"] = round(self._time(launcher(nat.K_TRANS, bi, 0), reps), 4)
        self.check()
        return out

    def profile(self, x: torch.Tensor | None = None, planes=None, src=None, flags=None,
                reps: int = 3) -> list:
        """Device milliseconds of every launch of one pass (averaged over `reps` passes after a
        warm-up), from CUDA events between launches: [(kind, block, layer, ms)] (the reference's
        `profile`, dense8s.py:1548-1563)."""
        if x is not None:
            xh = x[:self.nb].to(self.in_dtype).contiguous()
            inp, n = nat.Input(xh.data_ptr(), None, None, 0), xh.shape[0]
        else:
            inp = nat.Input(planes.data_ptr(), src.data_ptr(), None if flags is None else flags.data_ptr(), 1)
            n = min(self.nb, src.shape[0])
        buf = (nat.LaunchInfo * 512)()
        cnt = nat.I32()
        acc = None
        for r in range(reps + 1):
            nat.check(nat.lib().dn8_engine_profile(self._h, ctypes.byref(inp), n, self.out.data_ptr(), buf,
                                                   512, ctypes.byref(cnt), self.stream.cuda_stream),
                      "dn8_engine_profile", self._h)
            if r == 0:
                continue
            row = [(nat.KIND_NAMES[buf[k].kind], buf[k].block, buf[k].layer, buf[k].ms) for k in range(cnt.value)]
            acc = row if acc is None else [(a[0], a[1], a[2], a[3] + b[3]) for a, b in zip(acc, row)]
        return [(k, b, l, ms / reps) for k, b, l, ms in acc]
