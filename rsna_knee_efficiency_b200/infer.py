"""Study-level inference over the INT8 encoders: the part of the reference's inference loop
(src/knee/infer.py:974-1110, `_model_logits_budget_u8`, `_seed_logits_views_u8`, `_forward_split`)
that drives the encoder, restated for the benchmark's study workload.

A study has `n_windows` crop windows ("slots": uint8 volumes of S slices); each slot gives S - 2
slice triplets (stride 1, depth 3), so the study has n_windows x (S - 2) windows in slot-major order.
Which windows each seed's encoder reads is the reference's window budget
(src/knee/window_budget.py:57-123): the submission's design `parx` keeps, for seed f, the windows
at (position p + slot s + f) % 2 == 0, so two seeds cover every window exactly once and every seed
reads alternate positions of every slot. The stem gathers the triplets straight from the uint8
planes (the reference's `gather_u8_f16` fused into the stem), optionally adding the horizontally
flipped copy of every window (flip TTA). Per seed the head's logits are averaged over the seed's
images; the study logits are the mean over seeds. Studies are independent: ranks take contiguous
shards with no collective on the data path, and the host gathers the logits.
"""
from __future__ import annotations

import numpy as np
import torch

from .encoder import Dense8SEncoder

DEPTH = 3
DESIGNS = ("full", "par", "parx", "modQ[xR]", "qQfF", "scale")


def shard(n_items: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, end) share of rank `rank` (the reference splits studies per GPU the same
    way, infer.py:1065-1110)."""
    per = -(-n_items // world)
    start = min(n_items, rank * per)
    return start, min(n_items, start + per)


def seed_offsets(seed: int, n_slots: int, q: int) -> np.ndarray:
    """The per-slot grid offset o_f(s) of seed `seed` for step q (src/knee/window_budget.py:41-55):
    s % q for seed 0, a permutation of the same values (torch.randperm with a CPU generator seeded
    7919 * seed) for the others."""
    base = np.arange(n_slots) % q
    if seed == 0:
        return base
    g = torch.Generator().manual_seed(7919 * int(seed))
    return base[torch.randperm(n_slots, generator=g).numpy()]


def member_windows(design: str, member: int, n_slots: int, per: int, seed: int = 0) -> np.ndarray:
    """Sorted indices of the windows that member `member` (the TTA view) of seed `seed` reads, among
    the n_slots * per windows of a study in slot-major order: the reference's grid designs
    (`member_windows`, src/knee/window_budget.py:57-123) -- "full"; "parx" (p + s + seed + m) % 2 == 0;
    "par" and "modQ" / "modQxR" (p + o_f(s) + m) % Q < R; "qQfF" (p + s + F seed + m) % Q == 0;
    "scale" (s // (n_slots / 2) + m + seed) % 2 == 0."""
    s = np.repeat(np.arange(n_slots), per)
    p = np.tile(np.arange(per), n_slots)
    if design == "full":
        keep = np.ones(n_slots * per, bool)
    elif design == "parx":
        keep = (p + s + seed + member) % 2 == 0
    elif design == "par" or design.startswith("mod"):
        if design == "par":
            q, r = 2, 1
        else:
            q = int(design[3:].split("x")[0])
            r = int(design.split("x")[1]) if "x" in design else 1
        if not 0 < r <= q:
            raise ValueError(f"{design}: requires 0 < R <= Q")
        keep = (p + seed_offsets(seed, n_slots, q)[s] + member) % q < r
    elif design[:1] == "q" and "f" in design and design[1:].replace("f", "", 1).isdigit():
        q, f = (int(v) for v in design[1:].split("f"))
        if q < 1:
            raise ValueError(f"{design}: requires Q >= 1")
        keep = (p + s + f * seed + member) % q == 0
    elif design == "scale":
        if n_slots % 2:
            raise ValueError("scale: requires both crop scales (even number of slots)")
        keep = (s // (n_slots // 2) + member + seed) % 2 == 0
    else:
        raise ValueError(f"unknown design {design!r} (known: {DESIGNS})")
    return np.nonzero(keep)[0]


def plane_table(design: str, seed: int, studies: int, slices: int = 26, n_windows: int = 2,
                flip_tta: bool = False) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """(src int32 [n, 4], flags int32 [n], windows) of seed `seed`: image i of a call reads planes
    src[i, :3] of the call's volumes [n_windows, studies, slices, H, W] seen as planes (window s,
    study st, slice z -> plane (s * studies + st) * slices + z), flipped where flags[i] & 1. Images
    are study-major, then flip, then the seed's windows in slot-major order."""
    per = slices - DEPTH + 1
    idx = member_windows(design, 0, n_windows, per, seed=seed)
    if len(idx) == 0:
        raise ValueError(f"design {design!r}: seed {seed} reads no window")
    src, flags = [], []
    for st in range(studies):
        for f in ((0, 1) if flip_tta else (0,)):
            for w in idx:
                base = (int(w) // per * studies + st) * slices + int(w) % per
                src.append([base, base + 1, base + 2, 0])
                flags.append(f)
    return np.asarray(src, np.int32), np.asarray(flags, np.int32), idx


class StudyRunner:
    """Two (or more) seeds' encoders on one GPU, fed `studies` studies per call.

    `volumes` given to `run` is uint8 [n_windows, studies, S, H, W] on the device (window-major, so
    the planes of one window of all the call's studies are contiguous). Seed k (the k-th pack)
    reads the windows `member_windows(design, 0, n_windows, S - 2, seed=k)` of every study."""

    def __init__(self, packs: list[dict], dev: int, studies: int, slices: int = 26,
                 flip_tta: bool = False, zoom: tuple | None = None, design: str = "parx",
                 n_windows: int = 2) -> None:
        """`zoom` = (scale, tx, ty): the geometric view of the reference's TTA (`affine_windows`,
        src/knee/tta.py:131-149; the submission's view is (1.10, 0, 0)): the windows are zoomed on the
        device (`ops.zoom`) and encoded through the fp16 path instead of the stem's uint8 gather."""
        self.dev, self.studies, self.slices, self.flip_tta = dev, studies, slices, flip_tta
        self.design, self.n_windows = design, n_windows
        self.zoom = None if zoom is None or tuple(zoom) == (1.0, 0.0, 0.0) else tuple(float(z) for z in zoom)
        self.n_win = slices - DEPTH + 1
        d = self.device = f"cuda:{dev}"
        # per seed: the plane table (image -> planes of its three channels) and the flip flags
        self.windows, self.src, self.flags, self.per_view, self.n_img = [], [], [], [], []
        for k in range(len(packs)):
            src, flags, idx = plane_table(design, k, studies, slices, n_windows, flip_tta)
            self.windows.append(idx)
            self.src.append(torch.from_numpy(src).to(d))
            self.flags.append(torch.from_numpy(flags).to(d) if flip_tta else None)
            self.n_img.append(len(src))
            self.per_view.append(len(src) // studies)
        self.encoders = [Dense8SEncoder(p, dev, n) for p, n in zip(packs, self.n_img)]
        for e in self.encoders:
            if e.n_head < 1:
                raise ValueError("StudyRunner needs packs with a head (H_w, H_b)")
        self.n_out = self.encoders[0].n_head
        self.logits = [torch.zeros((n, self.n_out), dtype=torch.float32, device=d) for n in self.n_img]
        self.views = [torch.zeros((studies, self.n_out), dtype=torch.float32, device=d) for _ in packs]
        self.out = torch.zeros((studies, self.n_out), dtype=torch.float32, device=d)
        self.zbuf = None
        if self.zoom is not None:
            img = int(self.encoders[0].in_shape[2])
            self.zbuf = torch.empty((max(self.n_img), 3, img, img), dtype=torch.float16, device=d)

    @property
    def images_per_call(self) -> int:
        return sum(self.n_img)

    @property
    def launches_per_call(self) -> int:
        per_pass = 2 + 2 * sum(b["L"] for b in self.encoders[0].meta["blocks"]) + \
            sum(1 for b in self.encoders[0].meta["blocks"] if b["trans"])
        passes = sum(-(-n // e.nb) for n, e in zip(self.n_img, self.encoders))
        return per_pass * passes + (len(self.encoders) if self.zoom is not None else 0)

    def run(self, volumes: torch.Tensor) -> torch.Tensor:
        """Study logits [studies, n_out] (the mean over seeds of each seed's view mean)."""
        if (volumes.dim() != 5 or volumes.shape[0] != self.n_windows or volumes.shape[1] != self.studies
                or volumes.shape[2] != self.slices or volumes.dtype != torch.uint8):
            raise ValueError(f"volumes {tuple(volumes.shape)} {volumes.dtype}: expected uint8 "
                             f"[{self.n_windows}, {self.studies}, {self.slices}, H, W]")
        planes = volumes.reshape(-1, volumes.shape[-2], volumes.shape[-1])
        if self.zoom is None:
            # the seeds' passes are independent (own engines, buffers and streams): both start
            # after the caller's stream and run concurrently, so one seed's kernels fill the SMs
            # the other's leave idle at the end of a launch
            cur = torch.cuda.current_stream(self.encoders[0].dev)
            for enc in self.encoders:
                enc.stream.wait_stream(cur)
            for k, enc in enumerate(self.encoders):
                enc.enqueue_u8(planes, self.src[k], self.flags[k], self.logits[k], self.views[k], self.per_view[k])
            for enc in self.encoders:
                cur.wait_stream(enc.stream)
        else:
            # one zoom buffer serves every seed in turn
            from . import ops
            h, w = planes.shape[-2], planes.shape[-1]
            for k, enc in enumerate(self.encoders):
                zb = self.zbuf[:self.n_img[k]]
                ops.zoom(planes, self.src[k], zb, self.n_img[k], h, w, *self.zoom, flags=self.flags[k])
                enc.encode(zb, self.logits[k], self.views[k], self.per_view[k])
        torch.mean(torch.stack(self.views), 0, out=self.out)
        return self.out


def run_shard(runner, volumes, rank: int = 0, world: int = 1, studies=None) -> torch.Tensor:
    """Study logits [n_local, n_out] (float32, host) of this rank's contiguous shard of the studies
    (`studies`: indices into `volumes`, default all of them, in order; `volumes`: uint8 [windows,
    n_volumes, S, H, W] in host memory, pinned for overlap). Batches of `runner.studies` studies are
    copied to the device on a copy stream (two staging buffers, the next batch's copy overlapping
    this batch's encoders), run, and their logits read back into pinned host memory; the last batch
    is padded by repeating its last study. `runner` needs `studies`, `device`, `n_out` and
    `run(volumes_on_device)` (on the current stream)."""
    vols = torch.as_tensor(volumes)
    order = list(range(vols.shape[1])) if studies is None else [int(k) for k in studies]
    start, end = shard(len(order), world, rank)
    B, dev = runner.studies, runner.device
    starts = list(range(start, end, B))
    on_gpu = str(dev).startswith("cuda")
    out = torch.empty((end - start, runner.n_out), dtype=torch.float32, pin_memory=on_gpu)
    shape = (vols.shape[0], B) + tuple(vols.shape[2:])
    stages = [torch.empty(shape, dtype=torch.uint8, device=dev) for _ in range(2 if on_gpu else 1)]

    def fill(st, s0):
        k = min(B, end - s0)
        idx = order[s0:s0 + k]
        runs = []                                    # contiguous runs of volume indices
        for b, v in enumerate(idx):
            if runs and v == runs[-1][1] + runs[-1][2]:
                runs[-1][2] += 1
            else:
                runs.append([b, v, 1])
        for w in range(st.shape[0]):                 # one copy per window and run
            for b, v, c in runs:
                st[w, b:b + c].copy_(vols[w, v:v + c], non_blocking=True)
        if k < B:
            st[:, k:].copy_(st[:, k - 1:k].expand(-1, B - k, *st.shape[2:]))
        return k

    if not on_gpu:
        for s0 in starts:
            k = fill(stages[0], s0)
            out[s0 - start:s0 - start + k].copy_(runner.run(stages[0])[:k])
        return out
    cur = torch.cuda.current_stream(dev)
    copy = torch.cuda.Stream(dev)
    loaded = [torch.cuda.Event() for _ in stages]
    freed: list = [None, None]
    copy.wait_stream(cur)

    def load(j):
        with torch.cuda.stream(copy):
            if freed[j & 1] is not None:
                copy.wait_event(freed[j & 1])
            fill(stages[j & 1], starts[j])
            loaded[j & 1].record(copy)

    if starts:
        load(0)
    for j, s0 in enumerate(starts):
        if j + 1 < len(starts):
            load(j + 1)
        cur.wait_event(loaded[j & 1])
        logits = runner.run(stages[j & 1])
        freed[j & 1] = torch.cuda.Event()
        freed[j & 1].record(cur)
        k = min(B, end - s0)
        out[s0 - start:s0 - start + k].copy_(logits[:k], non_blocking=True)
    cur.synchronize()
    return out


def gather_logits(local: torch.Tensor, n_studies: int, device=None) -> torch.Tensor:
    """All ranks' shard logits, in study order [n_studies, n_out], on every rank (one all_gather of
    the padded shards; the only collective of the study path, outside the timed data path)."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return local
    world = dist.get_world_size()
    per = -(-n_studies // world)
    pad = torch.zeros((per, local.shape[1]), dtype=local.dtype, device=device or local.device)
    pad[:local.shape[0]].copy_(local)
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad)
    rows = [p[:shard(n_studies, world, r)[1] - shard(n_studies, world, r)[0]] for r, p in enumerate(parts)]
    return torch.cat(rows).to(local.device)


def make_volumes(n_studies: int, windows: int = 2, img: int = 512, slices: int = 26, seed: int = 0):
    """uint8 [windows, n_studies, slices, img, img]: study s window w from synthetic volume seed
    seed + 2 s + w."""
    from .synth import volume
    out = np.empty((windows, n_studies, slices, img, img), np.uint8)
    for s in range(n_studies):
        for w in range(windows):
            out[w, s] = volume(seed + 2 * s + w, S=slices, H=img, W=img)
    return out
