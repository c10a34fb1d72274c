"""Benchmark of the INT8 DenseNet169 encoder at 512 px on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N --steps K --warmup W

Workload: synthetic studies of two crop windows (uint8 volumes of 26 x 512 x
512 slices); two random-init DenseNet169 seeds (42, 43) calibrated at the 99.99th percentile over 8
seeded batches; each seed reads half of the study's 48 slice-triplet windows (the reference's
`parx` design: seed f keeps position p of slot s where (p + s + f) % 2 == 0); the windows go
through the fused stem (uint8 gather), 82 dense layers, 3 transitions and the pooling + linear head;
study logits = mean over seeds of the per-seed window-mean logits. A step = one call on `--studies`
studies per GPU (2 x 24 x studies images). Studies are independent: ranks shard them with no
collective on the data path (weak scaling); the logits are gathered on the host.

One JSON line (rank 0): `value` = images/s over all ranks with the study volumes resident in HBM;
`e2e` = the same through the public API with the volumes copied from pinned host memory and the
logits read back every step; `roofline` = the dominant kernel (conv1, all 82 layers) against the
measured HBM copy bandwidth, with every kernel family in `roofline.network` (`frac`: one pass profiled
launch by launch; `step_frac`: the timed step, whose two seed passes overlap, against the same
roofline time per pass); `sweep` = BASELINE
config 4 (1, 4, 16, 64 studies per GPU per step); `layers` = BASELINE config 1 (one launch per
layer shape on 24 images, summed per kernel and block); `cpu_baseline` = the CPU port of the
reference's INT8 path on this host. `--impl reference` times that CPU port alone (rank 0; other
ranks exit); `--layers [--impl reference]` prints the config-1 table of this repository's kernels
(or of the reference's own sm_100 kernels) alone.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count() or 1))   # oracle threads (set before loading)

METRIC = "INT8 DenseNet169 512px images/s & studies/s at 1/2/4/8 B200; % per-layer roofline"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=40)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--studies", type=int, default=16, help="studies per GPU per step")
    p.add_argument("--pool", type=int, default=4, help="distinct synthetic studies per GPU (repeated to fill a step)")
    p.add_argument("--img", type=int, default=512)
    p.add_argument("--flip-tta", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-seconds", type=float, default=12.0)
    p.add_argument("--lib", default=None, metavar="PATH",
                   help="load this build of libdn8b200.so instead of the in-tree one (same-box A/B of two builds)")
    p.add_argument("--design", default="parx", help="window design of the two seeds (infer.member_windows)")
    p.add_argument("--sweep", default="1,4,16,64",
                   help="studies per GPU of the batch sweep (BASELINE config 4: 24, 96, 384, 1536 images per seed)")
    p.add_argument("--no-sweep", action="store_true")
    p.add_argument("--no-layers", action="store_true", help="skip the config-1 micro-benchmark summary")
    p.add_argument("--layers", action="store_true",
                   help="only the config-1 micro-benchmark: one JSON line with every shape (ours, or with "
                        "--impl reference the reference's own sm_100 kernels), then exit")
    p.add_argument("--kernel", default=None, metavar="KIND:BLOCK:LAYER:N",
                   help="profiling aid: 3 + 1 launches of one kernel (conv1 / conv2 of layer LAYER of "
                        "block BLOCK, 0-based, trans of block BLOCK, or stem, on N images of random "
                        "activations in the engine's tile-major layout), then exit")
    return p.parse_args()


def peaks():
    """(HBM GB/s, dense INT8 TOP/s, source). The INT8 peak is taken as twice the measured dense bf16
    GEMM throughput (the tensor core's INT8 rate is twice its bf16 rate)."""
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return float(d["hbm_gbs"]), 2 * float(d["bf16_tflops"]), "measured"
    return FALLBACK_HBM_GBS, 2 * FALLBACK_BF16_TFLOPS, "fallback"


# ---- clocks during the timed region ------------------------------------------------------------
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.proc, self.rows = gpu, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            out, _ = self.proc.communicate(timeout=10)
            self.rows = [r.split(", ") for r in out.strip().splitlines() if r.count(",") >= 8]

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ---- CPU baseline: the port of the reference's INT8 path (oracle/) on this host -----------------
class CpuPort:
    """The port of the reference's INT8 path (oracle/, float64 emulate arithmetic) on this host's
    cores: one random-init seed-42 network, tables calibrated on two synthetic images."""

    def __init__(self, img: int):
        import torch
        from oracle import oracle as orc
        from rsna_knee_efficiency_b200 import densenet, pack as packmod, quant, synth
        torch.manual_seed(0)
        m = densenet.random_init(densenet.DenseNet169(), 42)
        cal = quant.calibrate(m, [torch.from_numpy(b) for b in synth.calibration_batches(1, 2, img, seed=1042)])
        plan = quant.make_plan(m, cal, img)
        self.orc, self.img = orc, img
        self.par, self.meta = quant.kernel_params(plan), packmod.pack_meta(plan, 1)
        self.x = synth.triplets(synth.volume(1, H=img, W=img))
        self.done = 0

    def sample(self, seconds: float) -> dict:
        """Images through the port for at least `seconds` (at least one image)."""
        done, t0 = 0, time.perf_counter()
        while True:
            self.orc.forward(self.par, self.meta, self.x[(self.done + done) % len(self.x)][None],
                             mode=self.orc.EMULATE)
            done += 1
            if time.perf_counter() - t0 > seconds:
                break
        dt = time.perf_counter() - t0
        self.done += done
        return {"value": round(done / dt, 4), "unit": "images/s", "cores": int(os.environ["OMP_NUM_THREADS"]),
                "kind": "port", "sample": f"{done} image(s) of 3x{self.img}x{self.img} (slice triplets of one "
                                          f"synthetic volume) through oracle/ in {dt:.1f} s"}


def cpu_baseline(seconds: float, img: int) -> dict:
    return CpuPort(img).sample(seconds)


def fp32_cpu(img: int, seconds: float = 6.0):
    """The reference's fp32 CPU path (DenseNet169 forward, batch 4) on this host, for context."""
    import torch
    from rsna_knee_efficiency_b200 import densenet
    torch.set_num_threads(os.cpu_count() or 1)
    m = densenet.random_init(densenet.DenseNet169(), 42)
    x = torch.rand(4, 3, img, img)
    with torch.no_grad():
        m(x)
        done, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            m(x)
            done += 4
    return round(done / (time.perf_counter() - t0), 3)


def run_reference(args, rank: int):
    if rank != 0:
        return
    port = CpuPort(args.img)
    per_step = args.cpu_seconds / max(1, args.steps)
    for _ in range(args.warmup):
        port.sample(0.0)
    t = [port.sample(per_step) for _ in range(args.steps)]
    imgs = statistics.fmean(float(r["value"]) for r in t)
    base = dict(t[-1])
    base["value"] = round(imgs, 4)
    base["sample"] = f"{args.steps} step(s) of >= {per_step:.1f} s each; last: {t[-1]['sample']}"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(imgs, 4), "unit": "images/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000.0 / imgs, 1), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8xs8->s32", "data": "synthetic",
        "config": {"workload": "reference INT8 path on the host CPU (oracle/ port of dense8s.emulate): "
                               f"slice-triplet images at {args.img} px, one per sample", "img": args.img},
        "cpu_baseline": base,
        "e2e": {"value": round(imgs, 4), "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "studies_per_s": round(imgs / 48.0, 5),
    }), flush=True)


# ---- the GPU arm ------------------------------------------------------------------------------
MAX_PASS = 768            # images per engine pass: conv1 addresses a block-1 launch below 2^31 bytes (< 1024 images)
SWEEP_IMAGES = 24_000     # images per sweep point (steps = this / images per step, at least 3)


def with_pass(pack: dict, n: int) -> dict:
    """The same tables with `n` images per engine pass."""
    return {**pack, "meta": {**pack["meta"], "n": int(n)}}


def build_packs(img: int, dev: str, n: int):
    import torch
    from rsna_knee_efficiency_b200 import densenet, pack as packmod, quant, synth
    packs = []
    for seed in (42, 43):
        m = densenet.random_init(densenet.DenseNet169(), seed).to(dev)
        batches = [torch.from_numpy(b).to(dev) for b in synth.calibration_batches(8, 4, img, seed=1000 + seed)]
        cal = quant.calibrate(m, batches, method="pct", pct=99.99)
        plan = quant.make_plan(m.cpu(), cal, img)
        packs.append(packmod.make_pack(plan, n, densenet.random_head(seed)))
    return packs


def launch_work(kind: str, blk: dict, l: int, n: int, img: int) -> tuple[float, float]:
    """(algorithmic HBM bytes, MACs) of one launch over n images: every tensor read or written once.
    conv1: store c_in + bottleneck 128 per pixel (+ weights); conv2: bottleneck 128 + slot 32 per
    pixel (+ weights); transition: c_tot per input pixel read, c_tot / 2 per pooled pixel written,
    MACs of the exact integer form (four 1x1 outputs per pooled pixel); stem: the three uint8 planes
    read and block 1's 64-channel input written, 7x7x3 MACs per conv output; head: last store read."""
    hw = blk["h"] * blk["w"]
    if kind == "conv1":
        cin = blk["c0"] + 32 * l
        return n * hw * (cin + 128) + cin * 128, n * hw * 128 * cin
    if kind == "conv2":
        return n * hw * 160 + 36864, n * hw * 32 * 1152
    ctot = blk["c0"] + 32 * blk["L"]
    if kind == "trans":
        return n * hw * ctot + n * hw // 4 * ctot // 2, n * hw * ctot * ctot // 2
    if kind == "stem":
        return n * (3 * img * img + 64 * hw), n * (img // 2) ** 2 * 64 * 147
    return n * hw * ctot, 0


def roofline(runner, hbm_gbs: float, i8_tops: float, peak_kind: str, vol_dev):
    """From the engine's per-launch CUDA events (one pass of the first seed, averaged over 3): the
    dominant kernel (conv1, all 82 layers: achieved = its algorithmic bytes / its time, against the
    measured HBM copy bandwidth) and, per kernel family / block and for the whole pass, the fraction
    t_roof / t_measured with t_roof = max(bytes / HBM, 2 MACs / INT8 peak) per launch."""
    enc = runner.encoders[0]
    prof = enc.profile(planes=vol_dev.reshape(-1, vol_dev.shape[-2], vol_dev.shape[-1]), src=runner.src[0],
                       flags=runner.flags[0], reps=3)
    blocks = enc.meta["blocks"]
    n, img = enc.nb, enc.in_shape[2]
    per = {}
    for kind, b, l, ms in prof:
        by, macs = launch_work(kind, blocks[b], l, n, img)
        t_roof = max(by / (hbm_gbs * 1e9), 2 * macs / (i8_tops * 1e12)) * 1e3
        for key in (kind, f"{kind}.b{b}"):
            k = per.setdefault(key, [0.0, 0.0, 0.0, 0])
            k[0] += by
            k[1] += ms
            k[2] += t_roof
            k[3] += 1
    c1 = per["conv1"]
    achieved = c1[0] / (c1[1] * 1e-3) / 1e9
    # DRAM traffic of conv1 over one pass from an ncu capture (profiles/), scaled to this pass size
    # (traffic grows with the images of a pass: every launch streams its layer's activations)
    traffic = None
    tf = ROOT / "profiles" / "dram_traffic_encoder_512_b384.json"
    if tf.exists():
        t = json.loads(tf.read_text())
        if t.get("conv1_dram_bytes_per_pass") and t.get("pass_images"):
            traffic = int(t["conv1_dram_bytes_per_pass"] * n / t["pass_images"])
    summary = {k: {"launches": v[3], "ms": round(v[1], 3), "GBps": round(v[0] / (v[1] * 1e-3) / 1e9, 1),
                   "roof_ms": round(v[2], 4), "frac": round(v[2] / v[1], 3)} for k, v in per.items()}
    kinds = [v for k, v in per.items() if "." not in k]
    roof_ms = sum(v[2] for v in kinds)
    pass_ms = sum(v[1] for v in kinds)
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_gbs, "unit": "GB/s",
            "frac": round(achieved / hbm_gbs, 4), "traffic": traffic, "peak_source": peak_kind,
            "kernel": "conv1 (gemm_kernel, all 82 launches of one pass; traffic per pass)",
            "algorithmic_bytes_per_pass": int(c1[0]),
            "network": {"frac": round(roof_ms / pass_ms, 4), "pass_ms": round(pass_ms, 3),
                        "roof_ms": round(roof_ms, 3), "int8_tops": i8_tops, "per_kind": summary}}


# ---- the single-layer micro-benchmark ----------------------------------------
LAYER_IMAGES = 24
# (side, block input channels c0, conv1 input channels swept) of blocks 1-4 at 512 px
LAYER_BLOCKS = [(128, 64, range(64, 257, 32)), (64, 128, range(128, 513, 32)),
                (32, 256, range(256, 1281, 32)), (16, 640, range(640, 1633, 32))]
TRANS_SHAPES = [(128, 256), (64, 512), (32, 1280)]          # (side, c_tot) of transitions 1-3
HEAD_SHAPE = (16, 640, 1664)                                # (side, c0, c_tot) of the last block
FLUSH_BYTES = 512 << 20                                     # > the 126 MB L2, written before every launch


class LayerData:
    """Seeded config-1 inputs on the device: int8 stores drawn from the requantised ReLU
    distribution (half zeros, the rest |N(0, 40)| clipped to 127), int8 weights ~U[-127, 127], BN
    scale / shift ~N(1, 0.1) / N(0, 0.1) folded into the prologue tables (A = scale / 40, B = shift),
    epilogue scales that spread the outputs over the u8 / int8 range."""

    def __init__(self, seed: int = 1):
        import torch
        self.torch = torch
        self.g = torch.Generator(device="cuda").manual_seed(seed)
        self.rng = __import__("numpy").random.default_rng(seed)

    def store(self, nbytes: int):
        t = self.torch
        v = t.randn(nbytes, generator=self.g, device="cuda").mul_(40).abs_().clamp_(max=127).round_()
        v[t.rand(nbytes, generator=self.g, device="cuda") < 0.5] = 0
        return v.to(t.int8)

    def u8(self, nbytes: int):
        return self.torch.randint(0, 256, (nbytes,), generator=self.g, device="cuda", dtype=self.torch.uint8)

    def weights(self, shape):
        return self.rng.integers(-127, 128, size=shape, dtype=__import__("numpy").int64).astype("int8")

    def prologue(self, c: int):
        """(ab [c, 2] float32, abh [c/2, 4] fp16 bits)."""
        import numpy as np
        from rsna_knee_efficiency_b200 import quant
        ab = np.stack([self.rng.normal(1, 0.1, c) / 40.0, self.rng.normal(0, 0.1, c)], 1).astype(np.float32)
        return ab, quant._abh(ab)

    def epilogue(self, cout: int, k_in: int, u8_out: bool):
        import numpy as np
        g = self.rng.normal(1, 0.1, cout) / (4 * 128 * 73 * np.sqrt(k_in))
        g = g * (1.0 if u8_out else 127.0)
        return np.stack([g, np.zeros(cout)], 1).astype(np.float32)


def _time_launch(fn, flush, reps: int = 7, warm: int = 2) -> float:
    """Median device ms of `fn` (one launch on the current stream), each launch after an L2 flush
    (a 512 MB write), bracketed by CUDA events on the launching stream. The flush also keeps the
    GPU busy long enough for the host to enqueue the launch, so the events time the kernel alone."""
    import torch
    for _ in range(warm):
        flush()
        fn()
    torch.cuda.synchronize()
    evs = []
    for _ in range(reps):
        flush()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        evs.append((e0, e1))
    torch.cuda.synchronize()
    return statistics.median(a.elapsed_time(b) for a, b in evs)


def _roof_ms(nbytes: float, macs: float, hbm: float, i8: float) -> float:
    return max(nbytes / (hbm * 1e9), 2 * macs / (i8 * 1e12)) * 1e3


def layer_shapes():
    """Every timed launch of config 1: (kind, block, c_in or c_tot, side, c0)."""
    out = []
    for bi, (side, c0, cins) in enumerate(LAYER_BLOCKS):
        out += [("conv1", bi, cin, side, c0) for cin in cins]
        out.append(("conv2", bi, 128, side, c0))
    out += [("trans", bi, ctot, side, ctot) for bi, (side, ctot) in enumerate(TRANS_SHAPES)]
    out.append(("head", 3, HEAD_SHAPE[2], HEAD_SHAPE[0], HEAD_SHAPE[1]))
    return out


def layer_work(kind: str, c: int, rows: int) -> tuple[float, float]:
    """(algorithmic HBM bytes, MACs) of one config-1 launch over `rows` pixels (as `launch_work`)."""
    if kind == "conv1":
        return rows * (c + 128) + c * 128, rows * 128 * c
    if kind == "conv2":
        return rows * 160 + 36864, rows * 32 * 1152
    if kind == "trans":
        return rows * c + rows // 4 * c // 2 + c * c // 2, rows * c * c // 2
    return rows * c, 0


def layers_ours(hbm: float, i8: float, tile: bool = False) -> list:
    """Config 1 through this repository's kernel entry points (include/dn8.h), one launch per
    shape; `tile`: conv1 reads the tile-major block store."""
    import numpy as np
    import torch
    from rsna_knee_efficiency_b200 import ops
    d = LayerData()
    flush_buf = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    flush = lambda: flush_buf.fill_(1)                                  # noqa: E731
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()    # noqa: E731
    n, rows_out = LAYER_IMAGES, []
    for kind, bi, c, side, c0 in layer_shapes():
        hw = side * side
        rows = n * hw
        if kind == "conv1":
            G = c // 32
            out = torch.empty(rows * 128, dtype=torch.uint8, device="cuda")
            w = dev(ops.prepare_conv1_weights(d.weights((G, 128, 32))))
            abh_d = dev(d.prologue(c)[1])
            gd = dev(d.epilogue(128, c, True))
            if tile:
                st = d.store(-(-rows // 128) * 128 * c)
                fn = lambda: ops.conv1(st, None, w, abh_d, gd, out, 0, G, n, hw, True, err=err,  # noqa: E731
                                       tile_groups=G)
            else:
                in0, seg = d.store(rows * c0), d.store(max(rows * (c - c0), 16))
                fn = lambda: ops.conv1(in0, seg, w, abh_d, gd, out, c0 // 32, G, n, hw, True, err=err)  # noqa: E731
        elif kind == "conv2":
            x = d.u8(rows * 128)
            out = torch.empty(rows * 32, dtype=torch.int8, device="cuda")
            w2 = dev(ops.prepare_conv2_weights(d.weights((4, 9, 32, 32))))
            sc = dev(d.epilogue(32, 1152, False)[:, 0].copy())
            fn = lambda: ops.conv2(x, w2, sc, out, n, side, side, err=err)  # noqa: E731
        elif kind == "trans":
            G = c // 32
            in0, seg = d.store(rows * c0 // 2), d.store(rows * c0 // 2)
            out = torch.empty(rows // 4 * c // 2, dtype=torch.int8, device="cuda")
            tw = dev(ops.prepare_trans_weights(d.weights((G, c // 2, 32))))
            _, abh = d.prologue(c)
            abh_d, gd = dev(abh), dev(d.epilogue(c // 2, c, False))
            fn = lambda: ops.trans(in0, seg, tw, abh_d, gd, out, G // 2, G, n, side, side, True, err=err)  # noqa: E731
        else:
            in0, seg = d.store(rows * c0), d.store(rows * (c - c0))
            fab = dev(d.prologue(c)[0])
            feat = torch.empty((n, c), dtype=torch.float32, device="cuda")
            fn = lambda: ops.head(in0, seg, fab, c0 // 32, c // 32, n, hw, feat=feat)  # noqa: E731
        ms = _time_launch(fn, flush)
        by, macs = layer_work(kind, c, rows)
        roof = _roof_ms(by, macs, hbm, i8)
        rows_out.append({"kind": kind, "block": bi, "c": c, "side": side, "rows": rows, "ms": round(ms, 4),
                         "GBps": round(by / (ms * 1e-3) / 1e9, 1), "roof_ms": round(roof, 4),
                         "frac": round(roof / ms, 3)})
        del fn
    torch.cuda.synchronize()
    if int(err.item()) != 0:
        raise RuntimeError(f"config 1 micro-benchmark: device error {int(err.item())}")
    return rows_out


def layers_reference(hbm: float, i8: float) -> list:
    """Config 1 through the reference's own sm_100 kernels (oracle/_ref, built from its source),
    launched as the reference launches them: conv1_w64_pl, conv2_t8x32_pl (128 x 128) /
    conv2_t16x16_pl, trans_w0 / trans_w1 (where c_out allows) and trans_q128, final_q."""
    import numpy as np
    import torch
    from oracle import refcu
    from rsna_knee_efficiency_b200 import quant
    if not refcu.available():
        raise RuntimeError("oracle/_ref not built (make -C oracle ref REF_DIR=<reference>/src/knee)")
    rk = refcu.RefKernels(0)
    d = LayerData()
    flush_buf = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    flush = lambda: flush_buf.fill_(1)                                  # noqa: E731
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()    # noqa: E731
    n, rows_out = LAYER_IMAGES, []
    for kind, bi, c, side, c0 in layer_shapes():
        hw = side * side
        rows = n * hw
        variants = []
        if kind == "conv1":
            G = c // 32
            in0, seg = d.store(rows * c0), d.store(max(rows * (c - c0), 16))
            out = torch.empty(rows * 128, dtype=torch.uint8, device="cuda")
            w = dev(quant._chunked(d.weights((128, c)).astype(np.int8)))
            abh = dev(d.prologue(c)[1])
            gd = dev(d.epilogue(128, c, True))
            variants.append(("conv1_w64_pl", lambda: rk.conv1(in0, seg, w, abh, gd, out, c0 // 32, G, n, hw, side)))
        elif kind == "conv2":
            x = d.u8(rows * 128)
            out = torch.empty(rows * 32, dtype=torch.int8, device="cuda")
            w2 = dev(d.weights((4, 9, 32, 32)))
            sc = dev(d.epilogue(32, 1152, False)[:, 0].copy())
            kern = "t8x32_pl" if side == 128 else "t16x16_pl"
            variants.append((f"conv2_{kern}", lambda: rk.conv2(x, w2, sc, out, n, side, side, kern)))
        elif kind == "trans":
            G, cout = c // 32, c // 2
            in0, seg = d.store(rows * c0 // 2), d.store(rows * c0 // 2)
            out = torch.empty(rows // 4 * cout, dtype=torch.int8, device="cuda")
            tw8 = d.weights((G, cout, 32))
            ab, abh = d.prologue(c)
            gdk = d.epilogue(cout, c, False)
            twh, abh_d, abd = dev(tw8.astype(np.float16)), dev(abh), dev(ab)
            gdf, gd = dev(gdk * 4), dev(gdk)
            tw = dev(tw8)
            for kind_w, bn in (("w0", 128), ("w1", 256)):
                if cout % bn == 0:
                    variants.append((f"trans_{kind_w}", lambda k=kind_w: rk.trans_w(k, in0, seg, twh, abh_d, gdf, out,
                                                                                  G // 2, G, n, side, side)))
            variants.append(("trans_q128", lambda: rk.trans_q128(in0, seg, tw, abd, gd, out, G // 2, G, n, side,
                                                                 side)))
        else:
            in0, seg = d.store(rows * c0), d.store(rows * (c - c0))
            fab = dev(d.prologue(c)[0])
            feat = torch.empty((n, c), dtype=torch.float32, device="cuda")
            variants.append(("final_q", lambda: rk.final_q(in0, c0 // 32, seg, n, hw, fab, feat, c)))
        by, macs = layer_work(kind, c, rows)
        roof = _roof_ms(by, macs, hbm, i8)
        for name, fn in variants:
            ms = _time_launch(fn, flush)
            rows_out.append({"kind": kind, "kernel": name, "block": bi, "c": c, "side": side, "rows": rows,
                             "ms": round(ms, 4), "GBps": round(by / (ms * 1e-3) / 1e9, 1),
                             "roof_ms": round(roof, 4), "frac": round(roof / ms, 3)})
        variants.clear()
    torch.cuda.synchronize()
    return rows_out


def layers_summary(rows: list) -> dict:
    """Per (kind, block): launches, ms, roof ms, fraction = sum roof / sum ms (each kind's fastest
    kernel where a shape has several)."""
    best = {}
    for r in rows:
        key = (r["kind"], r["block"], r["c"])
        if key not in best or r["ms"] < best[key]["ms"]:
            best[key] = r
    agg = {}
    for (kind, bi, _), r in best.items():
        a = agg.setdefault(f"{kind}.b{bi}", [0, 0.0, 0.0])
        a[0] += 1
        a[1] += r["ms"]
        a[2] += r["roof_ms"]
    return {k: {"launches": v[0], "ms": round(v[1], 4), "roof_ms": round(v[2], 4), "frac": round(v[2] / v[1], 3)}
            for k, v in agg.items()}


def one_kernel(spec: str, img: int) -> None:
    """Launches one kernel 3 + 1 times on random activations in the engine's layouts (tile-major
    block store), with the tables of a seeded random DenseNet169 calibrated on synthetic batches (a
    small, fixed case for ncu): conv1 / conv2 of layer LAYER of block BLOCK, the transition of block
    BLOCK, or the stem (BLOCK and LAYER unused) on N images."""
    import numpy as np
    import torch
    from rsna_knee_efficiency_b200 import densenet, ops, quant, synth
    kind, bi, li, n = spec.split(":")
    bi, li, n = int(bi), int(li), int(n)
    torch.manual_seed(0)
    m = densenet.random_init(densenet.DenseNet169(), 42)
    cal = quant.calibrate(m, [torch.from_numpy(b) for b in synth.calibration_batches(2, 2, img, seed=1042)])
    plan = quant.make_plan(m, cal, img)
    par = quant.kernel_params(plan)
    blk = plan.blocks[bi]
    hw, rows = blk.h * blk.w, n * blk.h * blk.w
    tiles = -(-rows // 128)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()    # noqa: E731
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    Gt = blk.c_tot // 32
    if kind == "conv1":
        cin = blk.c0 + 32 * li
        store = torch.randint(-127, 128, (tiles * Gt * 4096,), dtype=torch.int8, device="cuda")
        out = torch.empty(rows * 128, dtype=torch.uint8, device="cuda")
        w1 = dev(ops.prepare_conv1_weights(par[f"L{bi}_{li}_w1"]))
        ab, gd = dev(par[f"L{bi}_{li}_abh"]), dev(par[f"L{bi}_{li}_gdu"])
        for _ in range(4):
            ops.conv1(store, None, w1, ab, gd, out, blk.c0 // 32, cin // 32, n, hw, True, err=err, tile_groups=Gt)
    elif kind == "conv2":
        x = torch.randint(0, 80, (rows * 128,), dtype=torch.uint8, device="cuda")
        store = torch.empty(tiles * Gt * 4096, dtype=torch.int8, device="cuda")
        w2, sc = dev(ops.prepare_conv2_weights(par[f"L{bi}_{li}_w2k"])), dev(par[f"L{bi}_{li}_c2u"])
        for _ in range(4):
            ops.conv2(x, w2, sc, store, n, blk.h, blk.w, err=err, tile_groups=Gt, group=blk.c0 // 32 + li)
    elif kind == "trans":
        nxt = plan.blocks[bi + 1]
        store = torch.randint(-127, 128, (tiles * Gt * 4096,), dtype=torch.int8, device="cuda")
        Gn = nxt.c_tot // 32
        out = torch.empty(-(-(rows // 4) // 128) * Gn * 4096, dtype=torch.int8, device="cuda")
        tw = dev(ops.prepare_trans_weights(par[f"T{bi}_w"]))
        ab, gd = dev(par[f"T{bi}_abh"]), dev(par[f"T{bi}_gd"])
        for _ in range(4):
            ops.trans(store, None, tw, ab, gd, out, blk.c0 // 32, Gt, n, blk.h, blk.w, True, err=err,
                      tile_groups=Gt, out_tile_groups=Gn)
    elif kind == "stem":
        b0 = plan.blocks[0]
        planes = torch.from_numpy(synth.volume(3, H=img, W=img)).cuda()
        src = torch.tensor([[i % 24, i % 24 + 1, i % 24 + 2, 0] for i in range(n)], dtype=torch.int32).cuda()
        G0t = b0.c_tot // 32
        out = torch.empty(-(-(n * b0.h * b0.w) // 128) * G0t * 4096, dtype=torch.int8, device="cuda")
        w8, kc = dev(ops.prepare_stem_weights(par["S_w8"])), dev(par["S_kc"])
        for _ in range(4):
            ops.stem(planes, w8, kc, out, n, img, img, src=src, err=err, tile_groups=G0t)
    else:
        raise SystemExit(f"--kernel: unknown kind {kind!r} (conv1, conv2, trans or stem)")
    torch.cuda.synchronize()
    if int(err.item()) != 0:
        raise SystemExit(f"--kernel {spec}: device error {int(err.item())}")
    print(f"--kernel {spec}: 4 launches, no device error")


def main():
    args = parse()
    if args.lib:
        from rsna_knee_efficiency_b200 import _native
        _native.LIB_PATH = Path(args.lib).resolve()
        _native._lib = None
    if args.kernel:
        one_kernel(args.kernel, args.img)
        return
    if args.layers:
        if int(os.environ.get("RANK", "0")) != 0:
            return
        import torch
        torch.cuda.set_device(0)
        hbm, i8, kind = peaks()
        ref = args.impl == "reference"
        rows = layers_reference(hbm, i8) if ref else layers_ours(hbm, i8)
        print(json.dumps({"impl": "reference" if ref else "ours",
                          "what": f"BASELINE config 1 micro-benchmark, {LAYER_IMAGES} images per shape, L2 flushed "
                                  "before each launch, median of 7 launches (CUDA events on the launching stream)",
                          "peak_hbm_gbs": hbm, "peak_int8_tops": i8, "peak_source": kind,
                          "per_block": layers_summary(rows), "shapes": rows}), flush=True)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    import torch
    import torch.distributed as dist
    from rsna_knee_efficiency_b200.infer import StudyRunner, make_volumes, run_shard
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device(dev))
    # setup (untimed): tables of both seeds (calibrated once), engines, the resident synthetic studies
    S = args.studies
    plans = build_packs(args.img, dev, MAX_PASS)
    sweep = [] if args.no_sweep else [int(v) for v in args.sweep.split(",") if v]

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(*vals):
        t = torch.tensor(vals, dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return [float(v) for v in t]

    def setup(studies):
        per_seed = studies * 24 * (2 if args.flip_tta else 1)
        runner = StudyRunner([with_pass(p, min(per_seed, MAX_PASS)) for p in plans], local, studies,
                             flip_tta=args.flip_tta, design=args.design)
        pool = max(1, min(args.pool, studies))
        base = torch.from_numpy(make_volumes(pool, img=args.img, seed=10_000 * (rank + 1)))
        vol_host = base[:, torch.arange(studies) % pool].contiguous().pin_memory()   # [2, S, slices, H, W]
        return runner, vol_host, vol_host.to(dev), pool

    def measure(runner, vol_host, vol_dev, studies, steps, warmup, clocks=None):
        """(device ms of `steps` resident steps, device ms of the e2e loop over `steps` steps), each
        the max over ranks, after `warmup` untimed steps."""
        for _ in range(warmup):
            runner.run(vol_dev)
        barrier()
        for e in runner.encoders:
            e.check()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        if clocks is not None:
            clocks.__enter__()
        ev0.record()
        for _ in range(steps):
            runner.run(vol_dev)
        ev1.record()
        barrier()
        if clocks is not None:
            clocks.__exit__(None, None, None)
        ms = ev0.elapsed_time(ev1)
        # e2e: the public study loop (`run_shard`) from pinned host volumes: every step copies its
        # studies' volumes host -> device (overlapped with the previous step's encoders) and reads
        # the study logits back into pinned host memory
        order = torch.arange(steps * studies) % studies
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        logits = run_shard(runner, vol_host, studies=order)
        e1.record()
        barrier()
        assert logits.shape == (steps * studies, runner.n_out) and bool(torch.isfinite(logits).all())
        for e in runner.encoders:
            e.check()
        return max_over_ranks(ms, e0.elapsed_time(e1))

    hbm, i8, peak_kind = peaks()
    runner, vol_host, vol_dev, pool = setup(S)
    imgs_per_step = runner.images_per_call
    clk = Clocks(local)
    ms, ms_e2e = measure(runner, vol_host, vol_dev, S, args.steps, args.warmup, clk)
    value = imgs_per_step * args.steps * world / (ms * 1e-3)
    e2e = imgs_per_step * args.steps * world / (ms_e2e * 1e-3)
    imgs_per_study = imgs_per_step / S
    roof = roofline(runner, hbm, i8, peak_kind, vol_dev) if rank == 0 else None
    config_pass = runner.encoders[0].nb
    if roof is not None:
        # the whole step against its roofline: the step runs imgs_per_step / config_pass passes (the
        # seeds' passes overlap on their streams), each with the profiled pass's roofline time
        roof["network"]["step_frac"] = round(roof["network"]["roof_ms"] * imgs_per_step / config_pass
                                             / (ms / args.steps), 4)
    device_mb = runner.encoders[0].device_mb
    launches = runner.launches_per_call * args.steps
    n_out = runner.n_out
    h2d = int(vol_host[:, 0].numel() * S)
    for e in runner.encoders:
        e.close()
    del runner, vol_dev
    torch.cuda.empty_cache()

    # ---- per-GPU batch sweep (images per seed pass per GPU) ----
    sweep_out = []
    for sv in sweep:
        r2, vh, vd, _ = setup(sv)
        steps = max(3, -(-SWEEP_IMAGES // (r2.images_per_call)))
        m1, m2 = measure(r2, vh, vd, sv, steps, 3)
        ips = r2.images_per_call * steps * world / (m1 * 1e-3)
        row = {"studies_per_gpu": sv, "images_per_gpu_batch": r2.n_img[0], "pass_images": r2.encoders[0].nb,
               "passes_per_seed": -(-r2.n_img[0] // r2.encoders[0].nb), "steps": steps,
               "images_per_s": round(ips, 1), "studies_per_s": round(ips / (r2.images_per_call / sv), 2),
               "e2e_images_per_s": round(r2.images_per_call * steps * world / (m2 * 1e-3), 1),
               "ms_per_step": round(m1 / steps, 3)}
        if rank == 0:
            net = roofline(r2, hbm, i8, peak_kind, vd)["network"]
            row["network_frac"] = net["frac"]
            row["step_frac"] = round(net["roof_ms"] * r2.images_per_call / r2.encoders[0].nb / (m1 / steps), 4)
        sweep_out.append(row)
        for e in r2.encoders:
            e.close()
        del r2, vd
        torch.cuda.empty_cache()
        barrier()

    # ---- the single-layer micro-benchmark (rank 0, after the timed runs) ----
    layers = None
    if rank == 0 and not args.no_layers:
        layers = layers_summary(layers_ours(hbm, i8))

    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline:
            cpu = cpu_baseline(args.cpu_seconds, args.img)
            cpu["fp32_torch_images_per_s"] = fp32_cpu(args.img)
        print(json.dumps({
            "metric": METRIC, "value": round(value, 2), "unit": "images/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "u8xs8->s32", "data": "synthetic",
            "config": {"workload": f"two-seed study batch (BASELINE config 3 structure): {S} studies per GPU per "
                                   f"step, 2 crop windows x 24 slice triplets per study, seed k reads the "
                                   f"'{args.design}' half of the windows, {args.img} px, uint8 volumes gathered by "
                                   f"the stem{', flip TTA' if args.flip_tta else ''}",
                       "img": args.img, "studies_per_gpu_step": S, "images_per_gpu_step": imgs_per_step,
                       "pass_images": config_pass, "seeds": 2, "window_design": args.design,
                       "parallelism": f"studies sharded over {world} GPU(s), no collective",
                       "library": args.lib or "in-tree libdn8b200.so",
                       "l2": f"no flush: each step's working set (two block arenas, ~{device_mb:.0f} MB per seed) far "
                             f"exceeds the 126 MB L2; the step's {S} studies repeat {pool} distinct synthetic studies"},
            "studies_per_s": round(value / imgs_per_study, 3),
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e, 2), "unit": "images/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": int(S * n_out * 4), "steps": args.steps,
                    "api": "infer.run_shard (pinned host volumes -> study logits in pinned host memory)"},
            "gpu_launches": launches,
            "clocks": clk.summary(),
            "sweep": {"what": "BASELINE config 4: studies per GPU per step (24 images per seed pass per study; "
                              f"passes of at most {MAX_PASS} images), at this world size", "points": sweep_out},
            "layers": None if layers is None else
            {"what": f"BASELINE config 1: one launch per shape on {LAYER_IMAGES} images, L2 flushed before each "
                     "launch, summed per kernel and block (`--layers` prints every shape)", "per_block": layers},
        }), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
