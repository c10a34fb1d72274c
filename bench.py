"""Benchmark of the INT8 DenseNet169 encoder at 512 px on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N --steps K --warmup W

Workload: synthetic studies of two crop windows (uint8 volumes of 26 x 512 x
512 slices); two random-init DenseNet169 seeds (42, 43) calibrated at the 99.99th percentile over 8
seeded batches; seed k reads window k (half-window budget); 24 slice triplets per window go
through the fused stem (uint8 gather), 82 dense layers, 3 transitions and the pooling + linear head;
study logits = mean over seeds of the slice-mean logits. A step = one call on `--studies` studies
per GPU (2 x 24 x studies images). Studies are independent: ranks shard them with no collective on
the data path (weak scaling); the logits are gathered on the host.

One JSON line (rank 0): `value` = images/s over all ranks with the study volumes resident in HBM;
`e2e` = the same through the public API with the volumes copied from pinned host memory and the
logits read back every step; `roofline` = the dominant kernel (conv1, all 82 layers) against the
measured HBM copy bandwidth; `cpu_baseline` = the CPU port of the reference's INT8 path on this
host. `--impl reference` times that CPU port alone (rank 0; other ranks exit).
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
    p.add_argument("--kernel", default=None, metavar="KIND:BLOCK:LAYER:N",
                   help="profiling aid: 3 + 1 launches of one kernel (conv1 or conv2 of layer LAYER of "
                        "block BLOCK, 0-based, on N images of random activations), then exit")
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


def roofline(enc, runner, hbm_gbs: float, i8_tops: float, peak_kind: str, vol_dev):
    """From the engine's per-launch CUDA events (one pass, averaged over 3): the dominant kernel
    (conv1, all 82 layers: achieved = its algorithmic bytes / its time, against the measured HBM
    copy bandwidth) and, per kernel family / block and for the whole pass, the fraction
    t_roof / t_measured with t_roof = max(bytes / HBM, 2 MACs / INT8 peak) per launch."""
    prof = enc.profile(planes=vol_dev[0].reshape(-1, vol_dev.shape[-2], vol_dev.shape[-1]), src=runner.src,
                       flags=runner.flags, reps=3)
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


def one_kernel(spec: str, img: int) -> None:
    """Launches one dense-layer kernel 3 + 1 times on random activations, with the tables of a
    seeded random DenseNet169 calibrated on synthetic batches (a small, fixed case for ncu)."""
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
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    if kind == "conv1":
        cin = blk.c0 + 32 * li
        in0 = torch.randint(-127, 128, (rows * blk.c0,), dtype=torch.int8, device="cuda")
        seg = torch.randint(-127, 128, (max(li, 1) * rows * 32,), dtype=torch.int8, device="cuda")
        out = torch.empty(rows * 128, dtype=torch.uint8, device="cuda")
        w1 = dev(ops.prepare_conv1_weights(par[f"L{bi}_{li}_w1"]))
        ab, gd = dev(par[f"L{bi}_{li}_abh"]), dev(par[f"L{bi}_{li}_gdu"])
        for _ in range(4):
            ops.conv1(in0, seg, w1, ab, gd, out, blk.c0 // 32, cin // 32, n, hw, True, err=err)
    elif kind == "conv2":
        x = torch.randint(0, 80, (rows * 128,), dtype=torch.uint8, device="cuda")
        out = torch.empty(rows * 32, dtype=torch.int8, device="cuda")
        w2, sc = dev(ops.prepare_conv2_weights(par[f"L{bi}_{li}_w2k"])), dev(par[f"L{bi}_{li}_c2u"])
        for _ in range(4):
            ops.conv2(x, w2, sc, out, n, blk.h, blk.w, err=err)
    else:
        raise SystemExit(f"--kernel: unknown kind {kind!r} (conv1 or conv2)")
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
    # setup (untimed): packs, engines, the resident pool of synthetic studies
    S = args.studies
    per_view = 24 * (2 if args.flip_tta else 1)
    packs = build_packs(args.img, dev, S * per_view)        # one pass per seed per step
    pool = max(1, min(args.pool, S))
    base = torch.from_numpy(make_volumes(pool, img=args.img, seed=10_000 * (rank + 1)))
    vol_host = base[:, torch.arange(S) % pool].contiguous().pin_memory()      # [2, S, slices, H, W]
    vol_dev = vol_host.to(dev)
    runner = StudyRunner(packs, local, S, flip_tta=args.flip_tta)
    blocks_per_pool = 1
    imgs_per_step = runner.n_img * len(packs)

    def step(i, src):
        b = i % blocks_per_pool
        return runner.run(src[:, b * S:(b + 1) * S])

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for i in range(args.warmup):
        step(i, vol_dev)
    barrier()
    for e in runner.encoders:
        e.check()
    # ---- value: inputs resident in HBM ----
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with Clocks(local) as clk:
        ev0.record()
        for i in range(args.steps):
            step(i, vol_dev)
        ev1.record()
        barrier()
    ms = ev0.elapsed_time(ev1)
    # ---- e2e: the public study loop (`run_shard`) from pinned host volumes: every step copies its
    # studies' volumes host -> device (overlapped with the previous step's encoders) and reads the
    # study logits back into pinned host memory ----
    steps_e2e = args.steps
    order = torch.arange(steps_e2e * S) % S                      # every step's S studies, in order
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    logits_e2e = run_shard(runner, vol_host, studies=order)
    e1.record()
    barrier()
    assert logits_e2e.shape == (steps_e2e * S, runner.n_out) and bool(torch.isfinite(logits_e2e).all())
    ms_e2e = e0.elapsed_time(e1)
    for e in runner.encoders:
        e.check()
    # max over ranks (timing plumbing only)
    t = torch.tensor([ms, ms_e2e], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, ms_e2e = float(t[0]), float(t[1])
    total_imgs = imgs_per_step * args.steps * world
    value = total_imgs / (ms * 1e-3)
    e2e = imgs_per_step * steps_e2e * world / (ms_e2e * 1e-3)
    clocks = clk.summary()
    if rank == 0:
        hbm, i8, kind = peaks()
        roof = roofline(runner.encoders[0], runner, hbm, i8, kind, vol_dev)
        cpu = None
        if not args.no_cpu_baseline:
            cpu = cpu_baseline(args.cpu_seconds, args.img)
            cpu["fp32_torch_images_per_s"] = fp32_cpu(args.img)
        h2d = 2 * S * vol_host[0, 0].numel()
        print(json.dumps({
            "metric": METRIC, "value": round(value, 2), "unit": "images/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "u8xs8->s32", "data": "synthetic",
            "config": {"workload": f"two-seed study batch (BASELINE config 3 structure): {S} studies x 2 seeds x "
                                   f"{runner.per_view} slice triplets per GPU per step, {args.img} px, uint8 "
                                   f"volumes gathered by the stem{', flip TTA' if args.flip_tta else ''}",
                       "img": args.img, "studies_per_gpu_step": S, "images_per_gpu_step": imgs_per_step,
                       "pass_images": runner.encoders[0].nb, "seeds": 2,
                       "parallelism": f"studies sharded over {world} GPU(s), no collective",
                       "library": args.lib or "in-tree libdn8b200.so",
                       "l2": f"no flush: each step's working set (two block arenas, ~{runner.encoders[0].device_mb:.0f} "
                             f"MB per seed) far exceeds the 126 MB L2; the step's {S} studies repeat {pool} distinct synthetic studies"},
            "studies_per_s": round(value / (2 * runner.per_view), 3),
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e, 2), "unit": "images/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(S * runner.n_out * 4), "steps": steps_e2e,
                    "api": "infer.run_shard (pinned host volumes -> study logits in pinned host memory)"},
            "gpu_launches": runner.launches_per_call * args.steps,
            "clocks": clocks,
        }), flush=True)
    for e in runner.encoders:
        e.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
