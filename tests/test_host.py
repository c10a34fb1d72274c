"""Host logic without a GPU: pack format round trip, synthetic inputs, calibration, study sharding
and the multi-rank path (gloo, world size 2: shard -> run -> gather, max-over-ranks timing)."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rsna_knee_efficiency_b200 import densenet, infer, pack as packmod, quant, synth
from tests.helpers import plan_tables


def test_pack_round_trip(tmp_path):
    _, plan, par = plan_tables(64)
    head = densenet.random_head(3)
    f = tmp_path / "p.npz"
    packmod.save_pack(f, plan, 24, head)
    p = packmod.load_pack(f)
    assert packmod.is_pack(p)
    m = p["meta"]
    assert (m["format"], m["kind"], m["n"], m["img"], m["n_out"]) == (1, "dense8s", 24, 64, 4)
    assert m["conv2"] == "ours" and m["stem"] == "i8"
    assert [b["L"] for b in m["blocks"]] == [6, 12, 32, 32]
    assert [b["trans"] for b in m["blocks"]] == [True, True, True, False]
    mem = packmod.make_pack(plan, 24, head)
    assert set(p["par"]) == set(mem["par"])
    for k, v in mem["par"].items():
        np.testing.assert_array_equal(p["par"][k], v, err_msg=k)
    assert not any(k.endswith(("_gd", "_c2")) and k.startswith("L") for k in p["par"])
    assert {"H_w", "H_b"} <= set(p["par"])
    assert packmod.f16_layers(m) >= {(0, 0), ("t", 0)}


def test_encoder_rejects_foreign_packs():
    from rsna_knee_efficiency_b200.encoder import Dense8SEncoder
    _, plan, _ = plan_tables(64)
    p = packmod.make_pack(plan, 4)
    bad = dict(p, meta=dict(p["meta"], kind="dense8"))
    with pytest.raises(ValueError):
        Dense8SEncoder(bad, 0, 4)
    trt = dict(p, meta=dict(p["meta"], conv2="trt"))
    with pytest.raises(ValueError, match="TensorRT"):
        Dense8SEncoder(trt, 0, 4)


def test_synthetic_volume_is_seeded():
    a, b = synth.volume(7, S=5, H=64, W=64), synth.volume(7, S=5, H=64, W=64)
    assert a.dtype == np.uint8 and a.shape == (5, 64, 64)
    np.testing.assert_array_equal(a, b)
    assert not np.array_equal(a, synth.volume(8, S=5, H=64, W=64))
    t = synth.triplets(a)
    assert t.shape == (3, 3, 64, 64)
    np.testing.assert_array_equal(t[1], a[1:4])
    v = infer.make_volumes(3, img=32, slices=6, seed=5)
    assert v.shape == (2, 3, 6, 32, 32)
    np.testing.assert_array_equal(v[1, 2], synth.volume(5 + 2 * 2 + 1, S=6, H=32, W=32))


def test_calibrate_percentile_is_exact_order_statistic():
    """pct calibration = the ceil((1 - q) n)-th largest |x| over the union of all batches: per
    tensor for the conv inputs, per channel for the stored segments; checked on captured tensors."""
    torch.manual_seed(0)
    m = densenet.random_init(densenet.DenseNet169(), 5)
    batches = [torch.from_numpy(b) for b in synth.calibration_batches(3, 1, 32, seed=9)]
    q = 0.99
    cal = quant.calibrate(m, batches, method="pct", pct=100 * q)
    cal_max = quant.calibrate(m, batches, method="max")
    layer = m.features.denseblock2.denselayer4
    seen_in, seen_out = [], []
    h1 = layer.conv2.register_forward_pre_hook(lambda _m, i: seen_in.append(i[0].detach().clone()))
    h2 = layer.conv2.register_forward_hook(lambda _m, _i, y: seen_out.append(y.detach().clone()))
    with torch.no_grad():
        for x in batches:
            m(x)
    h1.remove()
    h2.remove()
    a = torch.cat([t.abs().reshape(-1) for t in seen_in]).double().sort(descending=True).values
    k = int(np.ceil((1 - q) * a.numel()))
    assert float(cal["in2.1.3"]) == pytest.approx(float(a[k - 1]), rel=1e-6)
    y = torch.cat([t.abs().transpose(0, 1).reshape(t.shape[1], -1) for t in seen_out], 1).double()
    kc = int(np.ceil((1 - q) * y.shape[1]))
    want = y.sort(1, descending=True).values[:, kc - 1].numpy()
    np.testing.assert_allclose(cal["conv2.1.3"], want, rtol=1e-6)
    np.testing.assert_allclose(cal_max["conv2.1.3"], y.amax(1).numpy(), rtol=1e-6)
    with pytest.raises(ValueError):
        quant.calibrate(m, batches, method="median")


def test_shard_partitions_studies():
    for n in (0, 1, 7, 8, 256, 4096, 255):
        for world in (1, 2, 3, 4, 8):
            spans = [infer.shard(n, world, r) for r in range(world)]
            covered = [i for s, e in spans for i in range(s, e)]
            assert covered == list(range(n))
            sizes = [e - s for s, e in spans]
            assert max(sizes, default=0) - min(sizes, default=0) <= -(-n // world)


class _FakeRunner:
    """CPU stand-in with the StudyRunner contract: logits = per-study statistics of the volumes."""

    def __init__(self, studies):
        self.studies, self.device, self.n_out, self.calls = studies, "cpu", 4, 0

    def run(self, vols):
        self.calls += 1
        v = vols.float()
        return torch.stack([v[0].mean((1, 2, 3)), v[1].mean((1, 2, 3)), v[0].amax((1, 2, 3)),
                            v[1].amin((1, 2, 3))], 1)


def _expected(vols):
    v = torch.as_tensor(vols).float()
    return torch.stack([v[0].mean((1, 2, 3)), v[1].mean((1, 2, 3)), v[0].amax((1, 2, 3)),
                        v[1].amin((1, 2, 3))], 1)


def test_run_shard_pads_last_batch():
    vols = infer.make_volumes(7, img=16, slices=4, seed=3)
    r = _FakeRunner(3)
    out = infer.run_shard(r, vols)
    assert r.calls == 3
    torch.testing.assert_close(out, _expected(vols))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n_studies, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        vols = infer.make_volumes(n_studies, img=16, slices=4, seed=11)
        local = infer.run_shard(_FakeRunner(2), vols, rank, world)
        full = infer.gather_logits(local, n_studies)
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        q.put((rank, local.shape[0], full.numpy(), float(t)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_studies", [5, 8])
def test_two_rank_shard_and_gather_gloo(n_studies):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n_studies, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = _expected(infer.make_volumes(n_studies, img=16, slices=4, seed=11)).numpy()
    assert [r[1] for r in res] == [e - s for s, e in (infer.shard(n_studies, 2, r) for r in range(2))]
    for _, _, full, tmax in res:
        np.testing.assert_allclose(full, want, rtol=1e-6)
        assert tmax == 2.0


def test_bench_work_model_matches_the_per_image_totals():
    """bench.py's per-launch algorithmic work summed over one 512 px image: 128.1 MB of HBM traffic
    (activations, every tensor once) and 17.55 GMAC (transitions in the exact full-res integer form)."""
    import bench
    blocks = [{"c0": 64, "h": 128, "w": 128, "L": 6}, {"c0": 128, "h": 64, "w": 64, "L": 12},
              {"c0": 256, "h": 32, "w": 32, "L": 32}, {"c0": 640, "h": 16, "w": 16, "L": 32}]
    tb = tm = 0
    for b, blk in enumerate(blocks):
        for l in range(blk["L"]):
            by, m = bench.launch_work("conv1", blk, l, 1, 512)
            tb, tm = tb + by - (blk["c0"] + 32 * l) * 128, tm + m
            by, m = bench.launch_work("conv2", blk, l, 1, 512)
            tb, tm = tb + by - 36864, tm + m
        if b < 3:
            by, m = bench.launch_work("trans", blk, 0, 1, 512)
            tb, tm = tb + by, tm + m
    for kind, blk in (("stem", blocks[0]), ("head", blocks[3])):
        by, m = bench.launch_work(kind, blk, 0, 1, 512)
        tb, tm = tb + by, tm + m
    assert abs(tb / 1e6 - 128.12) < 0.01
    assert abs(tm / 1e9 - 17.545) < 0.001


def test_run_shard_with_study_indices():
    """`studies` picks (and may repeat) volumes; shards follow that order."""
    vols = infer.make_volumes(4, img=16, slices=4, seed=21)
    order = [2, 0, 1, 1, 3, 2, 0]
    want = _expected(vols)[order]
    torch.testing.assert_close(infer.run_shard(_FakeRunner(3), vols, studies=order), want)
    a, b = infer.shard(len(order), 2, 1)
    torch.testing.assert_close(infer.run_shard(_FakeRunner(2), vols, rank=1, world=2, studies=order), want[a:b])


def test_member_windows_match_the_reference():
    """Every design, member and seed of tests/golden/member_windows.json (made by the reference's own
    `member_windows`) at the benchmark's 2 x 24 and the submission's 8 x 11 geometry."""
    import json
    from pathlib import Path
    cases = json.loads((Path(__file__).resolve().parent / "golden" / "member_windows.json").read_text())
    assert len(cases) == 192
    for c in cases:
        got = infer.member_windows(c["design"], c["member"], c["n_slots"], c["per"], seed=c["seed"])
        assert got.tolist() == c["windows"], c


def test_parx_seeds_cover_every_window_once():
    """Two seeds of `parx` read complementary halves: every (slot, position) exactly once, and each
    seed alternate positions of every slot."""
    per = 24
    a = infer.member_windows("parx", 0, 2, per, seed=0)
    b = infer.member_windows("parx", 0, 2, per, seed=1)
    assert sorted(a.tolist() + b.tolist()) == list(range(2 * per))
    for idx in (a, b):
        for slot in range(2):
            pos = idx[idx // per == slot] % per
            assert len(pos) == per // 2 and set(np.diff(pos)) == {2}


@pytest.mark.parametrize("flip", [False, True])
def test_plane_table_addresses_the_seed_windows(flip):
    """Image i of seed k reads the three slices of its window from the window-major volume planes."""
    studies, slices = 3, 26
    per = slices - 2
    for seed in (0, 1):
        src, flags, idx = infer.plane_table("parx", seed, studies, slices, 2, flip)
        nf = 2 if flip else 1
        assert src.shape == (studies * nf * len(idx), 4) and flags.shape == (len(src),)
        i = 0
        for st in range(studies):
            for f in range(nf):
                for w in idx:
                    s, p = divmod(int(w), per)
                    assert src[i, :3].tolist() == [(s * studies + st) * slices + p + d for d in range(3)]
                    assert flags[i] == f
                    i += 1


def test_reference_written_pack_loads():
    """tests/golden/ref_pack_64.npz was written by the reference's own save_pack (conv2 "ours",
    stem "i8"): load_pack reads its meta and tables, the fp16 / fp32 prologue choice per layer follows
    the reference's kernel kinds, and every table the engine needs is there with its dtype and size."""
    from pathlib import Path
    pk = packmod.load_pack(Path(__file__).resolve().parent / "golden" / "ref_pack_64.npz")
    meta, par = pk["meta"], pk["par"]
    assert packmod.is_pack(pk) and meta["conv2"] == "ours" and meta["stem"] == "i8" and meta["n"] == 2
    assert packmod.f16_layers(meta) == {(0, li) for li in range(6)} | {("t", 0)}
    for bi, b in enumerate(meta["blocks"]):
        for li in range(b["L"]):
            cin = b["c0"] + 32 * li
            assert par[f"L{bi}_{li}_w1"].shape == (cin // 32, 128, 32) and par[f"L{bi}_{li}_w1"].dtype == np.int8
            assert par[f"L{bi}_{li}_w2k"].shape == (4, 9, 32, 32)
            assert par[f"L{bi}_{li}_abh"].shape == (cin // 2, 4) and par[f"L{bi}_{li}_ab"].shape == (cin, 2)
            assert par[f"L{bi}_{li}_gdu"].dtype == np.float32 and par[f"L{bi}_{li}_c2u"].shape == (32,)
        if b["trans"]:
            ctot = b["c0"] + 32 * b["L"]
            assert par[f"T{bi}_w"].shape == (ctot // 32, ctot // 2, 32)
    assert par["S_w8"].shape == (64, 176) and par["S_kc"].shape == (128,)
    assert par["F_ab"].shape == (meta["n_features"], 2)
