"""Failure detection on the GPU without a GPU fault: a bounded device-side wait is made to run out on
purpose (dn8_test_inject_wait_fault: the store producer of the first CTA announces raw stage 0 of its
first tile but never copies it, under a short wait limit of 2^24 SM cycles, ~9 ms). The launch must
report the timeout through its error word -- and an engine through dn8_engine_check / `check()` as
DN8_EDEVICE -- every role must leave its loop and free its tensor memory, and the context must stay
usable: the next launch on the same buffers gives the oracle's bytes. Covered for conv1 on single CTAs
and on CTA pairs (cta_group::2, where the other CTA of the pair times out on its own)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from rsna_knee_efficiency_b200 import _native as nat
from rsna_knee_efficiency_b200 import ops, pack as packmod, synth
from rsna_knee_efficiency_b200.encoder import Dense8SEncoder
from tests.helpers import dev, planes_to_pixels, plan_tables, rand_store, tile_major

pytestmark = pytest.mark.gpu

LIMIT = 1 << 24                     # SM cycles: ~9 ms at 1.9 GHz, far above any legitimate wait here


@pytest.mark.parametrize("bi,li", [(1, 7), (3, 31)])          # G = 11 on single CTAs; G = 51 on CTA pairs
def test_conv1_wait_runs_out_and_the_context_stays_usable(bi, li):
    _, plan, par = plan_tables(512)
    b = plan.blocks[bi]
    N, HW = 2, b.h * b.w
    cin = b.c0 + 32 * li
    G, rows = cin // 32, N * HW
    X = rand_store(np.random.default_rng(5 * bi + li), (N, HW, cin), "relu")
    store = dev(tile_major(X))
    w = dev(ops.prepare_conv1_weights(par[f"L{bi}_{li}_w1"]))
    ab, gd = dev(par[f"L{bi}_{li}_abh"]), dev(par[f"L{bi}_{li}_gdu"])
    out = torch.zeros(rows * 128, dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert nat.lib().dn8_test_inject_wait_fault(1, LIMIT) == nat.DN8_OK
    ops.conv1(store, None, w, ab, gd, out, 0, G, N, HW, True, err=err, tile_groups=G)
    torch.cuda.synchronize()                                  # the kernel returned
    code = int(err.item())
    assert code & 0xF in (1, 2, 3) and code >> 4 > 0, f"expected a wait-timeout code with its site, got {code}"
    # the same launch again, unarmed: the oracle's bytes
    err.zero_()
    out.zero_()
    ops.conv1(store, None, w, ab, gd, out, 0, G, N, HW, True, err=err, tile_groups=G)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    want = orc.conv1(X.reshape(rows, cin), par[f"L{bi}_{li}_w1"], abh=par[f"L{bi}_{li}_abh"],
                     gd=par[f"L{bi}_{li}_gdu"], mode=orc.KERNEL)
    np.testing.assert_array_equal(planes_to_pixels(out, rows), want)


def test_engine_reports_the_timeout_then_runs_clean():
    _, plan, par = plan_tables(64)
    n = 2
    x = synth.triplets(synth.volume(21, H=64, W=64))[:n]
    enc = Dense8SEncoder(packmod.make_pack(plan, n), 0, n)
    xh = torch.from_numpy((x.astype(np.float32) / 255.0).astype(np.float16)).cuda()
    enc(xh)
    enc.check()
    assert nat.lib().dn8_test_inject_wait_fault(1, LIMIT) == nat.DN8_OK
    enc(xh)                                                   # block 1 layer 1's conv1 gives up
    with pytest.raises(nat.Dn8Error, match="bounded wait"):
        enc.check()
    got = enc(xh).cpu().numpy()                               # the next pass on the same engine
    enc.check()
    np.testing.assert_array_equal(got, orc.forward(par, packmod.pack_meta(plan, n), x, mode=orc.KERNEL))
    enc.close()


def test_hook_rejects_bad_arguments():
    lib = nat.lib()
    assert lib.dn8_test_inject_wait_fault(2, LIMIT) == nat.DN8_EINVAL
    assert lib.dn8_test_inject_wait_fault(1, 0) == nat.DN8_EINVAL
    assert lib.dn8_test_inject_wait_fault(0, 0) == nat.DN8_OK              # disarmed
