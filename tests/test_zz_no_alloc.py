"""dn8_head_noalloc: the pooling + head entry point whose per-view counters live in the library's
built-in scratch (no ticket array from the caller). Checked against dn8_head with an explicit
ticket array, for two calls in a row (the scratch must come back to zero after each call), and
its size limit (rejected before any CUDA call). Collected last on purpose: it must pass both alone
and after every other test of the suite."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from rsna_knee_efficiency_b200 import _native as nat
from rsna_knee_efficiency_b200 import densenet, ops
from tests.helpers import dev, plan_tables, rand_store, split_store


def test_noalloc_rejects_more_views_than_the_scratch_holds():
    """N / per_view above DN8_HEAD_SCRATCH_VIEWS is refused with EINVAL before any CUDA call (the
    pointers here are never dereferenced)."""
    lib = nat.lib()
    fake = 1 << 20                                            # 16-byte aligned, never used
    n = 2 * (nat.DN8_HEAD_SCRATCH_VIEWS + 1)
    a = nat.HeadArgs(fake, fake, fake, None, None, None, fake, fake, None,
                     20, 52, n, 256, 4, 2, 0)
    assert lib.dn8_head_noalloc(ctypes.byref(a), None) == nat.DN8_EINVAL
    assert b"scratch holds" in lib.dn8_last_error()
    a.tickets = fake                                          # a caller ticket array is refused too
    a.N = 8
    assert lib.dn8_head_noalloc(ctypes.byref(a), None) == nat.DN8_EINVAL


@pytest.mark.gpu
def test_noalloc_matches_head_on_two_calls_in_a_row():
    _, plan, par = plan_tables(512)
    b = plan.blocks[3]
    N, HW, per_view = 6, 256, 3
    rng = np.random.default_rng(2024)
    X = rand_store(rng, (N, HW, b.c_tot), "relu")
    in0, seg = split_store(X, b.c0)
    head = densenet.random_head(11)
    hw = dev(head.fc.weight.detach().numpy().astype(np.float32))
    hb = dev(head.fc.bias.detach().numpy().astype(np.float32))
    in0d, segd, fab = dev(in0), dev(seg), dev(par["F_ab"])
    G0, G = b.c0 // 32, b.c_tot // 32

    def buffers():
        return (torch.zeros((N, b.c_tot), dtype=torch.float32, device="cuda"),
                torch.zeros((N, 4), dtype=torch.float32, device="cuda"),
                torch.zeros((N // per_view, 4), dtype=torch.float32, device="cuda"))

    feat0, log0, view0 = buffers()
    tickets = torch.zeros(N // per_view, dtype=torch.int32, device="cuda")
    ops.head(in0d, segd, fab, G0, G, N, HW, feat=feat0, hw=hw, hb=hb, logits=log0, view_logits=view0,
             tickets=tickets, per_view=per_view)
    torch.cuda.synchronize()
    for _ in range(2):
        feat, log, view = buffers()
        ops.head_noalloc(in0d, segd, fab, G0, G, N, HW, feat=feat, hw=hw, hb=hb, logits=log,
                         view_logits=view, per_view=per_view)
        torch.cuda.synchronize()
        assert torch.equal(feat, feat0)
        assert torch.equal(log, log0)
        assert torch.equal(view, view0)
    assert int(tickets.abs().sum().item()) == 0
