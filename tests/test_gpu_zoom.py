"""The geometric test-time view on the GPU (`dn8_zoom`): the zoomed / shifted fp16 windows against
the reference's own operators for this view -- torch's `affine_grid` + `grid_sample` in fp16 on
the windows gathered through the reference's uint8 -> fp16 LUT (`affine_windows`,
src/knee/tta.py:131-149; LUT src/knee/data/fused_uint8.py:735) -- and the study path with the
submission's view (zoom 1.10) against the oracle fed with those windows."""
from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import oracle as orc
from rsna_knee_efficiency_b200 import densenet, infer, ops, pack as packmod, quant, synth

pytestmark = pytest.mark.gpu


def _torch_view(planes: torch.Tensor, src, flip, scale, tx, ty):
    """fp16 windows (N, 3, H, W) by the reference's operators: LUT gather, optional mirror, then
    affine_grid + grid_sample (bilinear, zeros, align_corners=False) in fp16."""
    lut = torch.arange(256, dtype=torch.uint8, device=planes.device).half().mul_(1.0 / 255.0)
    x = lut[planes[src[:, :3].long()].long()]                                    # (N, 3, H, W)
    if flip is not None:
        m = flip.bool()
        x[m] = torch.flip(x[m], dims=[-1])
    n, c, h, w = x.shape
    theta = torch.tensor([[1.0 / scale, 0.0, -2.0 * tx], [0.0, 1.0 / scale, -2.0 * ty]],
                         device=x.device, dtype=x.dtype).unsqueeze(0)
    grid = F.affine_grid(theta, (1, c, h, w), align_corners=False).expand(n, h, w, 2)
    return F.grid_sample(x, grid, mode="bilinear", padding_mode="zeros", align_corners=False)


@pytest.mark.parametrize("img,scale,tx,ty,flip", [(512, 1.10, 0.0, 0.0, False), (512, 0.95, 0.0, 0.0, True),
                                                  (512, 1.05, 0.03, -0.03, False), (64, 1.10, 0.0, 0.0, True),
                                                  (96, 0.95, -0.03, 0.03, True)])
def test_zoom_matches_reference_operators(img, scale, tx, ty, flip):
    vol = torch.from_numpy(synth.volume(21, S=8, H=img, W=img)).cuda()
    n = 5
    src = torch.tensor([[i, i + 1, i + 2, 0] for i in range(n)], dtype=torch.int32, device="cuda")
    flags = torch.tensor([i & 1 for i in range(n)], dtype=torch.int32, device="cuda") if flip else None
    out = torch.full((n, 3, img, img), float("nan"), dtype=torch.float16, device="cuda")
    ops.zoom(vol, src, out, n, img, img, scale, tx, ty, flags=flags)
    want = _torch_view(vol, src, flags, scale, tx, ty)
    torch.cuda.synchronize()
    got16, want16 = out.view(torch.int16), want.contiguous().view(torch.int16)
    diff = (got16.int() - want16.int()).abs()                # fp16 ulps (values are >= 0)
    assert int(diff.max()) == 0, (int(diff.max()), float((diff > 0).float().mean()))


def test_study_zoom_view_matches_oracle():
    img, studies, slices = 64, 2, 26
    packs, plans = [], []
    for seed in (42, 43):
        torch.manual_seed(0)
        m = densenet.random_init(densenet.DenseNet169(), seed)
        cal = quant.calibrate(m, [torch.from_numpy(b) for b in synth.calibration_batches(2, 2, img, seed=1000 + seed)])
        plan = quant.make_plan(m, cal, img)
        plans.append((plan, densenet.random_head(seed)))
        packs.append(packmod.make_pack(plan, studies * (slices - 2), plans[-1][1]))
    runner = infer.StudyRunner(packs, 0, studies, slices, zoom=(1.10, 0.0, 0.0))
    vols = infer.make_volumes(studies, img=img, slices=slices, seed=55)
    vd = torch.from_numpy(vols).cuda()
    got = runner.run(vd).cpu().numpy()
    for e in runner.encoders:
        e.check()
    want = np.zeros((studies, 4))
    planes = vd.reshape(-1, img, img)
    for k, (plan, head) in enumerate(plans):
        x = _torch_view(planes, runner.src[k], None, 1.10, 0.0, 0.0).cpu().numpy()
        f = orc.forward(quant.kernel_params(plan), packmod.pack_meta(plan, len(x)), x, mode=orc.KERNEL)
        np.testing.assert_array_equal(runner.encoders[k].out[:len(x)].cpu().numpy(), f)
        hw, hb = head.fc.weight.detach().double().numpy(), head.fc.bias.detach().double().numpy()
        want += (f.astype(np.float64) @ hw.T + hb).reshape(studies, -1, 4).mean(1) / 2
    np.testing.assert_allclose(got, want, atol=1e-5)
