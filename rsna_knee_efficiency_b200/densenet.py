"""DenseNet169 in fp32 PyTorch: the floating-point network the INT8 encoder quantises.

The module tree and state_dict names are those of torchvision/timm `densenet169` (the reference
restates the same network in `src/knee/models/densenet.py:27-104`): `features.conv0`,
`features.norm0`, `features.denseblock{b}.denselayer{l}.{norm1,conv1,norm2,conv2}`,
`features.transition{b}.{norm,conv}`, `features.norm5`. Keeping the names identical lets a
checkpoint trained with either load here, and lets `calibrate` / `make_plan` walk the same tree the
reference's do. `forward` returns the (N, 1664) global features: norm5, ReLU, spatial mean.

This file is also the fp32 CPU baseline of the benchmark (the reference's fp32 path) and the
reference for the "logits within 5e-2 of fp32" check.
"""
from __future__ import annotations

from collections import OrderedDict

import torch
import torch.nn as nn
import torch.nn.functional as F

GROWTH = 32
BOTTLENECK = 128                 # 4 * growth: conv1 output channels of every dense layer
STEM_C = 64
BLOCKS_169 = (6, 12, 32, 32)


class DenseLayer(nn.Module):
    """BN-ReLU-1x1 (c_in -> 128) then BN-ReLU-3x3 (128 -> 32); input is the list of earlier maps."""

    def __init__(self, c_in: int) -> None:
        super().__init__()
        self.norm1 = nn.BatchNorm2d(c_in)
        self.relu1 = nn.ReLU(inplace=True)
        self.conv1 = nn.Conv2d(c_in, BOTTLENECK, 1, bias=False)
        self.norm2 = nn.BatchNorm2d(BOTTLENECK)
        self.relu2 = nn.ReLU(inplace=True)
        self.conv2 = nn.Conv2d(BOTTLENECK, GROWTH, 3, padding=1, bias=False)

    def forward(self, feats: list[torch.Tensor]) -> torch.Tensor:
        h = self.conv1(self.relu1(self.norm1(torch.cat(feats, 1))))
        return self.conv2(self.relu2(self.norm2(h)))


class DenseBlock(nn.ModuleDict):
    def __init__(self, n_layers: int, c0: int) -> None:
        super().__init__()
        for i in range(n_layers):
            self.add_module(f"denselayer{i + 1}", DenseLayer(c0 + GROWTH * i))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        feats = [x]
        for layer in self.values():
            feats.append(layer(feats))
        return torch.cat(feats, 1)


class Transition(nn.Sequential):
    def __init__(self, c_in: int, c_out: int) -> None:
        super().__init__(OrderedDict(norm=nn.BatchNorm2d(c_in), relu=nn.ReLU(inplace=True),
                                     conv=nn.Conv2d(c_in, c_out, 1, bias=False),
                                     pool=nn.AvgPool2d(2, 2)))


class DenseNet169(nn.Module):
    """`forward(x)`: x (N, in_chans, H, W) float -> (N, 1664) features."""

    def __init__(self, in_chans: int = 3, blocks: tuple[int, ...] = BLOCKS_169) -> None:
        super().__init__()
        self.features = nn.Sequential(OrderedDict(
            conv0=nn.Conv2d(in_chans, STEM_C, 7, stride=2, padding=3, bias=False),
            norm0=nn.BatchNorm2d(STEM_C), relu0=nn.ReLU(inplace=True),
            pool0=nn.MaxPool2d(3, stride=2, padding=1)))
        c = STEM_C
        for b, n_layers in enumerate(blocks):
            self.features.add_module(f"denseblock{b + 1}", DenseBlock(n_layers, c))
            c += GROWTH * n_layers
            if b + 1 < len(blocks):
                self.features.add_module(f"transition{b + 1}", Transition(c, c // 2))
                c //= 2
        self.features.add_module("norm5", nn.BatchNorm2d(c))
        self.num_features = c

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        f = F.relu(self.features(x))
        return f.mean(dim=(2, 3))


@torch.no_grad()
def random_init(model: nn.Module, seed: int) -> nn.Module:
    """Seeded random weights for the synthetic benchmark: Kaiming-normal convolutions; every
    BatchNorm with weight ~ N(1, 0.1), bias ~ N(0, 0.1), running_mean ~ N(0, 0.1),
    running_var ~ U(0.5, 1.5). Returns the model in eval mode.
    """
    g = torch.Generator().manual_seed(seed)
    for m in model.modules():
        if isinstance(m, nn.Conv2d):
            fan_in = m.weight[0].numel()
            m.weight.copy_(torch.randn(m.weight.shape, generator=g) * (2.0 / fan_in) ** 0.5)
        elif isinstance(m, nn.BatchNorm2d):
            n = m.num_features
            m.weight.copy_(1.0 + 0.1 * torch.randn(n, generator=g))
            m.bias.copy_(0.1 * torch.randn(n, generator=g))
            m.running_mean.copy_(0.1 * torch.randn(n, generator=g))
            m.running_var.copy_(0.5 + torch.rand(n, generator=g))
    return model.eval()


class LinearHead(nn.Module):
    """The benchmark head: linear 1664 -> 4 per image, then the mean over the slices of a view."""

    def __init__(self, c: int = 1664, n_out: int = 4) -> None:
        super().__init__()
        self.fc = nn.Linear(c, n_out)

    def forward(self, feats: torch.Tensor, per_view: int) -> torch.Tensor:
        z = self.fc(feats)
        return z.view(-1, per_view, z.shape[-1]).mean(1)


@torch.no_grad()
def random_head(seed: int, c: int = 1664, n_out: int = 4, std: float = 0.02) -> LinearHead:
    g = torch.Generator().manual_seed(seed)
    h = LinearHead(c, n_out)
    h.fc.weight.copy_(std * torch.randn(n_out, c, generator=g))
    h.fc.bias.copy_(0.01 * torch.randn(n_out, generator=g))
    return h.eval()
