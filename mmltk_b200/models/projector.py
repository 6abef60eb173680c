"""Multi-scale projector: concatenated ViT taps -> C2f -> LayerNorm2d per level.

Reference (`src/rfdetr/layers/model.cpp:267-369,705-726`): single P4 level,
``C2f(4*384 -> 256, 3 bottlenecks, LayerNorm2d, SiLU)`` then ``LayerNorm2d``.
ConvX = Conv(no bias) -> LayerNorm2d (eps 1e-6) -> SiLU; Bottleneck = two 3x3
ConvX without a shortcut.

The level list is configuration here, laid out like upstream RF-DETR's
multi-scale projector: every level resamples EACH backbone tap on its own
(``stages_sampling[level][tap]``) and concatenates the results into that
level's C2f.  "P3" (scale 2) is one 2x2 stride-2 transposed conv per tap
(C -> C/2; the C2f then sees taps * C/2 channels), "P5" (scale 1/2) one
stride-2 3x3 ConvX per tap (C -> C), "P4" (scale 1) the tap unchanged (an
empty ``Sequential``, so a P4-only model has the reference's state-dict
layout), "P6" (scale 1/4) a stride-2 max-pool of the previous level's output.
Features are channels-last [B, h, w, C] throughout (LayerNorm2d is then a
plain last-dim LayerNorm, 1x1 convs and the 2x2/stride-2 transposed convs are
GEMMs); 3x3 convs are cuDNN channels-last convolutions, or with ``MMLTK_TC_CONV=1`` the stride-1
ones implicit GEMMs on the tcgen05 kernel (``ops.conv3x3``).
"""
from __future__ import annotations

from typing import List

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops


class LayerNorm2d(nn.Module):
    def __init__(self, channels: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(channels))
        self.bias = nn.Parameter(torch.zeros(channels))
        self.eps = eps

    def forward_nhwc(self, x: torch.Tensor, act: str = None) -> torch.Tensor:
        return ops.layer_norm(x, self.weight, self.bias, self.eps, act=act)


class ConvX(nn.Module):
    def __init__(self, cin: int, cout: int, k: int = 3, s: int = 1):
        super().__init__()
        self.k, self.s = k, s
        self.conv = nn.Conv2d(cin, cout, k, stride=s, padding=k // 2, bias=False)
        self.bn = LayerNorm2d(cout)

    def forward_nhwc(self, x: torch.Tensor) -> torch.Tensor:
        if self.k == 1 and self.s == 1:
            w = self.conv.weight.view(self.conv.weight.shape[0], -1)
            y = ops.linear(x, w)
        elif self.k == 3 and self.s == 1:
            y = ops.conv3x3(x, self.conv.weight)      # cuDNN, or the tcgen05 implicit GEMM (opt-in)
        else:
            xc = x.permute(0, 3, 1, 2)
            y = F.conv2d(xc, self.conv.weight.to(xc.dtype), None, self.s, self.k // 2).permute(0, 2, 3, 1)
        return self.bn.forward_nhwc(y, act="silu")      # norm + SiLU in one kernel on the GPU


class Bottleneck(nn.Module):
    def __init__(self, c1: int, c2: int):
        super().__init__()
        self.cv1 = ConvX(c1, c2, 3)
        self.cv2 = ConvX(c2, c2, 3)

    def forward_nhwc(self, x):
        return self.cv2.forward_nhwc(self.cv1.forward_nhwc(x))


class C2f(nn.Module):
    def __init__(self, c1: int, c2: int, n: int):
        super().__init__()
        self.c = c2 // 2
        self.cv1 = ConvX(c1, 2 * self.c, 1)
        self.cv2 = ConvX((2 + n) * self.c, c2, 1)
        self.m = nn.ModuleList(Bottleneck(self.c, self.c) for _ in range(n))

    def forward_nhwc(self, x):
        y = self.cv1.forward_nhwc(x)
        parts = [y[..., :self.c], y[..., self.c:]]
        for blk in self.m:
            parts.append(blk.forward_nhwc(parts[-1]))
        return self.cv2.forward_nhwc(torch.cat(parts, -1))


class ProjectorStage(nn.Sequential):
    """`projector.stages.<i>` = Sequential(C2f, LayerNorm2d)."""

    def forward_nhwc(self, x):
        return self[1].forward_nhwc(self[0].forward_nhwc(x))


class TransposedConv2x(nn.ConvTranspose2d):
    """2x2, stride-2 transposed conv on channels-last features.  Each input pixel writes its own
    2x2 output patch, so it is one GEMM ``[B*h*w, C] x [C, 4*C']`` plus a pixel shuffle."""

    def __init__(self, cin: int, cout: int):
        super().__init__(cin, cout, kernel_size=2, stride=2)

    def forward_nhwc(self, x: torch.Tensor) -> torch.Tensor:
        B, h, w, C = x.shape
        co = self.out_channels
        wm = self.weight.to(x.dtype).permute(2, 3, 1, 0).reshape(4 * co, C)     # rows (dy, dx, co)
        bias = self.bias.to(x.dtype).repeat(4)
        y = ops.linear(x, wm, bias)                                               # [B, h, w, 4*co]
        return y.view(B, h, w, 2, 2, co).permute(0, 1, 3, 2, 4, 5).reshape(B, 2 * h, 2 * w, co)


def _sampling_layer(level: str, c: int) -> nn.Sequential:
    if level == "P3":
        return nn.Sequential(TransposedConv2x(c, c // 2))
    if level == "P5":
        return nn.Sequential(ConvX(c, c, 3, 2))
    return nn.Sequential()      # P4: identity


def _level_channels(level: str, c: int) -> int:
    return c // 2 if level == "P3" else c


class MultiScaleProjector(nn.Module):
    def __init__(self, in_channels: int, num_taps: int, out_channels: int, levels, blocks: int = 3):
        super().__init__()
        self.levels = tuple(levels)
        self.extra_pool = self.levels[-1] == "P6"
        conv_levels = self.levels[:-1] if self.extra_pool else self.levels
        if not conv_levels:
            raise ValueError("the projector needs at least one of P3 / P4 / P5 before P6")
        self.stages_sampling = nn.ModuleList(
            nn.ModuleList(_sampling_layer(lvl, in_channels) for _ in range(num_taps)) for lvl in conv_levels)
        self.stages = nn.ModuleList(
            ProjectorStage(C2f(num_taps * _level_channels(lvl, in_channels), out_channels, blocks),
                           LayerNorm2d(out_channels)) for lvl in conv_levels)

    def forward(self, taps: List[torch.Tensor]) -> List[torch.Tensor]:
        outs = []
        for stage, sampling in zip(self.stages, self.stages_sampling):
            fused = []
            for tap, samp in zip(taps, sampling):
                h = tap
                for m in samp:
                    h = m.forward_nhwc(h)
                fused.append(h)
            x = ops.concat_channels(fused)     # no copy when the taps already sit side by side
            outs.append(stage.forward_nhwc(x))
        if self.extra_pool:
            outs.append(outs[-1][:, ::2, ::2, :])      # max-pool with kernel 1, stride 2
        return outs
