"""Multi-scale projector: concatenated ViT taps -> C2f -> LayerNorm2d per level.

Reference (`src/rfdetr/layers/model.cpp:267-369,705-726`): single P4 level,
``C2f(4*384 -> 256, 3 bottlenecks, LayerNorm2d, SiLU)`` then ``LayerNorm2d``.
ConvX = Conv(no bias) -> LayerNorm2d (eps 1e-6) -> SiLU; Bottleneck = two 3x3
ConvX without a shortcut.

The level list is configuration here: "P3" upsamples the taps x2 with a
transposed conv before its C2f, "P5" downsamples /2 with a strided 3x3 ConvX,
"P4" uses the taps as they are.  Features are channels-last [B, h, w, C]
throughout (LayerNorm2d is then a plain last-dim LayerNorm and 1x1 convs are
GEMMs); 3x3 convs run as cuDNN channels-last convolutions.
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

    def forward_nhwc(self, x: torch.Tensor) -> torch.Tensor:
        return ops.layer_norm(x, self.weight, self.bias, self.eps)


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
        else:
            xc = x.permute(0, 3, 1, 2)
            y = F.conv2d(xc, self.conv.weight.to(xc.dtype), None, self.s, self.k // 2).permute(0, 2, 3, 1)
        y = self.bn.forward_nhwc(y)
        return F.silu(y)


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


class Upsample2x(nn.Module):
    def __init__(self, c: int):
        super().__init__()
        self.conv = nn.ConvTranspose2d(c, c // 2, kernel_size=2, stride=2)
        self.bn = LayerNorm2d(c // 2)

    def forward_nhwc(self, x):
        y = F.conv_transpose2d(x.permute(0, 3, 1, 2), self.conv.weight.to(x.dtype), self.conv.bias.to(x.dtype),
                               stride=2).permute(0, 2, 3, 1)
        return F.gelu(self.bn.forward_nhwc(y))


class MultiScaleProjector(nn.Module):
    def __init__(self, in_channels: int, num_taps: int, out_channels: int, levels, blocks: int = 3):
        super().__init__()
        self.levels = tuple(levels)
        cin = in_channels * num_taps
        self.stages_sampling = nn.ModuleList()
        self.stages = nn.ModuleList()
        self.needs_sampling = any(l != "P4" for l in self.levels)
        for lvl in self.levels:
            if lvl == "P4":
                samp, c = nn.Identity(), cin
            elif lvl == "P3":
                samp, c = Upsample2x(cin), cin // 2
            elif lvl == "P5":
                samp, c = ConvX(cin, cin, 3, 2), cin
            else:  # P6
                samp, c = nn.Sequential(ConvX(cin, cin, 3, 2), ConvX(cin, cin, 3, 2)), cin
            self.stages_sampling.append(samp)
            self.stages.append(ProjectorStage(C2f(c, out_channels, blocks), LayerNorm2d(out_channels)))
        if not self.needs_sampling:
            # keep the reference's state-dict layout (`projector.stages.0.*` only)
            del self.stages_sampling

    def forward(self, taps: List[torch.Tensor]) -> List[torch.Tensor]:
        x = torch.cat(taps, -1)
        outs = []
        for i, lvl in enumerate(self.levels):
            h = x
            if self.needs_sampling:
                samp = self.stages_sampling[i]
                if isinstance(samp, nn.Sequential):
                    for m in samp:
                        h = m.forward_nhwc(h)
                elif not isinstance(samp, nn.Identity):
                    h = samp.forward_nhwc(h)
            outs.append(self.stages[i].forward_nhwc(h))
        return outs
