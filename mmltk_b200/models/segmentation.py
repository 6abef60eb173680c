"""Segmentation head (reference `src/rfdetr/layers/modules.cpp:229-397`).

DepthwiseConvBlock: dw3x3 -> LN(eps 1e-6) -> Linear -> GELU (-> gamma) + residual.
MlpBlock: LN -> Linear(d,4d) -> GELU -> Linear(4d,d) (-> gamma) + residual.
Mask logits = einsum("bchw,bnc->bnhw", spatial, queries) + bias on features
bilinearly resized to (H/4, W/4).  Training uses the sparse form (spatial
features, query features, bias) that the loss point-samples.
"""
from __future__ import annotations

from typing import List, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops


class DepthwiseConvBlock(nn.Module):
    def __init__(self, dim: int, layer_scale_init_value: float = 0.0):
        super().__init__()
        self.dwconv = nn.Conv2d(dim, dim, 3, padding=1, groups=dim)
        self.norm = nn.LayerNorm(dim, eps=1e-6)
        self.pwconv1 = nn.Linear(dim, dim)
        self.act = nn.GELU()
        self.gamma = nn.Parameter(torch.full((dim,), layer_scale_init_value)) if layer_scale_init_value > 0 else None

    def forward(self, x):  # x NCHW
        r = x
        x = F.conv2d(x, self.dwconv.weight.to(x.dtype), self.dwconv.bias.to(x.dtype), padding=1, groups=x.shape[1])
        x = x.permute(0, 2, 3, 1)
        x = ops.layer_norm(x, self.norm.weight, self.norm.bias, 1e-6)
        x = ops.linear(x, self.pwconv1.weight, self.pwconv1.bias, act="gelu")
        if self.gamma is not None:
            x = x * self.gamma.to(x.dtype)
        return x.permute(0, 3, 1, 2) + r


class MlpBlock(nn.Module):
    def __init__(self, dim: int, layer_scale_init_value: float = 0.0):
        super().__init__()
        self.norm_in = nn.LayerNorm(dim)
        self.layers = nn.ModuleList([nn.Linear(dim, dim * 4), nn.GELU(), nn.Linear(dim * 4, dim)])
        self.gamma = nn.Parameter(torch.full((dim,), layer_scale_init_value)) if layer_scale_init_value > 0 else None

    def forward(self, x):
        r = x
        x = ops.layer_norm(x, self.norm_in.weight, self.norm_in.bias, 1e-5)
        x = ops.linear(x, self.layers[0].weight, self.layers[0].bias, act="gelu")
        x = ops.linear(x, self.layers[2].weight, self.layers[2].bias)
        if self.gamma is not None:
            x = x * self.gamma.to(x.dtype)
        return x + r


class SegmentationHead(nn.Module):
    def __init__(self, in_dim: int, num_blocks: int, bottleneck_ratio=None, downsample_ratio: int = 4):
        super().__init__()
        self.downsample_ratio = downsample_ratio
        self.blocks = nn.ModuleList(DepthwiseConvBlock(in_dim) for _ in range(num_blocks))
        self.query_features_block = MlpBlock(in_dim)
        self.bias = nn.Parameter(torch.zeros(1))
        if bottleneck_ratio is not None:
            inter = in_dim // bottleneck_ratio
            self.spatial_features_proj = nn.Conv2d(in_dim, inter, 1)
            self.query_features_proj = nn.Linear(in_dim, inter)
        else:
            self.spatial_features_proj = None
            self.query_features_proj = None

    def _spatial(self, x):
        if self.spatial_features_proj is None:
            return x
        return F.conv2d(x, self.spatial_features_proj.weight.to(x.dtype), self.spatial_features_proj.bias.to(x.dtype))

    def _query(self, q):
        q = self.query_features_block(q)
        if self.query_features_proj is None:
            return q
        return ops.linear(q, self.query_features_proj.weight, self.query_features_proj.bias)

    def _resize(self, feats_nchw, image_size: Tuple[int, int]):
        h, w = image_size[0] // self.downsample_ratio, image_size[1] // self.downsample_ratio
        return F.interpolate(feats_nchw, size=(h, w), mode="bilinear", align_corners=False)

    def sparse_forward(self, spatial_nchw, queries: List[torch.Tensor], image_size, skip_blocks=False):
        """-> list of (spatial [B,C,h,w], query [B,N,C], bias [1]) per decoder layer."""
        x = self._resize(spatial_nchw, image_size)
        out = []
        if skip_blocks:
            return [(x, self._query(queries[0]), self.bias)]
        if len(queries) != len(self.blocks):
            raise ValueError("SegmentationHead query_features size must match block count")
        for blk, q in zip(self.blocks, queries):
            x = blk(x)
            out.append((self._spatial(x), self._query(q), self.bias))
        return out

    def forward(self, spatial_nchw, queries: List[torch.Tensor], image_size, skip_blocks=False):
        return [torch.einsum("bchw,bnc->bnhw", s, q) + b.to(s.dtype)
                for s, q, b in self.sparse_forward(spatial_nchw, queries, image_size, skip_blocks)]
