"""Windowed DINOv2 ViT backbone.

Behaviour follows the reference's `WindowedDinov2*` modules
(`src/rfdetr/layers/model.cpp:371-703`):

* patch embedding Conv2d(3->C, k=p, s=p) -> tokens [B, N, C]; cls token +
  learned position embedding (bicubic-antialias resize when the grid differs,
  `model.cpp:391-429`);
* windows: the token grid is cut into ``num_windows**2`` windows and the cls
  token is replicated into each window (`model.cpp:431-463`);
* pre-LN layers (eps 1e-6), q/k/v projections, SDPA with scale 1/sqrt(d),
  LayerScale + residual, MLP with exact-erf GELU; layers whose index is a
  tapped stage (except the last) attend across all windows of an image
  (`model.cpp:573-615`);
* taps at ``out_feature_indexes`` -> final LayerNorm -> drop cls -> un-window
  -> [B, C, H/p, W/p] (`model.cpp:653-680`).

B200 layout: tokens stay [B*W^2, 1+n, C] for the whole backbone; a
full-attention layer is a *view* [B, W^2*(1+n), C] of the same memory, so no
layer moves data to switch between windowed and global attention.  q/k/v are
one fused [3C, C] projection (one GEMM); the checkpoint still sees the
separate ``query``/``key``/``value`` tensors through state-dict hooks.
"""
from __future__ import annotations

import re

import math
import os
from typing import List

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops
from ..config import RfDetrConfig

# MMLTK_INFER_FUSED_RESIDUAL=0: inference runs the per-layer autograd-path ops (A/B timing)
_FUSED_RESIDUAL_INFERENCE = os.environ.get("MMLTK_INFER_FUSED_RESIDUAL", "1") != "0"


class PatchEmbeddings(nn.Module):
    def __init__(self, width: int, patch: int):
        super().__init__()
        self.patch = patch
        self.projection = nn.Conv2d(3, width, kernel_size=patch, stride=patch, bias=True)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        # patch conv == GEMM over unfolded non-overlapping patches
        B, C, H, W = x.shape
        p = self.patch
        if x.is_cuda:
            k = ops.kernels()
            if (p % 8 == 0 and W % 8 == 0 and not x.requires_grad and x.dtype in (torch.bfloat16, torch.float32)
                    and hasattr(k, "patch_unfold")):
                cols = k.patch_unfold(x.contiguous(), p)     # one pass, 16-byte runs (the pixels need no gradient)
            else:
                cols = x.view(B, C, H // p, p, W // p, p).permute(0, 2, 4, 1, 3, 5).reshape(
                    B * (H // p) * (W // p), C * p * p)
            w = self.projection.weight.reshape(self.projection.weight.shape[0], -1)
            return ops.linear(cols.to(w.dtype), w, self.projection.bias).view(B, (H // p) * (W // p), -1)
        return self.projection(x.to(self.projection.weight.dtype)).flatten(2).transpose(1, 2)


class Embeddings(nn.Module):
    def __init__(self, cfg: RfDetrConfig):
        super().__init__()
        C = cfg.vit_width
        self.width = C
        self.patch = cfg.patch_size
        self.num_windows = max(1, cfg.num_windows)
        self.cls_token = nn.Parameter(torch.randn(1, 1, C))
        self.mask_token = nn.Parameter(torch.zeros(1, C))
        self.position_embeddings = nn.Parameter(torch.randn(1, cfg.positional_encoding_size ** 2 + 1, C))
        self.patch_embeddings = PatchEmbeddings(C, cfg.patch_size)
        self._pos_cache = {}

    def interpolate_pos_encoding(self, n_patches: int, h: int, w: int) -> torch.Tensor:
        pos = self.position_embeddings
        n_pos = pos.shape[1] - 1
        if n_patches == n_pos and h == w:
            return pos
        cls_pos = pos[:, :1]
        patch_pos = pos[:, 1:]
        side = int(round(math.sqrt(n_pos)))
        ph, pw = h // self.patch, w // self.patch
        pp = patch_pos.reshape(1, side, side, -1).permute(0, 3, 1, 2).float()
        pp = F.interpolate(pp, size=(ph, pw), mode="bicubic", align_corners=False, antialias=True)
        pp = pp.to(pos.dtype).permute(0, 2, 3, 1).reshape(1, -1, pos.shape[-1])
        return torch.cat([cls_pos, pp], 1)

    def forward(self, pixels: torch.Tensor) -> torch.Tensor:
        B, _, H, W = pixels.shape
        tokens = self.patch_embeddings(pixels)  # [B, N, C]
        C = tokens.shape[-1]
        pos = self.interpolate_pos_encoding(tokens.shape[1], H, W).to(tokens.dtype)
        cls = (self.cls_token.to(tokens.dtype) + pos[:, :1]).expand(B, 1, C)
        tokens = tokens + pos[:, 1:]
        nw = self.num_windows
        if nw > 1:
            hp, wp = H // self.patch, W // self.patch
            hpw, wpw = hp // nw, wp // nw
            tokens = (tokens.view(B, nw, hpw, nw, wpw, C).permute(0, 1, 3, 2, 4, 5)
                      .reshape(B * nw * nw, hpw * wpw, C))
            cls = cls.repeat(nw * nw, 1, 1)
        return torch.cat([cls, tokens], 1)


def _qkv_state_hooks(module: nn.Module, width: int):
    """Expose the fused qkv projection as separate query/key/value tensors in state dicts."""

    def save_hook(mod, state, prefix, local_metadata):
        w = state.pop(prefix + "qkv_weight")
        b = state.pop(prefix + "qkv_bias")
        for i, name in enumerate(("query", "key", "value")):
            state[prefix + f"{name}.weight"] = w[i * width:(i + 1) * width]
            state[prefix + f"{name}.bias"] = b[i * width:(i + 1) * width]

    def load_pre_hook(state, prefix, local_metadata, strict, missing, unexpected, errors):
        names = [prefix + f"{n}.{t}" for n in ("query", "key", "value") for t in ("weight", "bias")]
        if all(n in state for n in names):
            state[prefix + "qkv_weight"] = torch.cat([state.pop(prefix + f"{n}.weight")
                                                      for n in ("query", "key", "value")], 0)
            state[prefix + "qkv_bias"] = torch.cat([state.pop(prefix + f"{n}.bias")
                                                    for n in ("query", "key", "value")], 0)

    module._register_state_dict_hook(save_hook)
    module._register_load_state_dict_pre_hook(load_pre_hook, with_module=False)


class SelfAttention(nn.Module):
    """`attention.attention` in the checkpoint: query/key/value Linear(C, C)."""

    def __init__(self, width: int, heads: int):
        super().__init__()
        self.width, self.heads = width, heads
        q = nn.Linear(width, width)
        k = nn.Linear(width, width)
        v = nn.Linear(width, width)
        self.qkv_weight = nn.Parameter(torch.cat([q.weight.data, k.weight.data, v.weight.data], 0))
        self.qkv_bias = nn.Parameter(torch.cat([q.bias.data, k.bias.data, v.bias.data], 0))
        _qkv_state_hooks(self, width)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        N, L, C = x.shape
        H = self.heads
        qkv = ops.linear(x, self.qkv_weight, self.qkv_bias)  # [N, L, 3C]
        return ops.qkv_attention(qkv, H)                      # [N, L, C]


class SelfOutput(nn.Module):
    def __init__(self, width: int):
        super().__init__()
        self.dense = nn.Linear(width, width)


class Attention(nn.Module):
    def __init__(self, width: int, heads: int):
        super().__init__()
        self.attention = SelfAttention(width, heads)
        self.output = SelfOutput(width)


class LayerScale(nn.Module):
    def __init__(self, width: int):
        super().__init__()
        self.lambda1 = nn.Parameter(torch.ones(width))


class Mlp(nn.Module):
    def __init__(self, width: int, hidden: int):
        super().__init__()
        self.fc1 = nn.Linear(width, hidden)
        self.fc2 = nn.Linear(hidden, width)


class ViTLayer(nn.Module):
    def __init__(self, width: int, heads: int, num_windows: int):
        super().__init__()
        self.num_windows = max(1, num_windows)
        self.norm1 = nn.LayerNorm(width, eps=1e-6)
        self.attention = Attention(width, heads)
        self.layer_scale1 = LayerScale(width)
        self.norm2 = nn.LayerNorm(width, eps=1e-6)
        self.mlp = Mlp(width, width * 4)
        self.layer_scale2 = LayerScale(width)

    def forward(self, x: torch.Tensor, full_attention: bool) -> torch.Tensor:
        NW, L, C = x.shape
        # (LN(x), x) as one node: the residual and the normalised branch's gradients meet in the
        # LayerNorm backward kernel
        h, x = ops.layer_norm_with_residual(x, self.norm1.weight, self.norm1.bias, 1e-6)
        if full_attention and self.num_windows > 1:
            w2 = self.num_windows ** 2
            h = h.view(NW // w2, w2 * L, C)
        a = self.attention.attention(h).view(NW, L, C)
        d = self.attention.output.dense
        x = ops.linear_scale_residual(a, d.weight, d.bias, self.layer_scale1.lambda1, x)
        h, x = ops.layer_norm_with_residual(x, self.norm2.weight, self.norm2.bias, 1e-6)
        return ops.mlp_scale_residual(h, self.mlp.fc1.weight, self.mlp.fc1.bias, self.mlp.fc2.weight,
                                      self.mlp.fc2.bias, self.layer_scale2.lambda1, x)

    def forward_inference(self, x: torch.Tensor, h: torch.Tensor, full_attention: bool):
        """The layer body without autograd, from its input x and h = norm1(x).  Returns (x1, y)
        with the layer output x1 + lambda2 * y left unformed: the next pre-norm (or the caller)
        forms it in the same pass as its LayerNorm, and the post-attention residual is formed
        by norm2 the same way -- no separate LayerScale-residual pass over the tokens."""
        NW, L, C = x.shape
        if full_attention and self.num_windows > 1:
            w2 = self.num_windows ** 2
            h = h.view(NW // w2, w2 * L, C)
        a = self.attention.attention(h).view(NW, L, C)
        d = self.attention.output.dense
        a = ops.linear(a, d.weight, d.bias)
        h, x1 = ops.scaled_residual_layer_norm(a, x, self.layer_scale1.lambda1, self.norm2.weight,
                                               self.norm2.bias, 1e-6)
        m = ops.linear(h, self.mlp.fc1.weight, self.mlp.fc1.bias, act="gelu")
        return x1, ops.linear(m, self.mlp.fc2.weight, self.mlp.fc2.bias)


class Encoder(nn.Module):
    def __init__(self, cfg: RfDetrConfig):
        super().__init__()
        self.layer = nn.ModuleList(ViTLayer(cfg.vit_width, cfg.vit_heads, cfg.num_windows)
                                   for _ in range(cfg.vit_depth))


class WindowedDinov2(nn.Module):
    """`backbone.0.encoder.encoder` in the checkpoint."""

    def __init__(self, cfg: RfDetrConfig):
        super().__init__()
        self.cfg = cfg
        self.embeddings = Embeddings(cfg)
        self.encoder = Encoder(cfg)
        self.layernorm = nn.LayerNorm(cfg.vit_width, eps=1e-6)
        self.taps = tuple(cfg.out_feature_indexes)
        self.grad_marks = None     # callable(i) run by GradMark's backward (data-parallel buckets)

    def forward(self, pixels: torch.Tensor) -> List[torch.Tensor]:
        """Returns the tapped feature maps, channels-last [B, h, w, C]."""
        B, _, H, W = pixels.shape
        p, nw = self.cfg.patch_size, max(1, self.cfg.num_windows)
        x = self.embeddings(pixels)
        states = {}
        full_stages = set(self.taps)
        if torch.is_grad_enabled() or not _FUSED_RESIDUAL_INFERENCE:
            marks = self.grad_marks if torch.is_grad_enabled() else None
            for i, layer in enumerate(self.encoder.layer):
                if marks is not None:
                    x = GradMark.apply(x, i, marks)
                if i in full_stages:
                    states[i] = x
                x = layer(x, i in full_stages)
        else:
            # inference: each layer's output x + lambda2 * y is formed by the next layer's norm1
            y = gamma = None
            for i, layer in enumerate(self.encoder.layer):
                n1 = layer.norm1
                if y is None:
                    h = ops.layer_norm(x, n1.weight, n1.bias, 1e-6)
                else:
                    h, x = ops.scaled_residual_layer_norm(y, x, gamma, n1.weight, n1.bias, 1e-6)
                if i in full_stages:
                    states[i] = x
                x, y = layer.forward_inference(x, h, i in full_stages)
                gamma = layer.layer_scale2.lambda1
            if y is not None:
                x = torch.addcmul(x, y, gamma.to(y.dtype))
        states[len(self.encoder.layer)] = x
        hp, wp = H // p, W // p
        hpw, wpw = hp // nw, wp // nw
        # final norm, cls drop and un-windowing of every tap in one mapped LayerNorm per tap, written
        # side by side along the channels (the projector's concatenated input)
        return ops.taps_layer_norm([states[s] for s in self.taps], self.layernorm.weight, self.layernorm.bias, 1e-6,
                                   B, nw, hpw, wpw)


class GradMark(torch.autograd.Function):
    """Identity whose backward calls ``cb(i)`` when the gradient reaches the input of ViT layer
    ``i``: by then the backward pass has produced every gradient of layers i.. and of everything
    after the backbone (the data-parallel sync starts reducing those while the pass goes on)."""

    @staticmethod
    def forward(ctx, x, i, cb):
        ctx.i, ctx.cb = i, cb
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        ctx.cb(ctx.i)
        return g, None, None


def grad_stage(name: str) -> int:
    """Backward-completion stage of a parameter (larger = complete earlier): 0 for the patch /
    position embeddings, 1 + i for ViT layer i, a large value for everything after the ViT
    (final encoder norm, projector, transformer, heads)."""
    if ".encoder.embeddings." in name:
        return 0
    m = re.search(r"\.encoder\.layer\.(\d+)\.", name)
    if m:
        return 1 + int(m.group(1))
    return 1 << 20


class DinoV2Wrapper(nn.Module):
    def __init__(self, cfg: RfDetrConfig):
        super().__init__()
        self.encoder = WindowedDinov2(cfg)

    def forward(self, pixels):
        return self.encoder(pixels)
