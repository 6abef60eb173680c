"""Sine position embedding of reference boxes (reference `src/rfdetr/layers/model.cpp:234-261`).

``sine_embed(pos, dim)``: pos [..., n] (n = 2: x, y or 4: x, y, w, h) -> [..., n * dim] with the
blocks in the order y, x[, w, h]; block entries 2i / 2i+1 are sin / cos of v * 2 pi / 10000^(2i/dim).

CUDA: one fused kernel each way (bf16 output, fp32 position gradient); CPU: the broadcast
torch expression below, which is also the test oracle.
"""
from __future__ import annotations

import math

import torch

from ._ext import kernels

__all__ = ["sine_embed", "sine_embed_reference", "sine_frequencies"]


def sine_frequencies(dim: int, device) -> torch.Tensor:
    """f_i = 2 pi / 10000^(2i / dim), i < dim / 2 (fp32)."""
    i = torch.arange(dim // 2, dtype=torch.float32, device=device)
    return (2 * math.pi) / (10000.0 ** (2 * i / dim))


def sine_embed_reference(pos: torch.Tensor, dim: int) -> torch.Tensor:
    p = pos.float()
    idx = torch.arange(p.shape[-1], device=p.device)
    idx = torch.where(idx < 2, 1 - idx, idx)                         # (y, x[, w, h]); built on the device
    a = p.index_select(-1, idx)[..., None] * sine_frequencies(dim, p.device)   # [..., n, dim/2]
    return torch.stack((a.sin(), a.cos()), -1).flatten(-3)


class _SineEmbedFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, pos, dim):
        p = pos.float().contiguous()
        freq = sine_frequencies(dim, p.device)
        ctx.save_for_backward(p, freq)
        ctx.dim = dim
        ctx.in_dtype = pos.dtype
        return kernels().sine_embed_fwd(p, dim, freq)

    @staticmethod
    def backward(ctx, g):
        p, freq = ctx.saved_tensors
        gp = kernels().sine_embed_bwd(p, ctx.dim, freq, g)
        return gp.to(ctx.in_dtype), None


def sine_embed(pos: torch.Tensor, dim: int) -> torch.Tensor:
    """bf16 on CUDA (the decoder's compute dtype), fp32 on CPU."""
    if pos.is_cuda and pos.shape[-1] in (2, 4) and (pos.shape[-1] * dim) % 256 == 0 and dim <= 256:
        return _SineEmbedFn.apply(pos, dim)
    return sine_embed_reference(pos, dim)
