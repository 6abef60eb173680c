"""Scaled dot-product attention for the windowed ViT and the Group-DETR decoder.

``attention(q, k, v)``: q/k/v [N, H, L, D] -> [N, H, L, D], softmax scale 1/sqrt(D).
Reference: `at::scaled_dot_product_attention` (`src/rfdetr/layers/model.cpp:498`) and
`nn::MultiheadAttention` (`model.cpp:917`).

On CUDA with bf16 and head_dim 64 this runs the framework's tcgen05 flash
attention (S = Q K^T accumulated in TMEM, online softmax on the tcgen05.ld
read-back, P V accumulated in TMEM).  Other shapes and the CPU path use the
math definition (the oracle).
"""
from __future__ import annotations

import math
import os

import torch
import torch.nn.functional as F

from ._ext import kernels

__all__ = ["attention", "attention_reference", "set_flash_enabled"]

_state = {"enabled": os.environ.get("MMLTK_TC_ATTN", "1") != "0"}


def set_flash_enabled(flag: bool) -> None:
    _state["enabled"] = bool(flag)


def attention_reference(q, k, v):
    scale = 1.0 / math.sqrt(q.shape[-1])
    s = torch.matmul(q.float(), k.float().transpose(-1, -2)) * scale
    p = torch.softmax(s, -1)
    return torch.matmul(p, v.float()).to(q.dtype)


class _FlashFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v):
        o, lse = kernels().flash_fwd(q, k, v)
        ctx.save_for_backward(q, k, v, o, lse)
        return o

    @staticmethod
    def backward(ctx, go):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = kernels().flash_bwd(go.contiguous(), q, k, v, o, lse)
        return dq, dk, dv


def _flash_ok(q):
    return (_state["enabled"] and q.is_cuda and q.dtype == torch.bfloat16 and q.shape[-1] == 64
            and hasattr(kernels(), "flash_fwd"))


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    if q.is_cuda:
        if _flash_ok(q):
            return _FlashFn.apply(q.contiguous(), k.contiguous(), v.contiguous())
        return F.scaled_dot_product_attention(q, k, v)
    return attention_reference(q, k, v)
