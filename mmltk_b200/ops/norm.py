"""LayerNorm over the last dimension (ViT eps 1e-6, decoder eps 1e-5, LayerNorm2d
as channels-last LN).  Reference: `torch::nn::LayerNorm` uses in
`src/rfdetr/layers/model.cpp:267-285,535-541,873-886` (libtorch kernel).

CUDA: one warp per row, fp32 statistics, bf16/fp32 I/O; backward computes dx
per row and dgamma/dbeta in the same launch (per-CTA partials added into fp32
accumulators, the last CTA writes or accumulates into ``.grad``).  CPU:
``torch.nn.functional.layer_norm`` (the oracle).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import kernels
from .gradacc import grad_target

__all__ = ["layer_norm"]


class _LayerNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, eps):
        shape = x.shape
        x2 = x.contiguous().view(-1, shape[-1])
        y, mean, rstd = kernels().layernorm_fwd(x2, weight, bias, float(eps))
        ctx.save_for_backward(x2, weight, mean, rstd)
        ctx.shape = shape
        ctx.params = (weight, bias)
        return y.view(shape)

    @staticmethod
    def backward(ctx, gy):
        x2, weight, mean, rstd = ctx.saved_tensors
        gy2 = gy.contiguous().view(x2.shape)
        wt, bt = grad_target(ctx.params[0]), grad_target(ctx.params[1])
        if wt is not None and bt is not None:   # weight / bias gradients added straight into .grad
            dx, _, _ = kernels().layernorm_bwd(gy2, x2, weight, mean, rstd, wt, bt)
            return dx.view(ctx.shape), None, None, None
        dx, dw, db = kernels().layernorm_bwd(gy2, x2, weight, mean, rstd)
        return dx.view(ctx.shape), dw, db, None


def layer_norm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float) -> torch.Tensor:
    if x.is_cuda and x.shape[-1] % 8 == 0 and x.dtype in (torch.bfloat16, torch.float32):
        return _LayerNormFn.apply(x, weight, bias, eps)
    return F.layer_norm(x, (x.shape[-1],), weight.to(x.dtype), bias.to(x.dtype), eps)
