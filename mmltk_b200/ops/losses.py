"""Dense negative term of the sigmoid classification losses.

``dense_focal_neg(x, coef) = sum(coef * sigmoid(x)^2 * softplus(x))`` over
every logit [B, Q, C] -- the loss each logit contributes as a negative in
IA-BCE (coef 1) and in the focal / varifocal / position-supervised branches
(coef 1 - alpha); see `src/rfdetr/detection_ops.cpp:715-775,1324-1364`.

CUDA: one reduction kernel reads the bf16 logits once (fp32 math, per-CTA
partials, no atomics); the backward is one elementwise kernel
``g * coef * s^2 * (2 (1 - s) softplus(x) + s)`` with s = sigmoid(x).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import kernels

__all__ = ["dense_focal_neg"]


class _DenseFocalNeg(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, coef):
        xc = x.contiguous()
        out = kernels().dense_focal_neg_fwd(xc, float(coef))
        ctx.save_for_backward(xc)
        ctx.coef = coef
        return out

    @staticmethod
    def backward(ctx, g):
        (x,) = ctx.saved_tensors
        return kernels().dense_focal_neg_bwd(x, g.contiguous(), float(ctx.coef)), None


def dense_focal_neg(x: torch.Tensor, coef: float) -> torch.Tensor:
    if x.is_cuda and hasattr(kernels(), "dense_focal_neg_fwd"):
        return _DenseFocalNeg.apply(x, coef)
    xf = x.float()
    return (coef * torch.sigmoid(xf) ** 2 * F.softplus(xf)).sum()
