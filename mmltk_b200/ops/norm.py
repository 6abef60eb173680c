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

__all__ = ["scaled_residual_layer_norm", "layer_norm", "add_layer_norm", "layer_norm_with_residual"]


class _LayerNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, eps):
        shape = x.shape
        x2 = x.contiguous().view(-1, shape[-1])
        y, mean, rstd = kernels().layernorm_fwd(x2, weight, bias, float(eps))[:3]
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
            dx = kernels().layernorm_bwd(gy2, x2, weight, mean, rstd, wt, bt)[0]
            return dx.view(ctx.shape), None, None, None
        dx, dw, db = kernels().layernorm_bwd(gy2, x2, weight, mean, rstd)[:3]
        return dx.view(ctx.shape), dw, db, None


def layer_norm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float) -> torch.Tensor:
    if x.is_cuda and x.shape[-1] % 8 == 0 and x.dtype in (torch.bfloat16, torch.float32):
        return _LayerNormFn.apply(x, weight, bias, eps)
    return F.layer_norm(x, (x.shape[-1],), weight.to(x.dtype), bias.to(x.dtype), eps)


class _AddLayerNormFn(torch.autograd.Function):
    """y = LN(a + b [+ rbias]) [, y + pos] in one kernel; the sum is stored for the backward.
    ``rbias`` is the bias of the linear that produced ``b`` (that linear runs without it): its
    gradient, the column sums of the norm's input gradient, comes out of the same backward
    kernel instead of a separate reduction."""

    @staticmethod
    def forward(ctx, a, b, weight, bias, pos, rbias, eps):
        shape = a.shape
        C = shape[-1]
        a2 = a.contiguous().view(-1, C)
        b2 = b.contiguous().view(-1, C)
        p2 = pos.contiguous().view(-1, C) if pos is not None else None
        rb = rbias.to(weight.dtype).contiguous() if rbias is not None else None
        y, mean, rstd, s, y2 = kernels().layernorm_fwd(a2, weight, bias, float(eps), b2, p2, rb)
        ctx.save_for_backward(s, weight, mean, rstd)
        ctx.shape = shape
        ctx.params = (weight, bias, rbias)
        ctx.has_pos = pos is not None
        if ctx.has_pos:
            return y.view(shape), y2.view(shape)
        return y.view(shape)

    @staticmethod
    def backward(ctx, gy, gy2=None):
        s, weight, mean, rstd = ctx.saved_tensors
        gy = gy.contiguous().view(s.shape) if gy is not None else torch.zeros_like(s)
        g2 = gy2.contiguous().view(s.shape) if (ctx.has_pos and gy2 is not None) else None
        w_p, b_p, rb_p = ctx.params
        wt, bt = grad_target(w_p), grad_target(b_p)
        rbt = grad_target(rb_p) if rb_p is not None else None
        want_rb = rb_p is not None and ctx.needs_input_grad[5]
        rb_ok = rbt is None or rbt.dtype == weight.dtype
        accumulate = wt is not None and bt is not None
        dx, dw, db, drb = kernels().layernorm_bwd(gy, s, weight, mean, rstd, wt if accumulate else None,
                                                  bt if accumulate else None, g2, None, want_rb,
                                                  rbt if (want_rb and rb_ok) else None)
        if accumulate:
            dw = db = None
        if want_rb and rbt is not None and rb_ok:
            drb = None                                # added into the bias' .grad by the kernel
        elif want_rb and drb is not None:
            drb = drb.to(rb_p.dtype)
        else:
            drb = None
        dx = dx.view(ctx.shape)
        gpos = gy2.view(ctx.shape) if g2 is not None else None
        return dx, dx, dw, db, gpos, drb, None


def add_layer_norm(a: torch.Tensor, b: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float,
                   pos: torch.Tensor = None, rbias: torch.Tensor = None):
    """LN(a + b [+ rbias]), and with ``pos`` also that + pos -- the post-norm residual of a decoder
    layer and the next query (with its position embedding) in one pass.  ``rbias``: the bias of
    the linear that produced ``b``, when that linear was run without it."""
    if (a.is_cuda and a.shape[-1] % 8 == 0 and a.dtype in (torch.bfloat16, torch.float32)
            and b.dtype == a.dtype and b.shape == a.shape and (pos is None or (pos.dtype == a.dtype
                                                                             and pos.shape == a.shape))):
        return _AddLayerNormFn.apply(a, b, weight, bias, pos, rbias, eps)
    x = a + b if rbias is None else a + b + rbias.to(a.dtype)
    y = F.layer_norm(x, (a.shape[-1],), weight.to(a.dtype), bias.to(a.dtype), eps)
    return (y, y + pos) if pos is not None else y


def scaled_residual_layer_norm(y: torch.Tensor, res: torch.Tensor, gamma: torch.Tensor, weight: torch.Tensor,
                               bias: torch.Tensor, eps: float):
    """(LN(res + gamma * y), res + gamma * y) without autograd: a LayerScale residual and the next
    pre-norm in one pass (inference).  On CUDA one LayerNorm kernel reads y and res, stores the
    sum and the normalised rows; elsewhere (or with autograd) the plain expression."""
    C = y.shape[-1]
    if (y.is_cuda and not torch.is_grad_enabled() and C % 8 == 0 and y.dtype in (torch.bfloat16, torch.float32)
            and res.dtype == y.dtype and res.shape == y.shape and gamma.dtype == weight.dtype
            and gamma.numel() == C):
        y2 = y.contiguous().view(-1, C)
        r2 = res.contiguous().view(-1, C)
        out, _m, _r, s = kernels().layernorm_fwd(y2, weight, bias, float(eps), r2, None, None,
                                                 gamma.contiguous())[:4]
        return out.view(y.shape), s.view(y.shape)
    x = res + gamma.to(y.dtype) * y
    return F.layer_norm(x, (C,), weight.to(y.dtype), bias.to(y.dtype), eps), x


class _LayerNormResidualFn(torch.autograd.Function):
    """(LN(x), x): the pre-norm block's normalised input and its residual stream as ONE node, so
    the two gradients that reach x are summed inside the LayerNorm backward kernel instead of
    by a separate add."""

    @staticmethod
    def forward(ctx, x, weight, bias, eps):
        shape = x.shape
        x2 = x.contiguous().view(-1, shape[-1])
        y, mean, rstd = kernels().layernorm_fwd(x2, weight, bias, float(eps))[:3]
        ctx.save_for_backward(x2, weight, mean, rstd)
        ctx.shape = shape
        ctx.params = (weight, bias)
        return y.view(shape), x.view_as(x)

    @staticmethod
    def backward(ctx, gy, gres):
        x2, weight, mean, rstd = ctx.saved_tensors
        gr = gres.contiguous().view(x2.shape) if gres is not None else None
        if gy is None:
            return (gres, None, None, None)
        gy2 = gy.contiguous().view(x2.shape)
        wt, bt = grad_target(ctx.params[0]), grad_target(ctx.params[1])
        if wt is not None and bt is not None:
            dx = kernels().layernorm_bwd(gy2, x2, weight, mean, rstd, wt, bt, None, gr)[0]
            return dx.view(ctx.shape), None, None, None
        dx, dw, db = kernels().layernorm_bwd(gy2, x2, weight, mean, rstd, None, None, None, gr)[:3]
        return dx.view(ctx.shape), dw, db, None


def layer_norm_with_residual(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float):
    """Returns (LN(x), x); use the second output as the block's residual input."""
    if x.is_cuda and x.shape[-1] % 8 == 0 and x.dtype in (torch.bfloat16, torch.float32) and x.requires_grad:
        return _LayerNormResidualFn.apply(x, weight, bias, eps)
    return layer_norm(x, weight, bias, eps), x
