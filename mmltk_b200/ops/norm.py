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

__all__ = ["scaled_residual_layer_norm", "layer_norm", "add_layer_norm", "layer_norm_with_residual",
           "taps_layer_norm", "concat_channels", "grouped_layer_norm"]


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


class _LayerNormSiluFn(torch.autograd.Function):
    """SiLU(LN(x)) in one kernel each way; the backward recomputes the pre-activation from x."""

    @staticmethod
    def forward(ctx, x, weight, bias, eps):
        shape = x.shape
        x2 = x.contiguous().view(-1, shape[-1])
        y, mean, rstd = kernels().layernorm_act_fwd(x2, weight, bias, float(eps), 1)
        ctx.save_for_backward(x2, weight, bias, mean, rstd)
        ctx.shape, ctx.params = shape, (weight, bias)
        return y.view(shape)

    @staticmethod
    def backward(ctx, gy):
        x2, weight, bias, mean, rstd = ctx.saved_tensors
        g2 = gy.contiguous().view(x2.shape)
        wt, bt = grad_target(ctx.params[0]), grad_target(ctx.params[1])
        if wt is not None and bt is not None:
            dx = kernels().layernorm_act_bwd(g2, x2, weight, bias, mean, rstd, 1, wt, bt)[0]
            return dx.view(ctx.shape), None, None, None
        dx, dw, db = kernels().layernorm_act_bwd(g2, x2, weight, bias, mean, rstd, 1)
        return dx.view(ctx.shape), dw, db, None


def layer_norm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float, act: str = None) -> torch.Tensor:
    """LayerNorm over the last dimension; ``act="silu"`` also applies SiLU (in the same kernel on the GPU)."""
    if x.is_cuda and x.shape[-1] % 8 == 0 and x.dtype in (torch.bfloat16, torch.float32):
        if act is None:
            return _LayerNormFn.apply(x, weight, bias, eps)
        if act == "silu" and hasattr(kernels(), "layernorm_act_fwd") and weight.dtype == bias.dtype:
            return _LayerNormSiluFn.apply(x, weight, bias, eps)
    y = F.layer_norm(x, (x.shape[-1],), weight.to(x.dtype), bias.to(x.dtype), eps)
    return F.silu(y) if act == "silu" else y


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


# ---------------------------------------------------------------------------------------------
# Backbone taps: the final LayerNorm of every tapped stage, written straight into the projector's
# input.  The stages are [windows, 1 + h*w tokens, C] in the windowed token order (a cls token per
# window); the projector wants the image grid [B, hp, wp, taps * C], taps side by side along the
# channels.  One mapped LayerNorm per tap writes each token row to its grid row (cls rows: nowhere)
# at the tap's channel offset, so the slice / un-window permute / concatenation copies (and their
# backward copies and zero fills) disappear; the backward reads each tap's gradient columns through
# the same map.

_TAP_MAPS = {}


def _tap_row_map(device, B: int, nw: int, hpw: int, wpw: int) -> torch.Tensor:
    """int32 [B * nw^2 * (1 + hpw*wpw)]: grid row (b, wy*hpw + iy, wx*wpw + ix) of each windowed token
    row, -1 for the cls rows.  Built with device kernels and cached per shape -- except while a CUDA
    graph is being captured, when the kernels are only recorded (the map is then the graph's own)."""
    key = (str(device), B, nw, hpw, wpw)
    m = _TAP_MAPS.get(key)
    if m is None:
        capturing = torch.cuda.is_current_stream_capturing()
        L = 1 + hpw * wpw
        r = torch.arange(B * nw * nw * L, device=device, dtype=torch.int64)
        win, t = r // L, r % L
        b, wy, wx = win // (nw * nw), (win % (nw * nw)) // nw, win % nw
        tt = (t - 1).clamp(min=0)
        iy, ix = tt // wpw, tt % wpw
        hp, wp = nw * hpw, nw * wpw
        grid = (b * hp + wy * hpw + iy) * wp + wx * wpw + ix
        m = torch.where(t == 0, torch.full_like(grid, -1), grid).to(torch.int32)
        if not capturing:
            _TAP_MAPS[key] = m
    return m


class _TapsNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, weight, bias, eps, ymap, grid, *states):
        B, hp, wp = grid
        T, C = len(states), states[0].shape[-1]
        # allocated in its final shape (not returned as a view), so the channel slices handed out
        # have it as their base and ``concat_channels`` can return it with its autograd history
        out = torch.empty(B, hp, wp, T * C, device=states[0].device, dtype=states[0].dtype)
        out2 = out.view(B * hp * wp, T * C)
        xs, stats = [], []
        for s, x in enumerate(states):
            x2 = x.contiguous().view(-1, C)
            mean, rstd = kernels().layernorm_fwd_map(x2, weight, bias, float(eps), ymap, out2, s * C)
            xs.append(x2)
            stats += [mean, rstd]
        ctx.save_for_backward(weight, ymap, *xs, *stats)
        ctx.T, ctx.C, ctx.shapes, ctx.params = T, C, [x.shape for x in states], (weight, bias)
        return out

    @staticmethod
    def backward(ctx, g):
        weight, ymap, *rest = ctx.saved_tensors
        T, C = ctx.T, ctx.C
        xs, stats = rest[:T], rest[T:]
        g2 = g.contiguous().view(-1, T * C)
        wt, bt = grad_target(ctx.params[0]), grad_target(ctx.params[1])
        gw = gb = None
        gxs = []
        k = kernels()
        for s in range(T):
            mean, rstd = stats[2 * s], stats[2 * s + 1]
            if wt is not None and bt is not None:      # weight / bias gradients added straight into .grad
                gx = k.layernorm_bwd_map(g2, s * C, ymap, xs[s], weight, mean, rstd, wt, bt)[0]
            elif gw is None:
                gx, gw, gb = k.layernorm_bwd_map(g2, s * C, ymap, xs[s], weight, mean, rstd)
            else:                                       # the taps share the norm: accumulate
                gx = k.layernorm_bwd_map(g2, s * C, ymap, xs[s], weight, mean, rstd, gw, gb)[0]
            gxs.append(gx.view(ctx.shapes[s]))
        return (None if wt is not None else gw, None if bt is not None else gb, None, None, None, *gxs)


def taps_layer_norm(states, weight, bias, eps: float, B: int, nw: int, hpw: int, wpw: int):
    """LayerNorm of every tapped stage [B * nw^2, 1 + hpw*wpw, C] (windowed token order) -> the
    image-grid features [B, nw*hpw, nw*wpw, C] of each tap, as adjacent channel slices of one
    [B, hp, wp, taps * C] tensor (``concat_channels`` of the list returns that tensor)."""
    x0 = states[0]
    C = x0.shape[-1]
    if (x0.is_cuda and x0.dtype in (torch.bfloat16, torch.float32) and C % 8 == 0
            and all(x.shape == x0.shape and x.dtype == x0.dtype for x in states)
            and x0.shape[0] == B * nw * nw and x0.shape[1] == 1 + hpw * wpw and hasattr(kernels(), "layernorm_fwd_map")):
        ymap = _tap_row_map(x0.device, B, nw, hpw, wpw)
        cat = _TapsNormFn.apply(weight, bias, eps, ymap, (B, nw * hpw, nw * wpw), *states)
        return [cat[..., s * C:(s + 1) * C] for s in range(len(states))]
    feats = []
    for x in states:
        h = layer_norm(x, weight, bias, eps)[:, 1:]
        if nw > 1:
            h = h.reshape(B, nw, nw, hpw, wpw, C).permute(0, 1, 3, 2, 4, 5)
        feats.append(h.reshape(B, nw * hpw, nw * wpw, C))
    return feats


def concat_channels(parts):
    """torch.cat(parts, -1), except when the parts are, in order, the adjacent channel slices that
    exactly cover one contiguous tensor (``taps_layer_norm``'s output): that tensor, with no copy."""
    if len(parts) == 1:
        return parts[0]
    base = parts[0]._base
    if base is not None and base.is_contiguous() and base.dim() == parts[0].dim():
        off, width = base.storage_offset(), 0
        ok = True
        for p in parts:
            if (p._base is not base or p.shape[:-1] != base.shape[:-1] or p.stride() != base.stride()
                    or p.storage_offset() != off + width):
                ok = False
                break
            width += p.shape[-1]
        if ok and width == base.shape[-1]:
            return base
    return torch.cat(parts, -1)


class _GroupedLayerNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, eps):
        shape = x.shape
        x2 = x.contiguous().view(-1, shape[-1])
        y, mean, rstd = kernels().layernorm_grouped_fwd(x2, weight, bias, float(eps))
        ctx.save_for_backward(x2, weight, mean, rstd)
        ctx.shape, ctx.params = shape, (weight, bias)
        return y.view(shape)

    @staticmethod
    def backward(ctx, gy):
        x2, weight, mean, rstd = ctx.saved_tensors
        g2 = gy.contiguous().view(x2.shape)
        wt, bt = grad_target(ctx.params[0]), grad_target(ctx.params[1])
        if wt is not None and bt is not None:
            dx = kernels().layernorm_grouped_bwd(g2, x2, weight, mean, rstd, wt, bt)[0]
            return dx.view(ctx.shape), None, None, None
        dx, dw, db = kernels().layernorm_grouped_bwd(g2, x2, weight, mean, rstd)
        return dx.view(ctx.shape), dw, db, None


def grouped_layer_norm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float) -> torch.Tensor:
    """x [G, ..., C] normalised over C with group g's affine weight[g], bias[g] (weight / bias [G, C])."""
    G, C = weight.shape
    if (x.is_cuda and x.dtype in (torch.bfloat16, torch.float32) and C % 8 == 0 and x.shape[0] == G
            and weight.dtype == bias.dtype and hasattr(kernels(), "layernorm_grouped_fwd")):
        return _GroupedLayerNormFn.apply(x, weight, bias, eps)
    y = F.layer_norm(x, (C,), None, None, eps)
    shape = (G,) + (1,) * (x.dim() - 2) + (C,)
    return y * weight.view(shape).to(y.dtype) + bias.view(shape).to(y.dtype)
