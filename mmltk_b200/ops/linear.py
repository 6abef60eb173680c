"""Dense layers with fused epilogues.

``linear(x, w, b, act)``                       y = act(x W^T + b)       act in {None, "gelu", "relu"}
``linear_scale_residual(x, w, b, gamma, res)`` y = res + gamma * (x W^T + b)   (ViT LayerScale + residual)

CUDA (bf16): one autograd node per layer.  The products run on the tensor
cores through ``gemm`` (``mmltk_b200.ops.gemm``: the framework's tcgen05/TMEM
kernel where the shape qualifies, cuBLAS otherwise); the memory-bound parts
are framework kernels: the bias gradient is a single-pass column sum
(``colsum``), the activation backward and the LayerScale backward
(``g_pre = gy * gamma`` together with ``g_gamma = colsum(gy * pre)``) are one
pass each.  This replaces autograd's generic ``AddmmBackward`` whose
bias-gradient reduction and zero-filled select/slice backwards dominated the
step profile.  CPU: the plain fp32 definition (the oracle).
Reference: every `torch::nn::Linear` of `src/rfdetr/layers/model.cpp` (cuBLAS).
"""
from __future__ import annotations

import os

import torch
import torch.nn.functional as F

from ._ext import kernels
from .gemm import _fits_nt, gemm_nn, gemm_nt, gemm_nt_epilogue, gemm_tn, gemm_tn_acc, tc_gemm_enabled
from .gradacc import grad_target

__all__ = ["ffn_add_norm", "gather_rows", "linear", "linear_pair", "linear_scale_residual", "mlp_scale_residual", "mlp_relu", "set_fused_linear"]

_ACTS = {None: 0, "none": 0, "gelu": 1, "relu": 2}
_COLSUM_CAP = 16384   # widest output whose column sums the GEMM epilogue accumulates (its fp32 scratch)
_state = {"enabled": os.environ.get("MMLTK_FUSED_LINEAR", "1") != "0",
          "fused_mlp": os.environ.get("MMLTK_FUSED_MLP", "0") == "1",
          "fused_ffn": os.environ.get("MMLTK_FUSED_FFN", "1") != "0"}


def set_fused_linear(flag: bool) -> None:
    _state["enabled"] = bool(flag)


def _act(y, act_id):
    if act_id == 1:
        return F.gelu(y)
    if act_id == 2:
        return F.relu(y)
    return y


def _ok(x, w):
    return (_state["enabled"] and x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16
            and x.shape[-1] % 8 == 0 and w.shape[0] % 8 == 0)


def _2d(t, n):
    t2 = t.reshape(-1, n)
    return t2 if t2.is_contiguous() else t2.contiguous()


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, act_id):
        shp = x.shape
        x2 = _2d(x, shp[-1])
        # ReLU: in the GEMM epilogue; its backward needs only the sign of the pre-activation,
        # which the output carries (y > 0 <=> pre > 0), so the epilogue stores y alone.
        # GELU: the GEMM writes the pre-activation (kept for the backward) and one elementwise pass
        # makes y -- measured faster than the epilogue form, whose erf work stalls the 8 epilogue
        # warps of the persistent GEMM.
        fused = gemm_nt_epilogue(x2, w, b, "relu", want_pre=False) if act_id == 2 else None
        bwd_act = act_id
        if fused is not None:
            y, pre = fused
        else:
            pre = gemm_nt(x2, w, b)               # x W^T + b
            if act_id == 1:
                # the GELU pass also writes GELU'(pre), saved instead of pre: the backward is
                # then a multiply (act 3) rather than a second erf evaluation
                y, pre = kernels().gelu_fwd_deriv(pre)
                bwd_act = 3
            else:
                y = _act(pre, act_id) if act_id else pre
        if act_id == 2:
            pre = y
        ctx.save_for_backward(x2, w, pre if act_id else None)
        ctx.act_id, ctx.has_bias, ctx.shp = bwd_act, b is not None, shp
        ctx.params = (w, b)                       # the Parameter objects (their .grad may be flat views)
        return y.view(*shp[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, gy):
        x2, w, pre = ctx.saved_tensors
        k = kernels()
        g = _2d(gy, w.shape[0])
        wt, bt = grad_target(ctx.params[0]), grad_target(ctx.params[1])
        want_b = ctx.has_bias and ctx.needs_input_grad[2]
        gb = None
        if ctx.act_id:
            if want_b:   # activation backward and bias gradient in one pass
                g, gb = k.act_bwd_bias(g, pre, ctx.act_id, bt)
            else:
                g = k.act_bwd(g, pre, ctx.act_id)
        elif want_b:
            gb = k.colsum(g, None, bt)
        gx = gemm_nn(g, w) if ctx.needs_input_grad[0] else None
        gw = None
        if ctx.needs_input_grad[1]:
            gw = gemm_tn(g, x2) if wt is None else gemm_tn_acc(g, x2, wt)
        return ((None if gx is None else gx.view(ctx.shp)), None if wt is not None else gw,
                None if bt is not None else gb, None)


class _LinearScaleResidual(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, gamma, res):
        shp = x.shape
        x2 = _2d(x, shp[-1])
        r2 = _2d(res, w.shape[0])
        fused = gemm_nt_epilogue(x2, w, b, "scale_residual", r2, gamma)
        if fused is not None:
            y, pre = fused                        # res + gamma * (x W^T + b) in the GEMM epilogue
        else:
            pre = gemm_nt(x2, w, b)
            y = torch.addcmul(r2, pre, gamma.to(pre.dtype))
        ctx.save_for_backward(x2, w, gamma, pre)
        ctx.shp = shp
        ctx.params = (w, b, gamma)
        return y.view(*shp[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, gy):
        x2, w, gamma, pre = ctx.saved_tensors
        k = kernels()
        g = _2d(gy, w.shape[0])
        wt, bt, gt = (grad_target(p) for p in ctx.params)
        # LayerScale and bias gradients in the same pass that makes g_pre
        if (gt is None) == (bt is None) and (bt is None or bt.dtype == gt.dtype):
            g_pre, g_gamma, gb = k.scale_bias_bwd(g, pre, gamma, gt, bt, gamma.dtype)
        else:
            g_pre, g_gamma = k.scale_bwd(g, pre, gamma, gt)
            gb = k.colsum(g_pre, None, bt)
        gx = gemm_nn(g_pre, w)
        gw = gemm_tn(g_pre, x2) if wt is None else gemm_tn_acc(g_pre, x2, wt)
        return (gx.view(ctx.shp), None if wt is not None else gw, None if bt is not None else gb,
                None if gt is not None else g_gamma, gy)


def linear(x: torch.Tensor, w: torch.Tensor, b=None, act=None) -> torch.Tensor:
    if _ok(x, w):
        return _Linear.apply(x, w, b, _ACTS[act])
    n = w.shape[0]
    if n % 8 and _ok(x, w.new_empty(8, w.shape[1])):
        # Output widths that are not a multiple of 8 (the 91-class heads, the 4-wide box heads) make
        # cuBLAS fall back to its 2-byte-aligned kernels, several times slower for the [B*Q, 91]
        # logits, the [4 * B*Q, 4] box deltas and their weight gradients.  Padding the weight rows to
        # a multiple of 8 keeps every product on the aligned path.
        pad = (-n) % 8
        wp = F.pad(w, (0, 0, 0, pad))
        bp = None if b is None else F.pad(b, (0, pad))
        return _Linear.apply(x, wp, bp, _ACTS[act])[..., :n].contiguous()
    return _act(F.linear(x, w.to(x.dtype), None if b is None else b.to(x.dtype)), _ACTS[act])


class _LinearPair(torch.autograd.Function):
    """(x W1^T + b1, x W2^T + b2): two linears that read the same input as one autograd node, so the
    input gradient is g1 W1 + g2 W2 from two GEMMs, the second accumulating into the first (beta = 1),
    instead of two GEMMs and a separate add of the two gradients."""

    @staticmethod
    def forward(ctx, x, w1, b1, w2, b2):
        shp = x.shape
        x2 = _2d(x, shp[-1])
        y1, y2 = gemm_nt(x2, w1, b1), gemm_nt(x2, w2, b2)
        ctx.save_for_backward(x2, w1, w2)
        ctx.params = (w1, b1, w2, b2)
        ctx.shp = shp
        return y1.view(*shp[:-1], w1.shape[0]), y2.view(*shp[:-1], w2.shape[0])

    @staticmethod
    def backward(ctx, g1, g2):
        x2, w1, w2 = ctx.saved_tensors
        k = kernels()
        outs = []
        gx = None
        for g, w, wp, bp in ((g1, w1, ctx.params[0], ctx.params[1]), (g2, w2, ctx.params[2], ctx.params[3])):
            if g is None:
                outs += [None, None]
                continue
            g = _2d(g, w.shape[0])
            wt, bt = grad_target(wp), grad_target(bp)
            gb = k.colsum(g, None, bt) if bp is not None else None
            gw = gemm_tn(g, x2) if wt is None else gemm_tn_acc(g, x2, wt)
            gx = gemm_nn(g, w) if gx is None else gx.addmm_(g, w)
            outs += [None if wt is not None else gw, None if bt is not None else gb]
        return (None if gx is None else gx.view(ctx.shp)), *outs


def linear_pair(x, w1, b1, w2, b2):
    """Two linears of the same input (the deformable attention's sampling offsets and attention
    weights), one autograd node whose input gradient needs no separate add."""
    if _ok(x, w1) and _ok(x, w2) and b1 is not None and b2 is not None and torch.is_grad_enabled():
        return _LinearPair.apply(x, w1, b1, w2, b2)
    return linear(x, w1, b1), linear(x, w2, b2)


def linear_scale_residual(x, w, b, gamma, res):
    if _ok(x, w) and gamma.dtype == x.dtype:
        return _LinearScaleResidual.apply(x, w, b, gamma, res)
    return res + gamma.to(x.dtype) * F.linear(x, w.to(x.dtype), b.to(x.dtype))


class _MlpScaleResidual(torch.autograd.Function):
    """y = res + gamma * (fc2(GELU(fc1(x)))) -- the ViT MLP sub-block as one autograd node, so that
    the backward can fuse across the two layers: the fc2 input-gradient GEMM multiplies by the
    stored GELU'(fc1 pre-activation) in its epilogue and accumulates the fc1 bias gradient from the
    same tile (no separate activation-backward pass over the [tokens, 4C] gradient).  Forward: fc1
    GEMM, one GELU pass that also stores GELU'(pre) (no erf in the GEMM epilogue), fc2 with the
    LayerScale + residual epilogue."""

    @staticmethod
    def forward(ctx, x, w1, b1, w2, b2, gamma, res):
        shp = x.shape
        x2 = _2d(x, shp[-1])
        r2 = _2d(res, w2.shape[0])
        h, d1 = kernels().gelu_fwd_deriv(gemm_nt(x2, w1, b1))
        y, pre2 = gemm_nt_epilogue(h, w2, b2, "scale_residual", r2, gamma, force=True)
        ctx.save_for_backward(x2, w1, d1, h, w2, gamma, pre2)
        ctx.params = (w1, b1, w2, b2, gamma)
        ctx.shp = shp
        return y.view(*shp[:-1], w2.shape[0])

    @staticmethod
    def backward(ctx, gy):
        x2, w1, d1, h, w2, gamma, pre2 = ctx.saved_tensors
        k = kernels()
        wt1, bt1, wt2, bt2, gt = (grad_target(p) for p in ctx.params)
        g = _2d(gy, w2.shape[0])
        if (gt is None) == (bt2 is None) and (bt2 is None or bt2.dtype == gt.dtype):
            g_pre2, g_gamma, gb2 = k.scale_bias_bwd(g, pre2, gamma, gt, bt2, gamma.dtype)
        else:
            g_pre2, g_gamma = k.scale_bwd(g, pre2, gamma, gt)
            gb2 = k.colsum(g_pre2, None, bt2)
        gw2 = gemm_tn(g_pre2, h) if wt2 is None else gemm_tn_acc(g_pre2, h, wt2)
        gb1 = bt1 if bt1 is not None else torch.empty(w1.shape[0], device=g.device, dtype=w1.dtype)
        # fc2 input gradient, GELU backward (x stored GELU') and the fc1 bias gradient in one GEMM launch
        g_pre1 = k.gemm_tc(g_pre2, w2, None, False, True, 8, False, d1, None, gb1, bt1 is not None)[0]
        gw1 = gemm_tn(g_pre1, x2) if wt1 is None else gemm_tn_acc(g_pre1, x2, wt1)
        gx = gemm_nn(g_pre1, w1)
        none_if = lambda t, v: None if t is not None else v
        return (gx.view(ctx.shp), none_if(wt1, gw1), none_if(bt1, gb1), none_if(wt2, gw2), none_if(bt2, gb2),
                none_if(gt, g_gamma), gy)


def mlp_scale_residual(x, w1, b1, w2, b2, gamma, res):
    """res + gamma * (GELU(x W1^T + b1) W2^T + b2); the cross-layer fused backward with
    ``MMLTK_FUSED_MLP=1``."""
    if (_state["fused_mlp"] and _ok(x, w1) and _ok(x, w2.new_empty(8, w2.shape[1])) and gamma.dtype == x.dtype
            and w1.shape[0] % 128 == 0 and tc_gemm_enabled()):
        x2 = x.reshape(-1, x.shape[-1])
        if _fits_nt(x2 if x2.is_contiguous() else x2.contiguous(), w1):
            return _MlpScaleResidual.apply(x, w1, b1, w2, b2, gamma, res)
    h = linear(x, w1, b1, act="gelu")
    return linear_scale_residual(h, w2, b2, gamma, res)


class _MlpRelu(torch.autograd.Function):
    """out = ReLU(x W1^T + b1) W2^T -- the decoder FFN (its output bias is added by the following
    norm) as one autograd node.  Forward: the first product with the ReLU in the tcgen05 epilogue
    (only h is stored: h > 0 <=> pre > 0).  Backward: the second layer's input-gradient GEMM applies
    the ReLU mask of h in its epilogue and sums the first layer's bias gradient from the stored
    tile (epilogue 5 + column sums), so the [tokens, 2048] gradient is written once and never
    re-read for the activation backward."""

    @staticmethod
    def forward(ctx, x, w1, b1, w2):
        shp = x.shape
        x2 = _2d(x, shp[-1])
        h, _ = gemm_nt_epilogue(x2, w1, b1, "relu", want_pre=False, force=True)
        out = gemm_nt(h, w2)
        ctx.save_for_backward(x2, w1, h, w2)
        ctx.params = (w1, b1, w2)
        ctx.shp = shp
        return out.view(*shp[:-1], w2.shape[0])

    @staticmethod
    def backward(ctx, gy):
        x2, w1, h, w2 = ctx.saved_tensors
        k = kernels()
        wt1, bt1, wt2 = (grad_target(p) for p in ctx.params)
        g = _2d(gy, w2.shape[0])
        gw2 = gemm_tn(g, h) if wt2 is None else gemm_tn_acc(g, h, wt2)
        gb1 = bt1 if bt1 is not None else torch.empty(w1.shape[0], device=g.device, dtype=w1.dtype)
        # dh = g W2 with the ReLU mask and the bias-gradient column sums in the GEMM epilogue
        g_pre1 = k.gemm_tc(g, w2, None, False, True, 5, False, h, None, gb1, bt1 is not None)[0]
        gw1 = gemm_tn(g_pre1, x2) if wt1 is None else gemm_tn_acc(g_pre1, x2, wt1)
        gx = gemm_nn(g_pre1, w1)
        none_if = lambda t, v: None if t is not None else v
        return gx.view(ctx.shp), none_if(wt1, gw1), none_if(bt1, gb1), none_if(wt2, gw2)


def mlp_relu(x, w1, b1, w2):
    """ReLU(x W1^T + b1) W2^T (no output bias), the decoder FFN; one fused autograd node on the
    tcgen05 GEMM where the shapes fit (``MMLTK_FUSED_FFN=0``: two separate linears)."""
    if (_state["fused_ffn"] and _ok(x, w1) and _ok(x, w2.new_empty(8, w2.shape[1])) and tc_gemm_enabled()
            and w1.shape[0] % 128 == 0 and w1.shape[0] <= _COLSUM_CAP and torch.is_grad_enabled()):
        x2 = x.reshape(-1, x.shape[-1])
        if _fits_nt(x2 if x2.is_contiguous() else x2.contiguous(), w1):
            return _MlpRelu.apply(x, w1, b1, w2)
    h = linear(x, w1, b1, act="relu")
    return linear(h, w2, None)



class _GatherRows(torch.autograd.Function):
    """table.index_select(0, rows) whose backward adds the rows' gradients back with packed bf16
    reductions in one kernel (rows may repeat: the two-stage head's groups pick overlapping tokens)."""

    @staticmethod
    def forward(ctx, table, rows):
        ctx.save_for_backward(rows)
        ctx.R = table.shape[0]
        return table.index_select(0, rows)

    @staticmethod
    def backward(ctx, g):
        (rows,) = ctx.saved_tensors
        return kernels().index_add_rows(g.contiguous(), rows, ctx.R), None


def gather_rows(table: torch.Tensor, rows: torch.Tensor) -> torch.Tensor:
    """table [R, C][rows] with a one-kernel backward on the GPU (bf16, C % 8 == 0)."""
    if (table.is_cuda and table.dtype == torch.bfloat16 and table.shape[1] % 8 == 0 and rows.dtype == torch.int64
            and hasattr(kernels(), "index_add_rows")):
        return _GatherRows.apply(table, rows)
    return table.index_select(0, rows)


class _FfnAddNormFn(torch.autograd.Function):
    """y = LN(x + ReLU(x W1^T + b1) W2^T + b2) [, y + pos]: the decoder's FFN sub-block and its
    post-norm as one node.  The backward runs the norm first, then the FFN on the norm's input
    gradient g, and forms the input gradient g + g_pre1 W1 in the last GEMM (beta = 1), so the two
    gradients that reach x (residual and FFN) need no separate add."""

    @staticmethod
    def forward(ctx, x, w1, b1, w2, b2, nw, nb, pos, eps):
        shp = x.shape
        C = shp[-1]
        x2 = _2d(x, C)
        h, _ = gemm_nt_epilogue(x2, w1, b1, "relu", want_pre=False, force=True)
        o = gemm_nt(h, w2)                                # b2 is added by the norm kernel
        p2 = pos.contiguous().view(-1, C) if pos is not None else None
        y, mean, rstd, s, y2 = kernels().layernorm_fwd(x2, nw, nb, float(eps), o, p2, b2.to(nw.dtype).contiguous())
        ctx.save_for_backward(x2, w1, h, w2, s, nw, mean, rstd)
        ctx.params = (w1, b1, w2, b2, nw, nb)
        ctx.shp, ctx.has_pos = shp, pos is not None
        if ctx.has_pos:
            return y.view(shp), y2.view(shp)
        return y.view(shp)

    @staticmethod
    def backward(ctx, gy, gy2=None):
        x2, w1, h, w2, s, nw, mean, rstd = ctx.saved_tensors
        k = kernels()
        wt1, bt1, wt2, bt2, nwt, nbt = (grad_target(p) for p in ctx.params)
        gy = gy.contiguous().view(s.shape) if gy is not None else torch.zeros_like(s)
        g2 = gy2.contiguous().view(s.shape) if (ctx.has_pos and gy2 is not None) else None
        acc_n = nwt is not None and nbt is not None
        b2_ok = bt2 is not None and bt2.dtype == nw.dtype
        g, dnw, dnb, db2 = k.layernorm_bwd(gy, s, nw, mean, rstd, nwt if acc_n else None, nbt if acc_n else None, g2,
                                           None, True, bt2 if b2_ok else None)
        # FFN backward on the norm's input gradient g: the second layer's input gradient on the
        # library GEMM, then one pass for the ReLU mask and the first bias's gradient (measured
        # faster than the tcgen05 GEMM with both in its epilogue: that product is load-bound)
        gw2 = gemm_tn(g, h) if wt2 is None else gemm_tn_acc(g, h, wt2)
        g_pre1, gb1 = k.act_bwd_bias(gemm_nn(g, w2), h, 2, bt1)
        gw1 = gemm_tn(g_pre1, x2) if wt1 is None else gemm_tn_acc(g_pre1, x2, wt1)
        gx = torch.addmm(g, g_pre1, w1)                   # residual + FFN input gradients
        none_if = lambda t, v: None if t is not None else v
        db2_out = None if b2_ok else (db2.to(ctx.params[3].dtype) if db2 is not None else None)
        gpos = g2.view(ctx.shp) if g2 is not None else None
        return (gx.view(ctx.shp), none_if(wt1, gw1), none_if(bt1, gb1), none_if(wt2, gw2), db2_out,
                None if acc_n else dnw, None if acc_n else dnb, gpos, None)


def ffn_add_norm(x, w1, b1, w2, b2, nw, nb, eps: float, pos=None):
    """LN(x + ReLU(x W1^T + b1) W2^T + b2) (and that + pos): the decoder's FFN block and post-norm,
    one fused node on the GPU where the FFN takes the tensor-core path, else the separate ops."""
    from .norm import add_layer_norm
    C = x.shape[-1]
    if (_state["fused_ffn"] and _ok(x, w1) and _ok(x, w2.new_empty(8, w2.shape[1])) and tc_gemm_enabled()
            and w1.shape[0] % 128 == 0 and w1.shape[0] <= _COLSUM_CAP and torch.is_grad_enabled()
            and C % 8 == 0 and (pos is None or (pos.dtype == x.dtype and pos.shape == x.shape))
            and b2 is not None):
        x2 = x.reshape(-1, C)
        if _fits_nt(x2 if x2.is_contiguous() else x2.contiguous(), w1):
            return _FfnAddNormFn.apply(x, w1, b1, w2, b2, nw, nb, pos, eps)
    h = mlp_relu(x, w1, b1, w2)
    return add_layer_norm(x, h, nw, nb, eps, pos=pos, rbias=b2)
