"""Scaled dot-product attention for the windowed ViT and the Group-DETR decoder.

``attention(q, k, v)``: q/k/v [N, H, L, D] -> [N, H, L, D], softmax scale 1/sqrt(D).
``qkv_attention(qkv, heads)``: packed projections [N, L, 3C] -> [N, L, C] (the ViT layout).
Reference: `at::scaled_dot_product_attention` (`src/rfdetr/layers/model.cpp:498`) and
`nn::MultiheadAttention` (`model.cpp:917`).

Sequences of at most 384 tokens with head dim 32 or 64 -- the Group-DETR decoder's
self-attention (300 queries per group, head dim 32) and the windowed ViT layers (325 tokens,
head dim 64) -- run the framework's own tcgen05 kernels forward and backward
(``short_attention``, ``attn_short.cu``: one CTA per (sequence, head), the whole score row in
tensor memory, exact softmax, dV / dK / dQ accumulated on chip), reading q / k / v straight out
of the projection outputs and writing the gradients straight into the projection gradients.
Longer sequences (the ViT's global layers) run cuDNN's sm100 flash attention (library kernel).
The framework's own tcgen05 forward (``attn_tc.cu``: q / k / v read by TMA straight
out of the packed projection, S and P.V accumulated in tensor memory, online softmax
in registers) is exact to the same tolerance but measured 1.3-2x slower than cuDNN on
the RF-DETR shapes (one softmax warpgroup per CTA leaves the tensor core idle while
it runs), so inference uses it only with ``MMLTK_ATTN_TC=1``.  ``qkv_attention``
owns the data layout around it: q, k and v are strided views straight into
the packed projection output (no split / permute copies), the output comes
back in [N, L, H, D] order so the output projection reads it without a
transpose, and in the backward pass dq / dk / dv are written into the packed
[N, L, 3, H, D] gradient with one contiguous stack.  The generic autograd
route (unbind + permute) costs two extra full passes over the gradients per
layer, one of them a slow strided concatenation.  CPU: the math definition
(the oracle).
"""
from __future__ import annotations

import math
import os

import torch
import torch.nn.functional as F

__all__ = ["attention", "attention_reference", "qkv_attention", "qkv_attention_reference", "qkv_attention_tc",
           "short_attention", "short_attention_ok"]

_USE_TC = os.environ.get("MMLTK_ATTN_TC", "0") == "1"
# "1": every sequence of at most 384 tokens on the short-sequence kernels; "d32": head dim 32 only
# (the decoder's self-attention); "0": none
_SHORT_MODE = os.environ.get("MMLTK_ATTN_SHORT", "0")
SHORT_MAX_L = 384


def _tma_ok(t: torch.Tensor) -> bool:
    return (t.is_cuda and t.dtype == torch.bfloat16 and t.dim() == 2 and t.stride(1) == 1 and t.stride(0) % 8 == 0
            and t.data_ptr() % 16 == 0)


def short_attention_ok(L: int, D: int, *sources: torch.Tensor) -> bool:
    """True when ``short_attention`` takes these operands (CUDA bf16 2-D sources, L <= 384,
    head dim 32 or 64)."""
    use = _SHORT_MODE == "1" or (_SHORT_MODE == "d32" and D == 32)
    return use and 1 <= L <= SHORT_MAX_L and D in (32, 64) and all(_tma_ok(t) for t in sources)


class _ShortAttnFn(torch.autograd.Function):
    """q / k from columns of ``a``, v from columns of ``b`` (or of ``a`` when b is None)."""

    @staticmethod
    def forward(ctx, a, b, cols, nseq, L, heads, D):
        from ._ext import kernels
        vs = a if b is None else b
        o, lse = kernels().attn_short_fwd(a, cols[0], a, cols[1], vs, cols[2], nseq, L, heads, D)
        ctx.save_for_backward(a, b, o, lse)
        ctx.cfg = (cols, nseq, L, heads, D)
        return o

    @staticmethod
    def backward(ctx, go):
        from ._ext import kernels
        a, b, o, lse = ctx.saved_tensors
        cols, nseq, L, heads, D = ctx.cfg
        go = go.contiguous()
        width = heads * D
        # the kernel writes every head's columns of dq / dk / dv; a source with other columns too
        # gets zeros there
        if b is None:
            da = (torch.empty_like if a.shape[1] == 3 * width else torch.zeros_like)(a)
            db, vdst = None, da
        else:
            da = (torch.empty_like if a.shape[1] == 2 * width else torch.zeros_like)(a)
            db = (torch.empty_like if b.shape[1] == width else torch.zeros_like)(b)
            vdst = db
        vs = a if b is None else b
        kernels().attn_short_bwd(a, cols[0], a, cols[1], vs, cols[2], o, go, lse, nseq, L, heads, D,
                                 da, cols[0], da, cols[1], vdst, cols[2])
        return da, db, None, None, None, None, None


def short_attention(a: torch.Tensor, b, cols, nseq: int, L: int, heads: int, D: int) -> torch.Tensor:
    """Softmax attention over ``nseq`` sequences of ``L`` tokens, on the tcgen05 short-sequence
    kernels.  ``a`` [nseq * L, *] holds q (head h at column cols[0] + h * D) and k (cols[1] + h * D);
    v is read from ``b`` at cols[2] + h * D, or from ``a`` when ``b`` is None.  Returns
    o [nseq * L, heads * D] (token-major, heads side by side)."""
    if torch.is_grad_enabled() and (a.requires_grad or (b is not None and b.requires_grad)):
        return _ShortAttnFn.apply(a, b, tuple(cols), nseq, L, heads, D)
    from ._ext import kernels
    vs = a if b is None else b
    return kernels().attn_short_fwd(a, cols[0], a, cols[1], vs, cols[2], nseq, L, heads, D)[0]


def attention_reference(q, k, v):
    scale = 1.0 / math.sqrt(q.shape[-1])
    s = torch.matmul(q.float(), k.float().transpose(-1, -2)) * scale
    p = torch.softmax(s, -1)
    return torch.matmul(p, v.float()).to(q.dtype)


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    if q.is_cuda:
        return F.scaled_dot_product_attention(q, k, v)
    return attention_reference(q, k, v)


def _split(qkv: torch.Tensor, heads: int):
    N, L, C3 = qkv.shape
    D = C3 // (3 * heads)
    v5 = qkv.view(N, L, 3, heads, D)
    return [v5[:, :, i].transpose(1, 2) for i in range(3)]   # [N, H, L, D] strided views


# cuDNN's SDPA backward through the framework's cuDNN-graph binding, writing dQ / dK / dV straight
# into the packed [N, L, 3 * C] gradient (``MMLTK_SDPA_PACKED=0``: PyTorch's backward + a stack copy)
_SDPA_PACKED = os.environ.get("MMLTK_SDPA_PACKED", "1") == "1"
_sdpa_ext = []


def _sdpa_packed():
    """The ``_sdpa_packed`` extension, or None where it is switched off or not built."""
    if not _SDPA_PACKED:
        return None
    if not _sdpa_ext:
        from ._ext import _load
        _sdpa_ext.append(_load("_sdpa_packed")[0])
    return _sdpa_ext[0]


class _QKVAttnFn(torch.autograd.Function):
    """Self-attention over a packed projection qkv [N, L, 3 * C] -> [N, L, C] on cuDNN.

    Forward: PyTorch's cuDNN SDPA on strided q / k / v views (its output and log-sum-exp are
    saved).  Backward: the same cuDNN SDPA backward node, built through the cuDNN graph API with
    the packed gradient's strides, so dQ / dK / dV land in their slices of d(qkv) with no copy
    (PyTorch's own backward allocates three dense gradients, which then need a concatenation)."""

    @staticmethod
    def forward(ctx, qkv, heads):
        N, L, C3 = qkv.shape
        C = C3 // 3
        ctx.shape = (N, L, heads, C // heads)
        ext = _sdpa_packed()
        if ext is not None:
            q, k, v = _split(qkv, heads)
            try:
                res = torch.ops.aten._scaled_dot_product_cudnn_attention(q, k, v, None, True, 0.0, False, False)
            except RuntimeError:
                res = None
            if res is not None:
                o, lse = res[0], res[1]
                ctx.save_for_backward(qkv, o, lse)
                ctx.packed = True
                return o.transpose(1, 2).reshape(N, L, C)
        ctx.packed = False
        leaves = [t.detach().requires_grad_() for t in _split(qkv, heads)]
        with torch.enable_grad():
            o = F.scaled_dot_product_attention(*leaves)           # [N, H, L, D]
        ctx.leaves, ctx.o = leaves, o
        return o.detach().transpose(1, 2).reshape(N, L, C)

    @staticmethod
    def backward(ctx, go):
        N, L, H, D = ctx.shape
        g = go.reshape(N, L, H, D).transpose(1, 2)
        if ctx.packed:
            qkv, o, lse = ctx.saved_tensors
            ext = _sdpa_packed()
            q, k, v = _split(qkv, H)
            dqkv = torch.empty_like(qkv)
            dq, dk, dv = _split(dqkv, H)
            scale = 1.0 / math.sqrt(D)
            if not torch.cuda.is_current_stream_capturing() or ext.has_plan(q, k, v, o, g, lse, dq, dk, dv, scale):
                ext.sdpa_bwd(q, k, v, o, g, lse, dq, dk, dv, scale)
                return dqkv, None
            # first call of this shape inside a stream capture: no cuDNN plan is built while
            # capturing; recompute the forward and take PyTorch's backward instead
            leaves = [t.detach().requires_grad_() for t in (q, k, v)]
            with torch.enable_grad():
                o2 = F.scaled_dot_product_attention(*leaves)
            dq, dk, dv = torch.autograd.grad(o2, leaves, g)
        else:
            dq, dk, dv = torch.autograd.grad(ctx.o, ctx.leaves, g)
            ctx.leaves = ctx.o = None
        # [N, L, 3, H, D]: one concatenation of (usually contiguous) [N, L, H, D] gradients
        dqkv = torch.stack([dq.transpose(1, 2), dk.transpose(1, 2), dv.transpose(1, 2)], dim=2)
        return dqkv.view(N, L, 3 * H * D), None


class _QKSplitAttnFn(torch.autograd.Function):
    """Self-attention whose q / k come from one projection qk [..., 2 * C] (q | k) and v from
    another [..., C]; rows are ``nseq`` sequences of ``L`` tokens.  cuDNN forward on strided views;
    the cuDNN-graph backward writes dQ / dK into d(qk) and dV into d(v) in place (PyTorch's backward
    would return dense dQ / dK that the split's backward then concatenates)."""

    @staticmethod
    def forward(ctx, qk, v, nseq, L, heads):
        C = v.shape[-1]
        D = C // heads
        q, k, vv = _qk_views(qk, v, nseq, L, heads, D)
        o, lse = torch.ops.aten._scaled_dot_product_cudnn_attention(q, k, vv, None, True, 0.0, False, False)[:2]
        ctx.save_for_backward(qk, v, o, lse)
        ctx.dims = (nseq, L, heads, D)
        return o.transpose(1, 2).reshape(v.shape)

    @staticmethod
    def backward(ctx, go):
        qk, v, o, lse = ctx.saved_tensors
        nseq, L, H, D = ctx.dims
        q, k, vv = _qk_views(qk, v, nseq, L, H, D)
        g = go.reshape(nseq, L, H, D).transpose(1, 2)
        dqk, dv = torch.empty_like(qk), torch.empty_like(v)
        dq, dk, dvv = _qk_views(dqk, dv, nseq, L, H, D)
        scale = 1.0 / math.sqrt(D)
        ext = _sdpa_packed()
        if not torch.cuda.is_current_stream_capturing() or ext.has_plan(q, k, vv, o, g, lse, dq, dk, dvv, scale):
            ext.sdpa_bwd(q, k, vv, o, g, lse, dq, dk, dvv, scale)
            return dqk, dv, None, None, None
        # first call of this shape inside a stream capture (no cuDNN plan is built while capturing)
        leaves = [t.detach().requires_grad_() for t in (q, k, vv)]
        with torch.enable_grad():
            o2 = F.scaled_dot_product_attention(*leaves)
        gq, gk, gv = torch.autograd.grad(o2, leaves, g)
        dq.copy_(gq)
        dk.copy_(gk)
        dvv.copy_(gv)
        return dqk, dv, None, None, None


def _qk_views(qk, v, nseq, L, H, D):
    qk5 = qk.view(nseq, L, 2, H, D)
    return (qk5[:, :, 0].transpose(1, 2), qk5[:, :, 1].transpose(1, 2),
            v.view(nseq, L, H, D).transpose(1, 2))


def qk_split_attention(qk: torch.Tensor, v: torch.Tensor, nseq: int, L: int, heads: int):
    """Attention of ``nseq`` sequences of ``L`` rows each, q | k packed in ``qk`` [..., 2C] and v
    [..., C] (contiguous); returns [..., C] in v's shape.  Training only: returns None without
    autograd or where the cuDNN path does not apply (the caller keeps its own formulation)."""
    if not (torch.is_grad_enabled() and (qk.requires_grad or v.requires_grad)):
        return None                 # inference keeps the caller's forward-only formulation
    if not (qk.is_cuda and qk.dtype in (torch.bfloat16, torch.float16) and v.dtype == qk.dtype
            and qk.is_contiguous() and v.is_contiguous() and _sdpa_packed() is not None
            and qk.shape[-1] == 2 * v.shape[-1] and v.shape[-1] % heads == 0):
        return None
    return _QKSplitAttnFn.apply(qk, v, nseq, L, heads)


def qkv_attention_reference(qkv: torch.Tensor, heads: int) -> torch.Tensor:
    N, L, C3 = qkv.shape
    q, k, v = _split(qkv, heads)
    return attention_reference(q, k, v).transpose(1, 2).reshape(N, L, C3 // 3)


def qkv_attention_tc(qkv: torch.Tensor, heads: int, want_lse: bool = False):
    """tcgen05 forward: qkv [N, L, 3 * heads * 64] bf16 -> o [N, L, heads * 64]
    (and, with ``want_lse``, the natural-log row log-sum-exp [N, heads, L] fp32)."""
    from ._ext import kernels
    o, lse = kernels().attn_fwd_tc(qkv, heads, want_lse)
    return (o, lse) if want_lse else o


def qkv_attention(qkv: torch.Tensor, heads: int) -> torch.Tensor:
    if qkv.is_cuda and qkv.dtype in (torch.bfloat16, torch.float16):
        N, L, C3 = qkv.shape
        D = C3 // (3 * heads)
        if qkv.is_contiguous() and short_attention_ok(L, D, qkv.view(N * L, C3)):
            C = C3 // 3
            return short_attention(qkv.view(N * L, C3), None, (0, C, 2 * C), N, L, heads, D).view(N, L, C)
        if torch.is_grad_enabled() and qkv.requires_grad:
            return _QKVAttnFn.apply(qkv, heads)
        if _USE_TC and qkv.dtype == torch.bfloat16 and qkv.shape[-1] == 3 * 64 * heads:
            return qkv_attention_tc(qkv, heads)
        N, L, C3 = qkv.shape
        o = F.scaled_dot_product_attention(*_split(qkv, heads))
        return o.transpose(1, 2).reshape(N, L, C3 // 3)
    return qkv_attention_reference(qkv, heads)
