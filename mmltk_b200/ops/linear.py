"""Dense layers with fused epilogues.

``linear(x, w, b, act)``            y = act(x W^T + b)            act in {None, "gelu", "relu"}
``linear_scale_residual(x, w, b, gamma, res)``  y = res + gamma * (x W^T + b)   (ViT LayerScale + residual)

On CUDA with bf16 operands these run the framework's tcgen05/TMEM GEMM
(``gemm_tc``: TMA-fed shared-memory tiles, accumulators in tensor memory, the
epilogue applied on the tcgen05.ld read-back).  The CPU path is the fp32 oracle.
Reference: every `torch::nn::Linear` of `src/rfdetr/layers/model.cpp` (cuBLAS).
"""
from __future__ import annotations

import os

import torch
import torch.nn.functional as F

from ._ext import kernels

__all__ = ["linear", "linear_scale_residual", "gemm_enabled", "set_gemm_enabled"]

_ACTS = {None: 0, "none": 0, "gelu": 1, "relu": 2}
_state = {"enabled": os.environ.get("MMLTK_TC_GEMM", "1") != "0"}


def gemm_enabled() -> bool:
    return _state["enabled"]


def set_gemm_enabled(flag: bool) -> None:
    _state["enabled"] = bool(flag)


def _act(y, act):
    if act == "gelu":
        return F.gelu(y)
    if act == "relu":
        return F.relu(y)
    return y


def _tc_ok(x, w):
    return (_state["enabled"] and x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16
            and x.shape[-1] % 64 == 0 and w.shape[0] % 64 == 0 and hasattr(kernels(), "gemm_tc"))


class _LinearTC(torch.autograd.Function):
    """y = act(x W^T + b) on the tcgen05 GEMM; backward uses the same GEMM with
    transposed operand descriptors (dX = dY' W, dW = dY'^T X)."""

    @staticmethod
    def forward(ctx, x, w, b, act_id):
        shp = x.shape
        x2 = x.reshape(-1, shp[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        k = kernels()
        if act_id == 0:
            y = k.gemm_tc(x2, w, b, 0, None, None)
            pre = None
        else:
            # keep the pre-activation for the backward of the activation
            pre = k.gemm_tc(x2, w, b, 0, None, None)
            y = k.bias_act(pre, None, act_id)
        ctx.save_for_backward(x2, w, pre)
        ctx.act_id = act_id
        ctx.has_bias = b is not None
        ctx.shp = shp
        return y.view(*shp[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, gy):
        x2, w, pre = ctx.saved_tensors
        k = kernels()
        gy2 = gy.reshape(-1, w.shape[0])
        if not gy2.is_contiguous():
            gy2 = gy2.contiguous()
        if ctx.act_id != 0:
            gy2 = k.act_bwd(gy2, pre, ctx.act_id)
        gx = k.gemm_tc_nn(gy2, w)              # [M,N] x [N,K] -> [M,K]
        gw = k.gemm_tc_tn(gy2, x2)             # [M,N]^T x [M,K] -> [N,K]
        gb = k.colsum(gy2) if ctx.has_bias else None
        return gx.view(ctx.shp), gw, gb, None


class _LinearScaleResidualTC(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, gamma, res):
        shp = x.shape
        x2 = x.reshape(-1, shp[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        r2 = res.reshape(-1, w.shape[0])
        if not r2.is_contiguous():
            r2 = r2.contiguous()
        k = kernels()
        pre = k.gemm_tc(x2, w, b, 0, None, None)
        y = k.scale_residual(pre, gamma, r2)
        ctx.save_for_backward(x2, w, gamma, pre)
        ctx.shp = shp
        return y.view(*shp[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, gy):
        x2, w, gamma, pre = ctx.saved_tensors
        k = kernels()
        gy2 = gy.reshape(-1, w.shape[0])
        if not gy2.is_contiguous():
            gy2 = gy2.contiguous()
        g_pre, g_gamma = k.scale_bwd(gy2, pre, gamma)
        gx = k.gemm_tc_nn(g_pre, w)
        gw = k.gemm_tc_tn(g_pre, x2)
        gb = k.colsum(g_pre)
        return gx.view(ctx.shp), gw, gb, g_gamma, gy


def linear(x: torch.Tensor, w: torch.Tensor, b=None, act=None) -> torch.Tensor:
    if _tc_ok(x, w):
        return _LinearTC.apply(x, w, b, _ACTS[act])
    return _act(F.linear(x, w.to(x.dtype), None if b is None else b.to(x.dtype)), act)


def linear_scale_residual(x, w, b, gamma, res):
    if _tc_ok(x, w):
        return _LinearScaleResidualTC.apply(x, w, b, gamma, res)
    return res + gamma.to(x.dtype) * F.linear(x, w.to(x.dtype), b.to(x.dtype))
