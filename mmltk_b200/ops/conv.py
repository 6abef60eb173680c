"""3 x 3 convolutions (stride 1, zero padding 1) of channels-last features on the tcgen05 GEMM.

The projector's C2f bottlenecks (reference ``ConvX``, ``src/rfdetr/layers/model.cpp:288-369``) run
3 x 3 convolutions on [B, h, w, C] features.  ``conv3x3`` computes them as implicit GEMMs: every tile
of a few image rows is one product [rows * w pixels, 9 C] x [9 C, N] whose A tiles are 4-D tensor
loads of the input shifted by each tap (``conv3x3_tc`` in ``gemm_tc.cu``; the padding is the loads'
zero fill), so no im2col matrix is written.  The input gradient is the same kernel on the output
gradient with the flipped, transposed weights; the weight gradient is the library's convolution
backward restricted to the weights.

Opt-in (``MMLTK_TC_CONV=1``): measured on one B200 for the RF-DETR-M C2f shape (8 x 36 x 36, 128 ->
128 channels) the forward takes 13.8 us against cuDNN's 10.0 us and forward + backward 45.1 against
35.2 us -- 96 tiles of three image rows leave a third of the SMs idle, and each CTA's operand loads
(a 128 x 128 tile per 64-deep K step) bound it well below the tensor core's rate.
"""
from __future__ import annotations

import os

import torch
import torch.nn.functional as F

from ._ext import kernels

__all__ = ["conv3x3", "conv3x3_ok"]

_state = {"enabled": os.environ.get("MMLTK_TC_CONV", "0") == "1"}


def conv3x3_ok(x: torch.Tensor, weight: torch.Tensor) -> bool:
    """True when the tensor-core path takes this input [B, H, W, C] and weight [N, C, 3, 3]."""
    if not (_state["enabled"] and x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 4):
        return False
    B, H, W, C = x.shape
    N = weight.shape[0]
    k = kernels()
    if not (hasattr(k, "conv3x3_tc") and C % 64 == 0 and N % 64 == 0 and x.data_ptr() % 16 == 0):
        return False
    rows = k.conv3x3_tc_rows(H, W)
    # one CTA per tile of `rows` image rows: below ~a fifth of the SMs (batch-1 inference) the
    # library convolution is faster
    return rows > 0 and B * (H // rows) >= 32


class _Conv3x3(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight):
        x = x.contiguous()
        wk = weight.to(x.dtype).permute(0, 2, 3, 1).contiguous()          # [N, 3, 3, C]
        y = kernels().conv3x3_tc(x, wk)
        ctx.save_for_backward(x, weight)
        return y

    @staticmethod
    def backward(ctx, gy):
        x, weight = ctx.saved_tensors
        gy = gy.contiguous()
        gx = gw = None
        if ctx.needs_input_grad[0]:
            # gx = conv(gy, w') with w'[c, n, dy, dx] = w[n, c, 2 - dy, 2 - dx]
            wf = weight.to(gy.dtype).flip(2, 3).permute(1, 2, 3, 0).contiguous()   # [C, 3, 3, N]
            gx = kernels().conv3x3_tc(gy, wf)
        if ctx.needs_input_grad[1]:
            gw = torch.ops.aten.convolution_backward(
                gy.permute(0, 3, 1, 2), x.permute(0, 3, 1, 2), weight.to(gy.dtype), None, [1, 1], [1, 1], [1, 1],
                False, [0, 0], 1, [False, True, False])[1].to(weight.dtype)
        return gx, gw


def conv3x3(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """y [B, H, W, N] = 3 x 3 convolution (stride 1, padding 1, no bias) of x [B, H, W, C] with
    weight [N, C, 3, 3]."""
    if conv3x3_ok(x, weight):
        return _Conv3x3.apply(x, weight)
    xc = x.permute(0, 3, 1, 2)
    return F.conv2d(xc, weight.to(xc.dtype), None, 1, 1).permute(0, 2, 3, 1)
