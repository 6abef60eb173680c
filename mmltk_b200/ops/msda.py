"""Multi-scale deformable attention (MSDeformAttn) as one fused op.

Reference behaviour: `MSDeformAttnImpl::forward` (`src/rfdetr/layers/model.cpp:829-871`)
computes ``softmax`` over levels x points, the sampling locations
``loc = ref_xy + off / P * ref_wh * 0.5`` and then calls the fp32 CUDA
im2col kernel (`src/rfdetr/cuda/ms_deform_im2col_cuda.cuh:481-525`) or the
``grid_sample`` reference (`model.cpp:769-804`).

Here the softmax, the location arithmetic and the bilinear sampling are ONE
sm_100a kernel that reads bf16 values directly (no fp32 upcast), and the
backward is one kernel that produces grad_value (fp32 vector reductions into a
scratch accumulator), grad of the raw offsets, grad of the attention logits
and grad of the reference boxes.  The CPU path below is the fp32 oracle.
"""
from __future__ import annotations

from typing import List, Sequence, Tuple

import torch
import torch.nn.functional as F

from ._ext import kernels

__all__ = ["msda", "msda_reference", "msda_core_reference"]


def msda_core_reference(value: torch.Tensor, shapes: Sequence[Tuple[int, int]], loc: torch.Tensor,
                        weights: torch.Tensor) -> torch.Tensor:
    """grid_sample oracle. value [B,S,H,D], loc [B,Lq,H,L,P,2] in [0,1], weights [B,Lq,H,L,P] -> [B,Lq,H*D]."""
    B, S, H, D = value.shape
    Lq, L, P = loc.shape[1], loc.shape[3], loc.shape[4]
    grids = 2.0 * loc - 1.0
    sampled = []
    start = 0
    for lvl, (h, w) in enumerate(shapes):
        v = value[:, start:start + h * w].flatten(2).transpose(1, 2).reshape(B * H, D, h, w)
        g = grids[:, :, :, lvl].transpose(1, 2).flatten(0, 1)  # [B*H, Lq, P, 2]
        sampled.append(F.grid_sample(v, g, mode="bilinear", padding_mode="zeros", align_corners=False))
        start += h * w
    s = torch.stack(sampled, dim=-2).flatten(-2)  # [B*H, D, Lq, L*P]
    a = weights.transpose(1, 2).reshape(B * H, 1, Lq, L * P)
    out = (s * a).sum(-1).view(B, H * D, Lq)
    return out.transpose(1, 2).contiguous()


def _locations(ref: torch.Tensor, offsets: torch.Tensor) -> torch.Tensor:
    # ref [B,Lq,L,4] (cx,cy,w,h) ; offsets [B,Lq,H,L,P,2]
    P = offsets.shape[4]
    r = ref[:, :, None, :, None, :]
    return r[..., :2] + offsets / P * r[..., 2:] * 0.5


def msda_reference(value, shapes, ref, offsets, attn_logits):
    """Full fused-op semantics on plain torch ops (any device, differentiable)."""
    B, Lq, H, L, P, _ = offsets.shape
    w = torch.softmax(attn_logits.float().view(B, Lq, H, L * P), -1).view(B, Lq, H, L, P)
    loc = _locations(ref.float(), offsets.float())
    return msda_core_reference(value.float(), shapes, loc, w)


class _MsdaFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, value, ref, offsets, attn_logits, shapes_t, starts_t):
        value = value.contiguous()
        ref = ref.contiguous()
        offsets = offsets.contiguous()
        attn_logits = attn_logits.contiguous()
        out = kernels().msda_fwd(value, shapes_t, starts_t, ref, offsets, attn_logits)
        ctx.save_for_backward(value, ref, offsets, attn_logits, shapes_t, starts_t)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        value, ref, offsets, attn_logits, shapes_t, starts_t = ctx.saved_tensors
        gv, gref, goff, glog = kernels().msda_bwd(grad_out.contiguous(), value, shapes_t, starts_t, ref, offsets,
                                                  attn_logits)
        return gv, gref, goff, glog, None, None


_shape_cache = {}


def _shape_tensors(shapes, device):
    key = (tuple(tuple(s) for s in shapes), device)
    t = _shape_cache.get(key)
    if t is None:
        starts = [0]
        for h, w in shapes[:-1]:
            starts.append(starts[-1] + h * w)
        t = (torch.tensor(shapes, dtype=torch.int32, device=device).view(-1, 2),
             torch.tensor(starts, dtype=torch.int32, device=device))
        _shape_cache[key] = t
    return t


def msda(value: torch.Tensor, shapes: List[Tuple[int, int]], ref: torch.Tensor, offsets: torch.Tensor,
         attn_logits: torch.Tensor) -> torch.Tensor:
    """Fused MSDeformAttn sampling.

    value [B,S,H,D] ; ref [B,Lq,L,4] (cx,cy,w,h normalised) ; offsets [B,Lq,H,L,P,2] (raw linear output) ;
    attn_logits [B,Lq,H,L*P] (raw linear output).  Returns [B,Lq,H*D] in value's dtype (fp32 on CPU).
    """
    if value.is_cuda:
        shapes_t, starts_t = _shape_tensors(shapes, value.device)
        return _MsdaFn.apply(value, ref, offsets, attn_logits, shapes_t, starts_t)
    return msda_reference(value, shapes, ref, offsets, attn_logits).to(value.dtype)
