"""Mask losses for the segmentation presets (reference
`src/rfdetr/detection_ops.cpp:550-625,1394-1441`).

For every matched (image, query, target): mask logits are rebuilt from the
sparse head output (spatial features . query features + bias), points are
chosen by uncertainty (3x oversampling, 75% most uncertain |logit| + 25%
uniform), logits are bilinearly point-sampled (align_corners=False), target
masks are sampled at the same points (nearest), and
``loss_mask_ce = mean-over-points BCE`` and
``loss_mask_dice = 1 - (2 sum(p t) + 1) / (sum p + sum t + 1)`` are summed over
matches and divided by num_boxes.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ..ops._ext import kernels

__all__ = ["point_sample", "point_sample_reference", "uncertain_point_coords", "mask_losses"]


def point_sample_reference(inp: torch.Tensor, coords: torch.Tensor, mode: str = "bilinear") -> torch.Tensor:
    """``grid_sample`` form (zero padding, align_corners=False): the CPU path and test oracle."""
    grid = 2.0 * coords[:, :, None, :] - 1.0
    return F.grid_sample(inp, grid.to(inp.dtype), mode=mode, padding_mode="zeros", align_corners=False)[..., 0]


class _PointSampleFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, inp, coords):
        ctx.save_for_backward(coords)
        ctx.hw = (inp.shape[-2], inp.shape[-1])
        ctx.dtype = inp.dtype
        return kernels().point_sample(inp, coords)

    @staticmethod
    def backward(ctx, g):
        (coords,) = ctx.saved_tensors
        gin = kernels().point_sample_bwd(g, coords, ctx.hw[0], ctx.hw[1])
        return gin.to(ctx.dtype), None


def point_sample(inp: torch.Tensor, coords: torch.Tensor, mode: str = "bilinear") -> torch.Tensor:
    """inp [N,C,H,W], coords [N,P,2] in [0,1] (x, y) -> [N,C,P].  Bilinear on CUDA runs the
    point-sample kernel (one thread per output, 4-corner atomics in backward)."""
    if mode == "bilinear" and inp.is_cuda and inp.dtype in (torch.float32, torch.bfloat16):
        return _PointSampleFn.apply(inp, coords)
    return point_sample_reference(inp, coords, mode)


def uncertain_point_coords(logits: torch.Tensor, num_points: int, oversample: int = 3,
                           importance: float = 0.75) -> torch.Tensor:
    N = logits.shape[0]
    ns = num_points * oversample
    coords = torch.rand(N, ns, 2, device=logits.device)
    pl = point_sample(logits, coords)                          # [N,1,ns]
    unc = -pl[:, 0].abs()
    nu = int(importance * num_points)
    parts = []
    if nu > 0:
        idx = unc.topk(nu, dim=1)[1]
        parts.append(torch.gather(coords, 1, idx[..., None].expand(-1, -1, 2)))
    if num_points - nu > 0:
        parts.append(torch.rand(N, num_points - nu, 2, device=logits.device))
    return torch.cat(parts, 1)


def _matched_mask_logits(layer, m):
    valid = m["valid"]
    bidx, q = m["bidx"], m["q"]
    if "sparse_masks" in layer:
        spatial, query, bias = layer["sparse_masks"]            # [B,C,h,w], [B,Q,C], [1]
        qf = query[bidx, q]                                     # [B,G,T,C]
        B, G, T, C = qf.shape
        sp = spatial[bidx.reshape(-1)]                          # [N,C,h,w]
        logits = torch.einsum("nchw,nc->nhw", sp, qf.reshape(-1, C)) + bias.to(sp.dtype)
    else:
        pm = layer["pred_masks"]                                # [B,Q,h,w]
        logits = pm[bidx, q].reshape(-1, pm.shape[-2], pm.shape[-1])
    return logits[:, None].float(), valid.reshape(-1)


def mask_losses(layer, m, targets, cfg, num_boxes):
    src, valid = _matched_mask_logits(layer, m)                 # [N,1,h,w]
    N, _, h, w = src.shape
    npts = max(h, h * w // cfg.mask_point_sample_ratio)
    with torch.no_grad():
        coords = uncertain_point_coords(src, npts)
    logits = point_sample(src, coords)[:, 0]                    # [N,P]
    with torch.no_grad():
        # target mask rows: image b's masks start at mask_offsets[b]
        offs = torch.as_tensor(targets.mask_offsets, device=src.device)
        B, G, T = m["valid"].shape
        t_idx = torch.arange(T, device=src.device)[None, None, :].expand(B, G, T)
        rows = (offs[:, None, None] + t_idx).reshape(-1).clamp(max=max(0, targets.masks.shape[0] - 1))
        Hm, Wm = targets.masks.shape[-2:]
        if src.is_cuda:
            # target masks bit-packed once, then sampled (nearest) at the points: no dense float copies
            bits = kernels().pack_masks(targets.masks)[rows]
            labels = kernels().sample_packed_masks(bits, Hm, Wm, coords)
        else:
            tm = targets.masks[rows].float()[:, None]           # [N,1,Hm,Wm]
            labels = point_sample_reference(tm, coords, mode="nearest")[:, 0]
    zero = torch.zeros((), device=src.device)
    ce = F.binary_cross_entropy_with_logits(logits, labels, reduction="none").mean(1)
    p = logits.sigmoid()
    dice = 1 - (2 * (p * labels).sum(-1) + 1) / (p.sum(-1) + labels.sum(-1) + 1)
    return {"loss_mask_ce": torch.where(valid, ce, zero).sum() / num_boxes,
            "loss_mask_dice": torch.where(valid, dice, zero).sum() / num_boxes}
