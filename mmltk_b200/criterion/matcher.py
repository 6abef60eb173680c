"""Hungarian matcher with Group-DETR groups.

Reference: `compute_matcher_indices_for_layers` (`src/rfdetr/detection_ops.cpp:1167-1279`)
- cost = set_cost_class * (a (1-p)^2 softplus(-x) - (1-a) p^2 softplus(x))[label]
       + set_cost_bbox * L1(cxcywh) - set_cost_giou * GIoU, a = 0.25
  (`detection_ops.cpp:967-1062`, kernel `src/rfdetr/cuda/detr_ops_cuda.cu:117-152`);
- non-finite costs replaced by max finite + max |finite| + 1 (`detection_ops.cpp:412-459`);
- one LSAP per (layer, image, group) over that group's queries
  (`detection_ops.cpp:1138-1165`), indices offset by the group.

Output: ``match [NL, B, G, T] int32`` -- for target slot t of image b the
matched query index of group g in layer l (in [0, Q)), -1 if unmatched.

CUDA: one cost kernel for all layers + the warp-per-problem LSAP kernel
(nothing is copied to the host).  CPU: the same cost in torch ops + the C++
solver on the worker pool.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch
import torch.nn.functional as F

from ..ops._ext import kernels, native
from ..utils.boxes import cxcywh_to_xyxy, generalized_box_iou
from .targets import Targets

__all__ = ["matcher_cost_reference", "hungarian_match", "mask_cost"]

FOCAL_ALPHA = 0.25


def matcher_cost_reference(logits: Sequence[torch.Tensor], boxes: Sequence[torch.Tensor], targets: Targets,
                           w_class: float, w_bbox: float, w_giou: float) -> torch.Tensor:
    """[NL, B, Q, T] fp32 cost with torch ops (CPU oracle)."""
    out = []
    T = targets.slots
    for lg, bx in zip(logits, boxes):
        x = lg.float()
        B, Q, C = x.shape
        lab = targets.labels.clamp(0, C - 1)                       # [B,T]
        xs = torch.gather(x, 2, lab[:, None, :].expand(B, Q, T))   # [B,Q,T]
        p = xs.sigmoid()
        a = FOCAL_ALPHA
        cls = a * (1 - p) ** 2 * F.softplus(-xs) - (1 - a) * p ** 2 * F.softplus(xs)
        pb = bx.float()
        l1 = (pb[:, :, None, :] - targets.boxes[:, None, :, :]).abs().sum(-1)
        giou = torch.stack([generalized_box_iou(cxcywh_to_xyxy(pb[b]), cxcywh_to_xyxy(targets.boxes[b]))
                            for b in range(B)])
        c = w_class * cls + w_bbox * l1 - w_giou * giou
        valid = targets.valid()[:, None, :]
        out.append(torch.where(valid, c, torch.zeros_like(c)))
    return torch.stack(out)


def mask_cost(layer: dict, targets: Targets, ce_coef: float, dice_coef: float, ratio: int) -> torch.Tensor:
    """[B, Q, T] mask matching cost (reference `detection_ops.cpp:1085-1136`): one random point set
    per call, shared by every query; predicted logits sampled at the points (bilinear, from the
    sparse head form: sampled spatial features x query features + bias), target masks sampled
    nearest; sigmoid-CE and dice costs as GEMMs over the point axis (K5 in GEMM form)."""
    from .masks import point_sample
    with torch.no_grad():
        if "sparse_masks" in layer:
            spatial, query, bias = layer["sparse_masks"]                # [B,C,h,w], [B,Q,C], [1]
            B, Cf, h, w = spatial.shape
            P = max(1, h * w // ratio)
            pts = torch.rand(1, P, 2, device=spatial.device)
            feat = point_sample(spatial.float(), pts.expand(B, P, 2))   # [B, C, P]
            x = torch.bmm(query.float(), feat) + bias.float()            # [B, Q, P]
        else:
            pm = layer["pred_masks"]                                     # [B, Q, h, w]
            B, Q, h, w = pm.shape
            P = max(1, h * w // ratio)
            pts = torch.rand(1, P, 2, device=pm.device)
            x = point_sample(pm.float().flatten(0, 1)[:, None], pts.expand(B * Q, P, 2))[:, 0].view(B, Q, P)
        T = targets.slots
        offs = torch.as_tensor(targets.mask_offsets, device=x.device)
        rows = (offs[:, None] + torch.arange(T, device=x.device)[None]).clamp(max=max(0, targets.masks.shape[0] - 1))
        tm = targets.masks[rows.reshape(-1)].float()[:, None]           # [B*T, 1, Hm, Wm]
        t = point_sample(tm, pts.expand(B * T, P, 2), mode="nearest")[:, 0].view(B, T, P)
        pos, neg = F.softplus(-x), F.softplus(x)
        ce = (torch.bmm(pos, t.transpose(1, 2)) + torch.bmm(neg, (1 - t).transpose(1, 2))) / P
        sig = x.sigmoid()
        num = 2 * torch.bmm(sig, t.transpose(1, 2))
        den = sig.sum(-1)[:, :, None] + t.sum(-1)[:, None, :]
        dice = 1 - (num + 1) / (den + 1)
        return ce_coef * ce + dice_coef * dice


def hungarian_match(logits: List[torch.Tensor], boxes: List[torch.Tensor], targets: Targets, groups: int,
                    w_class: float = 2.0, w_bbox: float = 5.0, w_giou: float = 2.0, mask_costs=None,
                    status_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """mask_costs: optional list (one per layer) of [B, Q, T] costs added before the assignment.

    status_out: optional int32 device tensor [1]; the GPU solver's status word (non-zero when a
    bounded augmenting-path search gave up and the assignment is partial) is OR-ed into it on the
    device, so a caller can check it once per step without a host sync here."""
    with torch.no_grad():
        dev = logits[0].device
        if dev.type == "cuda":   # cost build + batched LSAP on the device (any target / query ratio)
            k = kernels()
            cost = k.matcher_cost([l.detach() for l in logits], [b.detach() for b in boxes], targets.labels,
                                  targets.boxes, targets.counts, w_class, w_bbox, w_giou, FOCAL_ALPHA)
            if mask_costs is not None:
                cost += torch.stack(mask_costs).to(cost.dtype)
            match, status = k.lsap_batched(cost, targets.counts, groups)
            if status_out is not None:
                status_out.bitwise_or_(status)
            return match
        cost = matcher_cost_reference(logits, boxes, targets, w_class, w_bbox, w_giou)
        if mask_costs is not None:
            cost = cost + torch.stack(mask_costs).float()
        m = native().match_batched(cost.cpu(), targets.counts.cpu().to(torch.int64), groups)
        return m.to(dev)
