"""Box utilities (reference `src/rfdetr/detection_ops.cpp:630-713`)."""
from __future__ import annotations

import torch

__all__ = ["cxcywh_to_xyxy", "xyxy_to_cxcywh", "box_iou", "generalized_box_iou", "aligned_iou", "aligned_giou"]


def cxcywh_to_xyxy(b: torch.Tensor) -> torch.Tensor:
    cx, cy, w, h = b.unbind(-1)
    return torch.stack([cx - 0.5 * w, cy - 0.5 * h, cx + 0.5 * w, cy + 0.5 * h], -1)


def xyxy_to_cxcywh(b: torch.Tensor) -> torch.Tensor:
    x0, y0, x1, y1 = b.unbind(-1)
    return torch.stack([(x0 + x1) / 2, (y0 + y1) / 2, x1 - x0, y1 - y0], -1)


def _area(b):
    return (b[..., 2] - b[..., 0]).clamp(min=0) * (b[..., 3] - b[..., 1]).clamp(min=0)


def box_iou(a: torch.Tensor, b: torch.Tensor):
    """Pairwise IoU of xyxy boxes [N,4] x [M,4] -> (iou [N,M], union [N,M])."""
    area_a, area_b = _area(a), _area(b)
    lt = torch.max(a[:, None, :2], b[None, :, :2])
    rb = torch.min(a[:, None, 2:], b[None, :, 2:])
    wh = (rb - lt).clamp(min=0)
    inter = wh[..., 0] * wh[..., 1]
    union = area_a[:, None] + area_b[None, :] - inter
    return inter / union, union


def generalized_box_iou(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    iou, union = box_iou(a, b)
    lt = torch.min(a[:, None, :2], b[None, :, :2])
    rb = torch.max(a[:, None, 2:], b[None, :, 2:])
    wh = (rb - lt).clamp(min=0)
    area = wh[..., 0] * wh[..., 1]
    return iou - (area - union) / area


def _aligned_inter_union(a, b):
    lt = torch.max(a[..., :2], b[..., :2])
    rb = torch.min(a[..., 2:], b[..., 2:])
    wh = (rb - lt).clamp(min=0)
    inter = wh[..., 0] * wh[..., 1]
    union = _area(a) + _area(b) - inter
    return inter, union


def aligned_iou(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    inter, union = _aligned_inter_union(a, b)
    return inter / union


def aligned_giou(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    inter, union = _aligned_inter_union(a, b)
    iou = inter / union
    lt = torch.min(a[..., :2], b[..., :2])
    rb = torch.max(a[..., 2:], b[..., 2:])
    wh = (rb - lt).clamp(min=0)
    area = wh[..., 0] * wh[..., 1]
    return iou - (area - union) / area
