"""Detection post-process: top-k over the flattened query x class scores,
labels, xyxy pixel boxes and (segmentation) binary masks.

Reference: `src/rfdetr/inference/postprocess.cpp:19-238`.  On CUDA the
selection, sigmoid, box conversion and scaling are one kernel
(``csrc/kernels/postprocess.cu``); the masks of the selected queries are
bilinearly resized to the image and thresholded at 0.
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch
import torch.nn.functional as F

from ..ops._ext import kernels

__all__ = ["postprocess", "postprocess_reference"]


def postprocess_reference(logits: torch.Tensor, boxes: torch.Tensor, k: int, size: Tuple[int, int]) -> Dict:
    """Plain torch statement (CPU path and test oracle).  Ties: lowest flat index first."""
    B, Q, C = logits.shape
    flat = logits.float().reshape(B, Q * C)
    # stable descending order: sort by (-value, index)
    order = torch.sort(flat, dim=1, descending=True, stable=True).indices[:, :k]
    scores = flat.gather(1, order).sigmoid()
    q = torch.div(order, C, rounding_mode="floor")
    labels = order % C
    bx = boxes.float().gather(1, q[..., None].expand(-1, -1, 4))
    cx, cy, w, h = bx.unbind(-1)
    w, h = w.clamp(min=0), h.clamp(min=0)
    H, W = size
    xyxy = torch.stack([(cx - 0.5 * w) * W, (cy - 0.5 * h) * H, (cx + 0.5 * w) * W, (cy + 0.5 * h) * H], -1)
    return {"scores": scores, "labels": labels, "boxes": xyxy, "queries": q.to(torch.int32)}


def postprocess(out: Dict, k: int, size: Tuple[int, int], masks: bool = True,
                mask_size: Optional[Tuple[int, int]] = None) -> Dict:
    logits, boxes = out["pred_logits"], out["pred_boxes"]
    k = min(k, logits.shape[1] * logits.shape[2])
    if logits.is_cuda:
        s, l, b, q = kernels().topk_postprocess(logits, boxes, k, None, float(size[0]), float(size[1]))
        res = {"scores": s, "labels": l, "boxes": b, "queries": q}
    else:
        res = postprocess_reference(logits, boxes, k, size)
    if masks and "pred_masks" in out:
        pm = out["pred_masks"]                                           # [B,Q,h,w]
        q = res["queries"].long()
        sel = pm.gather(1, q[..., None, None].expand(-1, -1, pm.shape[-2], pm.shape[-1]))
        up = F.interpolate(sel.float(), size=mask_size or size, mode="bilinear", align_corners=False)
        res["masks"] = up > 0
    return res
