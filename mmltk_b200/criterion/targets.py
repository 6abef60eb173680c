"""Padded, static-shape detection targets.

The reference keeps a ragged list of per-image targets (`PreparedTargets`,
`include/mmltk/rfdetr/detection_types.h`).  Here every batch is padded to a
fixed number of target slots ``T`` so that matcher and losses have static
shapes (no host sync, CUDA-graph friendly): ``boxes [B,T,4]`` (normalised
cxcywh), ``labels [B,T]`` and ``counts [B]``.  Padding slots hold a harmless
dummy box so that no masked-out computation can produce NaN.
"""
from __future__ import annotations

import dataclasses
from typing import List, Optional, Sequence

import torch

__all__ = ["Targets", "pad_targets", "PAD_BOX"]

PAD_BOX = (0.5, 0.5, 0.25, 0.25)


@dataclasses.dataclass
class Targets:
    boxes: torch.Tensor          # [B, T, 4] fp32 cxcywh normalised
    labels: torch.Tensor         # [B, T] int64
    counts: torch.Tensor         # [B] int32 (same device as boxes)
    counts_host: List[int]
    masks: Optional[torch.Tensor] = None        # [sum(counts), Hm, Wm] bool (segmentation), image-major
    mask_offsets: Optional[List[int]] = None    # first mask row of each image

    @property
    def batch(self) -> int:
        return self.boxes.shape[0]

    @property
    def slots(self) -> int:
        return self.boxes.shape[1]

    def valid(self) -> torch.Tensor:
        t = torch.arange(self.slots, device=self.boxes.device)
        return t[None, :] < self.counts[:, None].to(t.dtype)

    def to(self, device, non_blocking: bool = False) -> "Targets":
        return Targets(self.boxes.to(device, non_blocking=non_blocking),
                       self.labels.to(device, non_blocking=non_blocking),
                       self.counts.to(device, non_blocking=non_blocking), list(self.counts_host),
                       None if self.masks is None else self.masks.to(device, non_blocking=non_blocking),
                       self.mask_offsets)

    def total(self) -> int:
        return int(sum(self.counts_host))


def pad_targets(per_image: Sequence[dict], slots: Optional[int] = None, device=None) -> Targets:
    """per_image: list of {"boxes": [n,4] cxcywh, "labels": [n], optional "masks": [n,H,W] bool}."""
    counts = [int(t["boxes"].shape[0]) for t in per_image]
    T = max(1, slots if slots is not None else max(counts + [1]))
    if max(counts + [0]) > T:
        raise ValueError(f"an image has {max(counts)} targets, more than the {T} slots")
    B = len(per_image)
    boxes = torch.tensor(PAD_BOX, dtype=torch.float32).repeat(B, T, 1)
    labels = torch.zeros(B, T, dtype=torch.int64)
    masks = []
    offsets = []
    off = 0
    for i, t in enumerate(per_image):
        n = counts[i]
        if n:
            boxes[i, :n] = torch.as_tensor(t["boxes"], dtype=torch.float32)
            labels[i, :n] = torch.as_tensor(t["labels"], dtype=torch.int64)
        offsets.append(off)
        if "masks" in t and t["masks"] is not None:
            masks.append(torch.as_tensor(t["masks"], dtype=torch.bool))
            off += n
    m = torch.cat(masks, 0) if masks else None
    tg = Targets(boxes, labels, torch.tensor(counts, dtype=torch.int32), counts, m, offsets if masks else None)
    return tg.to(device) if device is not None else tg
