"""COCO-style AP over a compiled split (native evaluator,
``csrc/host/coco_eval.cpp``) with a cross-rank reduction.

Each rank can evaluate a disjoint shard of the images; :meth:`CocoEvaluator.reduce`
all-gathers the compact per-prediction match records (5 doubles each) so every
rank ends with the full-dataset metric.  The reference evaluates on rank 0 only
(`src/rfdetr/training/train.cpp:1922-1925,2135-2140`); the metric definition is
the same (see the C++ header).
"""
from __future__ import annotations

from typing import Dict, Optional, Sequence

import torch

from ..ops._ext import native

__all__ = ["CocoEvaluator"]


class CocoEvaluator:
    def __init__(self, dataset, masks: bool = False, max_dets: int = 500):
        reader = dataset.reader if hasattr(dataset, "reader") else native().DatasetReader(str(dataset))
        self.masks = masks
        self.max_dets = max_dets
        self.ev = native().CocoEvaluator(reader, masks, max_dets)

    def add(self, indices: Sequence[int], scores: torch.Tensor, labels: torch.Tensor, boxes_xyxy: torch.Tensor,
            masks: Optional[torch.Tensor] = None) -> None:
        """scores/labels [B,K], boxes [B,K,4] xyxy pixels of the compiled image, masks [B,K,H,W] (bool/uint8)."""
        self.ev.add_batch(list(int(i) for i in indices), scores, labels, boxes_xyxy,
                          masks if (self.masks and masks is not None) else None)

    def reduce(self, group=None, gather=None) -> None:
        """All-gather every rank's match records (collective: every rank calls it).  ``gather``:
        a tensor all-gather (``FusedGradSync.all_gather_tensor``: peer-memory reads over NVLink)
        used instead of the process group's object all-gather."""
        import torch.distributed as dist
        if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
            return
        for mask in ([False, True] if self.masks else [False]):
            mine = self.ev.export_matches(mask)
            if gather is not None:
                parts = gather(mine)
            else:
                parts = [None] * dist.get_world_size(group)
                dist.all_gather_object(parts, mine, group=group)
            rank = dist.get_rank(group)
            for r, t in enumerate(parts):
                if r != rank and t.numel():
                    self.ev.import_matches(t, mask)

    def summarize(self) -> Dict[str, Dict[str, float]]:
        out = {"bbox": self.ev.summarize(False)}
        if self.masks:
            out["segm"] = self.ev.summarize(True)
        return out

    @property
    def num_images(self) -> int:
        return self.ev.num_images()
