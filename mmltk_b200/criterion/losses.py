"""Set criterion: matcher + classification / box / mask losses for every
supervised layer (reference `detection_loss_dict` / `weighted_detection_loss`,
`src/rfdetr/detection_ops.cpp:1303-1597`).

All loss terms are computed from the static-shape match table, so nothing
here synchronises with the host.  The classification losses are split into a
dense term over every (image, query, class) logit -- the value every logit
would have if it were a negative -- plus a correction on the matched
(image, query, label) entries.  This is exactly the reference's formula
(e.g. IA-BCE ``sum(neg*x - logsigmoid(x)*(pos+neg)) / num_boxes`` with
``pos = t``, ``neg = 1 - t`` on matched entries and ``pos = 0``,
``neg = sigmoid(x)^2`` elsewhere, `detection_ops.cpp:1324-1342`) without
materialising the [B, Q, C] weight tensors.
"""
from __future__ import annotations

from typing import Callable, Dict, List, Optional

import torch
import torch.nn.functional as F

from ..config import RfDetrConfig
from ..utils.boxes import aligned_giou, aligned_iou, cxcywh_to_xyxy
from .matcher import hungarian_match
from .masks import mask_losses
from .targets import Targets

__all__ = ["SetCriterion"]

GAMMA = 2.0


def _dense_neg(x: torch.Tensor, coef: float) -> torch.Tensor:
    """sum(coef * sigmoid(x)^2 * softplus(x)) -- every logit treated as a negative."""
    from ..ops import dense_focal_neg
    return dense_focal_neg(x, coef)


class SetCriterion:
    def __init__(self, cfg: RfDetrConfig, world_size: int = 1,
                 all_reduce: Optional[Callable[[torch.Tensor], torch.Tensor]] = None):
        self.cfg = cfg
        self.world_size = max(1, world_size)
        self.all_reduce = all_reduce
        self.weight_dict = cfg.loss_weight_dict()

    # ---------------------------------------------------------------- helpers
    def num_boxes(self, targets: Targets, groups: int) -> torch.Tensor:
        """Reference `detection_ops.cpp:1485-1510`: sum of targets (x groups), summed over
        ranks, / world size, clamped >= 1.  Stays on the device."""
        n = targets.counts.sum().float()
        if not self.cfg.sum_group_losses:
            n = n * groups
        n = n.reshape(1)
        if self.all_reduce is not None and self.world_size > 1:
            n = self.all_reduce(n)
        return (n / self.world_size).clamp(min=1.0).reshape(())

    def _gather(self, layer, match_l, targets):
        """Matched predictions of one layer: returns dict of [B,G,T,...] tensors + valid mask."""
        logits, boxes = layer["pred_logits"], layer["pred_boxes"]
        B, Q, C = logits.shape
        G, T = match_l.shape[1], match_l.shape[2]
        valid = match_l >= 0
        q = match_l.clamp(min=0).long()                                       # [B,G,T]
        bidx = torch.arange(B, device=q.device)[:, None, None].expand(B, G, T)
        src_boxes = boxes[bidx, q].float()                                    # [B,G,T,4]
        tgt_boxes = targets.boxes[:, None].expand(B, G, T, 4)
        labels = targets.labels.clamp(0, C - 1)[:, None].expand(B, G, T)
        x_m = logits[bidx, q, labels].float()                                 # [B,G,T]
        return dict(valid=valid, q=q, bidx=bidx, src_boxes=src_boxes, tgt_boxes=tgt_boxes, labels=labels, x_m=x_m)

    def loss_labels(self, layer, m, num_boxes, log: bool) -> Dict[str, torch.Tensor]:
        cfg = self.cfg
        x = layer["pred_logits"]
        valid = m["valid"]
        x_m = m["x_m"]
        alpha = cfg.focal_alpha
        zero = torch.zeros((), device=x.device)
        if cfg.ia_bce_loss:
            dense = _dense_neg(x, 1.0)
            with torch.no_grad():
                iou = aligned_iou(cxcywh_to_xyxy(m["src_boxes"]), cxcywh_to_xyxy(m["tgt_boxes"]))
                t = (torch.sigmoid(x_m) ** alpha * iou.clamp(min=0) ** (1 - alpha)).clamp(min=0.01)
            p = torch.sigmoid(x_m)
            corr = (1 - t) * x_m + F.softplus(-x_m) - p ** GAMMA * F.softplus(x_m)
            loss = (dense + torch.where(valid, corr, zero).sum()) / num_boxes
        elif cfg.use_position_supervised_loss or cfg.use_varifocal_loss:
            dense = _dense_neg(x, 1 - alpha)
            with torch.no_grad():
                iou = aligned_iou(cxcywh_to_xyxy(m["src_boxes"]), cxcywh_to_xyxy(m["tgt_boxes"]))
                iou = torch.where(valid, iou, zero)
                if cfg.use_position_supervised_loss:
                    per_img = iou.flatten(1).amax(1)[:, None, None]
                    tt = iou / (per_img + 1e-8)
                else:
                    tt = iou
            p = torch.sigmoid(x_m)
            bce = F.softplus(x_m) - tt * x_m
            if cfg.use_position_supervised_loss:
                pos = alpha * bce * (tt - p).abs() ** GAMMA
            else:
                pos = tt * bce
            neg = (1 - alpha) * p ** GAMMA * F.softplus(x_m)
            corr = torch.where(valid & (tt > 0), pos - neg, zero)
            loss = (dense + corr.sum()) / num_boxes
        else:  # sigmoid focal
            dense = _dense_neg(x, 1 - alpha)
            p = torch.sigmoid(x_m)
            pos = alpha * F.softplus(-x_m) * (1 - p) ** GAMMA
            neg = (1 - alpha) * p ** GAMMA * F.softplus(x_m)
            loss = (dense + torch.where(valid, pos - neg, zero).sum()) / num_boxes
        out = {"loss_ce": loss}
        if log:
            with torch.no_grad():
                rows = x[m["bidx"], m["q"]]                                   # [B,G,T,C]
                correct = (rows.argmax(-1) == m["labels"]) & valid
                n = valid.sum().clamp(min=1)
                out["class_error"] = 100.0 - correct.sum() * 100.0 / n
        return out

    def loss_boxes(self, m, num_boxes) -> Dict[str, torch.Tensor]:
        valid = m["valid"]
        zero = torch.zeros((), device=valid.device)
        l1 = (m["src_boxes"] - m["tgt_boxes"]).abs().sum(-1)
        giou = aligned_giou(cxcywh_to_xyxy(m["src_boxes"]), cxcywh_to_xyxy(m["tgt_boxes"]))
        return {"loss_bbox": torch.where(valid, l1, zero).sum() / num_boxes,
                "loss_giou": torch.where(valid, 1 - giou, zero).sum() / num_boxes}

    @staticmethod
    def loss_cardinality(layer, targets) -> Dict[str, torch.Tensor]:
        with torch.no_grad():
            lg = layer["pred_logits"]
            card = (lg.argmax(-1) != lg.shape[-1] - 1).sum(1).float()
            return {"cardinality_error": (card - targets.counts.float()).abs().mean()}

    # ---------------------------------------------------------------- main
    def __call__(self, outputs: Dict, targets: Targets, training: bool = True):
        from ..models.rfdetr import RFDETR
        cfg = self.cfg
        groups = max(1, cfg.group_detr) if training else 1
        layers = RFDETR.supervised_layers(outputs)
        # layers with the same query count are matched in one batched call (normally all of them;
        # the two-stage layer has fewer queries only when the feature map has fewer tokens than queries)
        match: List[torch.Tensor] = [None] * len(layers)
        by_q: Dict[int, List[int]] = {}
        for i, l in enumerate(layers):
            by_q.setdefault(l["pred_logits"].shape[1], []).append(i)
        for q, idx in by_q.items():
            g = groups if q % groups == 0 else 1
            mm = hungarian_match([layers[i]["pred_logits"] for i in idx], [layers[i]["pred_boxes"] for i in idx],
                                 targets, g, cfg.set_cost_class, cfg.set_cost_bbox, cfg.set_cost_giou)
            for j, i in enumerate(idx):
                match[i] = mm[j]
        num_boxes = self.num_boxes(targets, groups)
        n_dec = 1 + len(outputs.get("aux_outputs", []))
        losses: Dict[str, torch.Tensor] = {}
        for li, layer in enumerate(layers):
            if li == 0:
                suffix = ""
            elif li < n_dec:
                suffix = f"_{li - 1}"
            else:
                suffix = "_enc"
            if li > 0 and not cfg.aux_loss:
                break
            m = self._gather(layer, match[li], targets)
            part = {}
            part.update(self.loss_labels(layer, m, num_boxes, log=(li == 0)))
            part.update(self.loss_cardinality(layer, targets))
            part.update(self.loss_boxes(m, num_boxes))
            if cfg.segmentation and targets.masks is not None:
                part.update(mask_losses(layer, m, targets, cfg, num_boxes))
            for k, v in part.items():
                losses[k + suffix] = v
        return losses, match

    def weighted(self, losses: Dict[str, torch.Tensor]) -> torch.Tensor:
        total = None
        for k, w in self.weight_dict.items():
            if k in losses:
                total = losses[k] * w if total is None else total + losses[k] * w
        if total is None:
            raise RuntimeError("criterion returned no weighted losses")
        return total
