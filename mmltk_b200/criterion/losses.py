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

import os
from typing import Callable, Dict, List, Optional

import torch
import torch.nn.functional as F

from ..config import RfDetrConfig
from ..utils.boxes import aligned_giou, aligned_iou, cxcywh_to_xyxy
from .matcher import hungarian_match, mask_cost
from .masks import mask_losses
from .targets import Targets

__all__ = ["SetCriterion"]

GAMMA = 2.0


def _dense_neg(x: torch.Tensor, coef: float) -> torch.Tensor:
    """sum(coef * sigmoid(x)^2 * softplus(x)) -- every logit treated as a negative."""
    from ..ops import dense_focal_neg
    return dense_focal_neg(x, coef)


class _DetLossFn(torch.autograd.Function):
    """Dense negative term + fused matched-pair terms of every layer: [NL, 4] =
    (dense, correction, L1, 1 - GIoU) sums.  Backward writes the logits gradients
    once (dense kernel, then the matched entries adjusted in place) and the box
    gradients by scatter -- no per-layer index / zero-fill / add chains."""

    @staticmethod
    def forward(ctx, match, tgt_boxes, labels, mode, alpha, coef, *tensors):
        from ..ops import kernels
        k = kernels()
        nl = len(tensors) // 2
        logits = [t.contiguous() for t in tensors[:nl]]
        boxes = [t.contiguous() for t in tensors[nl:]]
        dense = torch.stack([k.dense_focal_neg_fwd(x, coef) for x in logits])
        sums = k.matched_loss_fwd(logits, boxes, match, tgt_boxes, labels, mode, alpha)
        ctx.save_for_backward(match, tgt_boxes, labels, *logits, *boxes)
        ctx.cfg = (mode, alpha, coef, nl)
        return torch.cat([dense[:, None], sums], 1)

    @staticmethod
    def backward(ctx, g):
        from ..ops import kernels
        k = kernels()
        match, tgt, labels, *rest = ctx.saved_tensors
        mode, alpha, coef, nl = ctx.cfg
        logits, boxes = list(rest[:nl]), list(rest[nl:])
        g = g.float().contiguous()
        glog = [k.dense_focal_neg_bwd(x, g[i, 0], coef) for i, x in enumerate(logits)]
        gbox = [torch.zeros_like(b) for b in boxes]
        k.matched_loss_bwd(logits, boxes, match, tgt, labels, g[:, 1:].contiguous(), glog, gbox, mode, alpha)
        return (None,) * 6 + tuple(glog) + tuple(gbox)


# (dense, correction, L1, 1-GIoU) sums -> (loss_ce, loss_bbox, loss_giou) numerators
_COMBINE = [[1.0, 0.0, 0.0], [1.0, 0.0, 0.0], [0.0, 1.0, 0.0], [0.0, 0.0, 1.0]]


class SetCriterion:
    def __init__(self, cfg: RfDetrConfig, world_size: int = 1,
                 all_reduce: Optional[Callable[[torch.Tensor], torch.Tensor]] = None):
        self.cfg = cfg
        self.world_size = max(1, world_size)
        self.all_reduce = all_reduce
        self.weight_dict = cfg.loss_weight_dict()
        # fused CUDA path for the detection terms (the per-layer torch statement is the oracle)
        self.fused = os.environ.get("MMLTK_FUSED_LOSS", "1") != "0"
        self._match_full = None
        # optional int32 device word [1] that collects the GPU assignment solver's status (the
        # training engine points it at its per-step flags and raises when it is non-zero)
        self.match_status: Optional[torch.Tensor] = None

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
        self._match_full = None
        for q, idx in by_q.items():
            g = groups if q % groups == 0 else 1
            mcost = None
            if cfg.segmentation and targets.masks is not None and all(
                    ("sparse_masks" in layers[i] or "pred_masks" in layers[i]) for i in idx):
                mcost = [mask_cost(layers[i], targets, cfg.mask_ce_loss_coef, cfg.mask_dice_loss_coef,
                                   cfg.mask_point_sample_ratio) for i in idx]
            mm = hungarian_match([layers[i]["pred_logits"] for i in idx], [layers[i]["pred_boxes"] for i in idx],
                                 targets, g, cfg.set_cost_class, cfg.set_cost_bbox, cfg.set_cost_giou, mcost,
                                 status_out=self.match_status)
            for j, i in enumerate(idx):
                match[i] = mm[j]
            if len(by_q) == 1:
                self._match_full = mm          # [NL, B, G, T], layers in order
        num_boxes = self.num_boxes(targets, groups)
        n_dec = 1 + len(outputs.get("aux_outputs", []))
        if self._fused_ok(layers, by_q):
            return self._fused(layers, match, targets, num_boxes, n_dec), match
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

    # ---------------------------------------------------------------- fused path
    def _fused_ok(self, layers, by_q) -> bool:
        cfg = self.cfg
        if not self.fused or cfg.use_varifocal_loss or cfg.use_position_supervised_loss or len(by_q) != 1:
            return False
        x = layers[0]["pred_logits"]
        if not x.is_cuda or len(layers) > 16:
            return False
        from ..ops import kernels
        if not hasattr(kernels(), "matched_loss_fwd"):
            return False
        return all(l["pred_logits"].shape == x.shape and l["pred_logits"].dtype == x.dtype and
                   l["pred_boxes"].dtype == layers[0]["pred_boxes"].dtype for l in layers)

    def _fused(self, layers, match, targets, num_boxes, n_dec) -> Dict[str, torch.Tensor]:
        cfg = self.cfg
        if cfg.ia_bce_loss:
            mode, coef = 0, 1.0
        else:
            mode, coef = 1, 1.0 - cfg.focal_alpha
        nl = len(layers) if cfg.aux_loss else 1
        full = self._match_full
        mt = full[:nl] if full is not None and full.shape[0] >= nl else torch.stack(match[:nl])
        mt = mt.to(torch.int32).contiguous()
        out = _DetLossFn.apply(mt, targets.boxes.float().contiguous(), targets.labels.contiguous(), mode,
                               float(cfg.focal_alpha), coef, *[l["pred_logits"] for l in layers[:nl]],
                               *[l["pred_boxes"] for l in layers[:nl]])
        if getattr(self, "_comb_dev", None) is None or self._comb_dev.device != out.device:
            self._comb_dev = torch.tensor(_COMBINE, device=out.device, dtype=out.dtype)   # once, before capture
        per = (out @ self._comb_dev) / num_boxes                                 # [NL, 3]
        losses: Dict[str, torch.Tensor] = {"_det_per_layer": per}
        names = ("loss_ce", "loss_bbox", "loss_giou")
        suffixes = []
        for li in range(nl):
            suffix = "" if li == 0 else (f"_{li - 1}" if li < n_dec else "_enc")
            suffixes.append(suffix)
            for j, n in enumerate(names):
                losses[n + suffix] = per[li, j]
        self._fused_suffixes = suffixes
        with torch.no_grad():   # logging terms of the main layer (reference logs them per step)
            main = layers[0]
            m = self._gather(main, match[0], targets)
            rows = main["pred_logits"][m["bidx"], m["q"]]
            valid = m["valid"]
            n = valid.sum().clamp(min=1)
            losses["class_error"] = 100.0 - ((rows.argmax(-1) == m["labels"]) & valid).sum() * 100.0 / n
            losses.update(self.loss_cardinality(main, targets))
        if cfg.segmentation and targets.masks is not None:
            for li in range(nl):
                m = self._gather(layers[li], match[li], targets)
                for k, v in mask_losses(layers[li], m, targets, cfg, num_boxes).items():
                    losses[k + suffixes[li]] = v
        return losses

    def weighted(self, losses: Dict[str, torch.Tensor]) -> torch.Tensor:
        total = None
        covered = set()
        per = losses.get("_det_per_layer")
        if per is not None:
            # detection terms of every layer in one multiply-reduce
            key = (per.shape[0], per.device)
            if getattr(self, "_wmat_key", None) != key:
                w = [[self.weight_dict.get(n + s, 0.0) for n in ("loss_ce", "loss_bbox", "loss_giou")]
                     for s in self._fused_suffixes]
                self._wmat = torch.tensor(w, device=per.device, dtype=per.dtype)
                self._wmat_key = key
            total = (per * self._wmat).sum()
            covered = {n + s for s in self._fused_suffixes for n in ("loss_ce", "loss_bbox", "loss_giou")}
        for k, w in self.weight_dict.items():
            if k in losses and k not in covered:
                total = losses[k] * w if total is None else total + losses[k] * w
        if total is None:
            raise RuntimeError("criterion returned no weighted losses")
        return total
