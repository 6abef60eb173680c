"""RF-DETR detector (counterpart of `NativeRfDetrModel`, reference
`src/rfdetr/layers/model.cpp:1643-1921`).

Module tree (= state-dict key layout of the official checkpoints):
``backbone.0.encoder.encoder.*`` (windowed DINOv2), ``backbone.0.projector.*``,
``transformer.*``, ``class_embed``, ``bbox_embed.layers.*``,
``refpoint_embed``, ``query_feat``, optional ``segmentation_head.*``.

Outputs (training and eval) are a dict:
``pred_logits`` [B,Q,K], ``pred_boxes`` [B,Q,4] (cxcywh, normalised),
``aux_outputs`` (list of dicts, decoder layers 0..L-2), ``enc_outputs`` (two-stage
proposals) and, for segmentation, ``pred_masks`` (eval, dense) or
``sparse_masks`` (training).  ``layers`` lists every supervised layer in the
matcher order of the reference (main, aux..., enc).
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional

import torch
import torch.nn as nn

from .. import ops
from ..config import RfDetrConfig, config_from_preset
from .backbone import DinoV2Wrapper
from .projector import MultiScaleProjector
from .segmentation import SegmentationHead
from .transformer import Mlp, Transformer, reparam_boxes

__all__ = ["RFDETR", "build_model"]


class PositionEmbeddingSine(nn.Module):
    """Parameter-free sine position embedding (reference `src/rfdetr/layers/modules.cpp:96-227`).

    The decoder of the reference computes it but never consumes it (the
    ``pos`` argument of `NativeDecoderImpl::forward` is unused), so the model
    only provides it for API parity."""

    def __init__(self, num_pos_feats=128, temperature=10000.0, normalize=True, scale=2 * math.pi):
        super().__init__()
        self.num_pos_feats, self.temperature, self.normalize, self.scale = num_pos_feats, temperature, normalize, scale
        self._cache = {}

    def full_valid(self, batch: int, h: int, w: int, device) -> torch.Tensor:
        key = (h, w, str(device))
        base = self._cache.get(key)
        if base is None:
            y = torch.arange(1, h + 1, dtype=torch.float32, device=device).view(1, h, 1).expand(1, h, w)
            x = torch.arange(1, w + 1, dtype=torch.float32, device=device).view(1, 1, w).expand(1, h, w)
            if self.normalize:
                y = y / (h + 1e-6) * self.scale
                x = x / (w + 1e-6) * self.scale
            d = torch.arange(self.num_pos_feats, dtype=torch.float32, device=device)
            d = self.temperature ** (2 * torch.div(d, 2, rounding_mode="floor") / self.num_pos_feats)
            px, py = x[..., None] / d, y[..., None] / d
            px = torch.stack((px[..., 0::2].sin(), px[..., 1::2].cos()), 4).flatten(3)
            py = torch.stack((py[..., 0::2].sin(), py[..., 1::2].cos()), 4).flatten(3)
            base = torch.cat((py, px), 3).permute(0, 3, 1, 2).contiguous()
            self._cache[key] = base
        return base.expand(batch, -1, h, w)


class Backbone(nn.Module):
    """`backbone.0`: DINOv2 encoder + projector."""

    def __init__(self, cfg: RfDetrConfig):
        super().__init__()
        self.encoder = DinoV2Wrapper(cfg)
        self.projector = MultiScaleProjector(cfg.vit_width, len(cfg.out_feature_indexes), cfg.hidden_dim,
                                             cfg.projector_levels, cfg.projector_blocks)

    def forward(self, pixels):
        return self.projector(self.encoder(pixels))


class RFDETR(nn.Module):
    def __init__(self, cfg: RfDetrConfig):
        super().__init__()
        cfg.validate()
        self.cfg = cfg
        Q = max(1, cfg.num_queries * max(1, cfg.group_detr))
        self.backbone = nn.ModuleList([Backbone(cfg), PositionEmbeddingSine(cfg.hidden_dim // 2)])
        self.transformer = Transformer(cfg)
        self.class_embed = nn.Linear(cfg.hidden_dim, max(1, cfg.num_classes))
        self.bbox_embed = Mlp(cfg.hidden_dim, cfg.hidden_dim, 4, 3)
        self.refpoint_embed = nn.Embedding(Q, 4)
        self.query_feat = nn.Embedding(Q, cfg.hidden_dim)
        self.segmentation_head = SegmentationHead(cfg.hidden_dim, max(1, cfg.dec_layers)) if cfg.segmentation else None
        with torch.no_grad():
            self.refpoint_embed.weight.zero_()
            self.class_embed.bias.fill_(-math.log((1 - 0.01) / 0.01))
            self.bbox_embed.layers[-1].weight.zero_()
            self.bbox_embed.layers[-1].bias.zero_()

    # ------------------------------------------------------------------ data-parallel buckets
    @staticmethod
    def grad_stage(name: str) -> int:
        """Backward-completion stage of a parameter (see ``backbone.grad_stage``)."""
        from .backbone import grad_stage
        return grad_stage(name)

    def grad_mark_count(self) -> int:
        """Number of gradient marks one backward pass raises (one per ViT layer input)."""
        return len(self.backbone[0].encoder.encoder.encoder.layer)

    def set_grad_marks(self, cb) -> None:
        """``cb(i)`` is called during backward when the gradient reaches ViT layer i's input
        (None: no marks)."""
        self.backbone[0].encoder.encoder.grad_marks = cb

    # ------------------------------------------------------------------ forward
    def forward(self, pixels: torch.Tensor, include_masks: bool = True) -> Dict:
        cfg = self.cfg
        training = self.training
        B, _, H, W = pixels.shape
        feats = self.backbone[0](pixels)  # channels-last per level
        nq = cfg.num_queries * max(1, cfg.group_detr) if training else cfg.num_queries
        # the full tables when every query is used (a full-range slice's backward zero-fills + copies)
        ref_w, qf_w = self.refpoint_embed.weight, self.query_feat.weight
        if nq != ref_w.shape[0]:
            ref_w, qf_w = ref_w[:nq], qf_w[:nq]
        t = self.transformer(feats, ref_w, qf_w, training,
                             bbox_embed=None if cfg.lite_refpoint_refine else self.bbox_embed)
        hs = t["hs"]                      # [Ldec, B, Q, C]
        refs = t["refs"]                  # [1 or Ldec, B, Q, 4]
        logits = ops.linear(hs, self.class_embed.weight, self.class_embed.bias)
        delta = self.bbox_embed(hs)
        if cfg.bbox_reparam:
            boxes = reparam_boxes(delta, refs)
        else:
            boxes = (delta + refs).sigmoid()
        L = hs.shape[0]
        lg, bx = logits.unbind(0), boxes.unbind(0)   # one backward node per tensor (no per-layer zero fill)
        out = {"pred_logits": lg[L - 1], "pred_boxes": bx[L - 1],
               "aux_outputs": [{"pred_logits": lg[i], "pred_boxes": bx[i]} for i in range(L - 1)]}
        groups = max(1, cfg.group_detr) if training else 1
        if cfg.two_stage and "enc_memory" in t:
            enc_logits = self.transformer.encoder_class_logits(t["enc_memory"], groups)
            out["enc_outputs"] = {"pred_logits": enc_logits, "pred_boxes": t["enc_boxes"]}
        if self.segmentation_head is not None and include_masks:
            spatial = feats[0].permute(0, 3, 1, 2)
            queries = [hs[i] for i in range(L)]
            if training:
                sp = self.segmentation_head.sparse_forward(spatial, queries, (H, W))
                for i in range(L - 1):
                    out["aux_outputs"][i]["sparse_masks"] = sp[i]
                out["sparse_masks"] = sp[L - 1]
                if "enc_outputs" in out:
                    out["enc_outputs"]["sparse_masks"] = self.segmentation_head.sparse_forward(
                        spatial, [t["enc_memory"]], (H, W), skip_blocks=True)[0]
            else:
                dense = self.segmentation_head(spatial, queries, (H, W))
                for i in range(L - 1):
                    out["aux_outputs"][i]["pred_masks"] = dense[i]
                out["pred_masks"] = dense[L - 1]
                if "enc_outputs" in out:
                    out["enc_outputs"]["pred_masks"] = self.segmentation_head(
                        spatial, [t["enc_memory"]], (H, W), skip_blocks=True)[0]
        return out

    @staticmethod
    def supervised_layers(out: Dict) -> List[Dict]:
        """Layers in the reference's matcher order: main, aux 0..L-2, enc."""
        main = {k: v for k, v in out.items() if k not in ("aux_outputs", "enc_outputs")}
        layers = [main] + list(out.get("aux_outputs", []))
        if "enc_outputs" in out:
            layers.append(out["enc_outputs"])
        return layers

    # ------------------------------------------------------------ class resize
    def reinitialize_detection_head(self, num_classes: int) -> None:
        """Resize class heads by repeating rows (reference `model.cpp:208-232,1675-1687`)."""

        def resize(t):
            if t.shape[0] == num_classes:
                return t.detach().clone()
            reps = max(1, -(-num_classes // t.shape[0]))
            return t.detach().repeat(reps, *([1] * (t.dim() - 1)))[:num_classes].contiguous()

        with torch.no_grad():
            ce = self.class_embed
            new = nn.Linear(ce.in_features, num_classes, device=ce.weight.device, dtype=ce.weight.dtype)
            new.weight.copy_(resize(ce.weight))
            new.bias.copy_(resize(ce.bias))
            self.class_embed = new
            g = self.transformer.enc_out_class_embed
            w = torch.stack([resize(g.weight[i]) for i in range(g.groups)])
            b = torch.stack([resize(g.bias[i]) for i in range(g.groups)])
            g.weight = nn.Parameter(w)
            g.bias = nn.Parameter(b)
        self.cfg.num_classes = num_classes


def build_model(preset: str = "rf-detr-medium", **overrides) -> RFDETR:
    return RFDETR(config_from_preset(preset, **overrides))
