"""Model / loss configuration (counterpart of `NativeRfDetrConfig`,
reference `include/mmltk/rfdetr/artifacts.h:11-46`, built from a preset by
`make_config_from_preset`, `src/rfdetr/layers/model.cpp:1374-1401`).

Unlike the reference, the backbone width/depth/heads, the tapped stages and
the projector levels are configuration, not constants, so that a ViT-B
backbone with a P3+P5 projector can be built from the same code.
"""
from __future__ import annotations

import dataclasses
from typing import Optional

from .presets import PresetSpec, find_preset

__all__ = ["RfDetrConfig", "config_from_preset"]


@dataclasses.dataclass
class RfDetrConfig:
    preset_name: str = "rf-detr-nano"
    resolution: int = 384
    segmentation: bool = False
    num_classes: int = 91
    num_queries: int = 300
    num_select: int = 300
    dec_layers: int = 2
    group_detr: int = 13
    two_stage: bool = True
    hidden_dim: int = 256
    patch_size: int = 16
    num_windows: int = 2
    positional_encoding_size: int = 24
    sa_nheads: int = 8
    ca_nheads: int = 16
    dec_n_points: int = 2
    dim_feedforward: int = 2048
    bbox_reparam: bool = True
    lite_refpoint_refine: bool = True
    # backbone / projector shape
    vit_width: int = 384
    vit_depth: int = 12
    vit_heads: int = 6
    out_feature_indexes: tuple = (3, 6, 9, 12)
    projector_levels: tuple = ("P4",)
    projector_blocks: int = 3
    # loss configuration
    cls_loss_coef: float = 1.0
    bbox_loss_coef: float = 5.0
    giou_loss_coef: float = 2.0
    mask_ce_loss_coef: float = 1.0
    mask_dice_loss_coef: float = 1.0
    sum_group_losses: bool = False
    use_varifocal_loss: bool = False
    use_position_supervised_loss: bool = False
    ia_bce_loss: bool = True
    aux_loss: bool = True
    mask_point_sample_ratio: int = 16
    focal_alpha: float = 0.25
    set_cost_class: float = 2.0
    set_cost_bbox: float = 5.0
    set_cost_giou: float = 2.0

    @property
    def num_feature_levels(self) -> int:
        return len(self.projector_levels)

    @property
    def vit_head_dim(self) -> int:
        return self.vit_width // self.vit_heads

    @property
    def train_queries(self) -> int:
        return self.num_queries * max(1, self.group_detr)

    def tokens_per_side(self, resolution: Optional[int] = None) -> int:
        return (resolution or self.resolution) // self.patch_size

    def validate(self) -> None:
        if self.hidden_dim % self.ca_nheads:
            raise ValueError("hidden_dim must be divisible by ca_nheads")
        if self.vit_width % self.vit_heads:
            raise ValueError("vit_width must be divisible by vit_heads")
        side = self.tokens_per_side()
        if self.num_windows > 1 and side % self.num_windows:
            raise ValueError(
                f"{side} patches per side cannot be split into {self.num_windows} windows "
                f"(resolution {self.resolution}, patch {self.patch_size})")
        for lvl in self.projector_levels:
            if lvl not in ("P3", "P4", "P5", "P6"):
                raise ValueError(f"unknown projector level {lvl}")

    def loss_weight_dict(self) -> dict:
        """Loss name -> coefficient (reference `detection_ops.cpp:1451-1478`)."""
        base = {"loss_ce": self.cls_loss_coef, "loss_bbox": self.bbox_loss_coef, "loss_giou": self.giou_loss_coef}
        if self.segmentation:
            base["loss_mask_ce"] = self.mask_ce_loss_coef
            base["loss_mask_dice"] = self.mask_dice_loss_coef
        out = dict(base)
        if self.aux_loss:
            for i in range(self.dec_layers - 1):
                for k, v in base.items():
                    out[f"{k}_{i}"] = v
            if self.two_stage:
                for k, v in base.items():
                    out[f"{k}_enc"] = v
        return out


def config_from_preset(preset, **overrides) -> RfDetrConfig:
    spec: PresetSpec = find_preset(preset) if isinstance(preset, str) else preset
    if spec is None:
        raise ValueError(f"unknown RF-DETR preset: {preset}")
    cfg = RfDetrConfig(
        preset_name=spec.name, resolution=spec.resolution, segmentation=spec.segmentation,
        num_classes=spec.num_classes, num_queries=spec.num_queries, num_select=spec.num_select,
        dec_layers=spec.dec_layers, group_detr=spec.group_detr, two_stage=spec.two_stage,
        hidden_dim=spec.hidden_dim, patch_size=spec.patch_size, num_windows=spec.num_windows,
        positional_encoding_size=spec.positional_encoding_size, vit_width=spec.vit_width,
        vit_depth=spec.vit_depth, vit_heads=spec.vit_heads, out_feature_indexes=tuple(spec.out_feature_indexes),
        projector_levels=tuple(spec.projector_levels), cls_loss_coef=spec.cls_loss_coef,
        bbox_loss_coef=spec.bbox_loss_coef, giou_loss_coef=spec.giou_loss_coef,
        mask_ce_loss_coef=spec.mask_ce_loss_coef, mask_dice_loss_coef=spec.mask_dice_loss_coef,
    )
    for k, v in overrides.items():
        if not hasattr(cfg, k):
            raise AttributeError(f"RfDetrConfig has no field {k}")
        setattr(cfg, k, v)
    cfg.validate()
    return cfg
