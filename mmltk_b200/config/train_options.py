"""Training options, optimizer recipes and augmentation config.

Mirrors `TrainOptions` (reference `include/mmltk/rfdetr/train.h:16-66`), the
optimizer recipes with per-field override tracking
(`include/mmltk/rfdetr/train_recipe.h:14-102`) and `GpuAugmentationConfig`
(`include/mmltk/rfdetr/train_types.h:19-42`).
"""
from __future__ import annotations

import dataclasses
import math
from typing import List, Optional

__all__ = ["AugGroup", "AugmentationConfig", "TrainOptions", "RECIPES", "apply_recipe", "lr_scale", "warmup_momentum"]


@dataclasses.dataclass
class AugGroup:
    probability: float = 0.5
    min_strength: float = 0.05
    max_strength: float = 0.5

    def valid(self) -> bool:
        vals = (self.probability, self.min_strength, self.max_strength)
        return (all(math.isfinite(v) for v in vals) and 0.0 <= self.probability <= 1.0
                and 0.0 <= self.min_strength <= self.max_strength <= 1.0)


@dataclasses.dataclass
class AugmentationConfig:
    enabled: bool = False
    geometry: AugGroup = dataclasses.field(default_factory=AugGroup)
    resize: AugGroup = dataclasses.field(default_factory=AugGroup)
    color: AugGroup = dataclasses.field(default_factory=AugGroup)
    noise: AugGroup = dataclasses.field(default_factory=AugGroup)
    blur: AugGroup = dataclasses.field(default_factory=AugGroup)
    occlusion: AugGroup = dataclasses.field(default_factory=AugGroup)
    copy_paste_probability: float = 0.5

    def valid(self) -> bool:
        groups = (self.geometry, self.resize, self.color, self.noise, self.blur, self.occlusion)
        return all(g.valid() for g in groups) and 0.0 <= self.copy_paste_probability <= 1.0


RECIPE_FIELDS = ("lr", "lr_encoder", "lr_component_decay", "encoder_layer_decay", "momentum", "weight_decay",
                 "warmup_epochs", "warmup_momentum", "lr_min_factor", "lr_drop", "lr_scheduler")

RECIPES = {
    "adamw": dict(lr=1e-4, lr_encoder=1.5e-4, lr_component_decay=0.7, encoder_layer_decay=0.8, momentum=0.95,
                  weight_decay=1e-4, warmup_epochs=0.0, warmup_momentum=0.0, lr_min_factor=0.0, lr_drop=100,
                  lr_scheduler="step"),
    "muon": dict(lr=2e-4, lr_encoder=3e-4, lr_component_decay=0.7, encoder_layer_decay=0.8, momentum=0.9,
                 weight_decay=5e-4, warmup_epochs=3.0, warmup_momentum=0.8, lr_min_factor=0.01, lr_drop=100,
                 lr_scheduler="cosine"),
}


@dataclasses.dataclass
class TrainOptions:
    train_compiled: Optional[str] = None
    val_compiled: Optional[str] = None
    test_compiled: Optional[str] = None
    output_dir: Optional[str] = None
    weights: Optional[str] = None
    resume: Optional[str] = None
    preset: str = ""
    resolution: int = 0
    batch_size: int = 1
    val_batch_size: int = 0
    epochs: int = 1
    grad_accum_steps: int = 1
    optimizer: str = "adamw"
    lr: float = 1e-4
    lr_encoder: float = 1.5e-4
    lr_component_decay: float = 0.7
    encoder_layer_decay: float = 0.8
    momentum: float = 0.95
    weight_decay: float = 1e-4
    warmup_epochs: float = 0.0
    warmup_momentum: float = 0.0
    lr_min_factor: float = 0.0
    lr_drop: int = 100
    lr_scheduler: str = "step"
    clip_max_norm: float = 0.1
    fused_optimizer: bool = True
    freeze_encoder: bool = False
    use_ema: bool = False
    ema_decay: float = 0.993
    ema_tau: int = 100
    validation_loss: bool = False
    validation_profile: bool = False
    eval_max_dets: int = 500
    augmentation: AugmentationConfig = dataclasses.field(default_factory=AugmentationConfig)
    device_id: int = 0
    device_ids: List[int] = dataclasses.field(default_factory=list)
    workers: int = 0
    lanes: int = 0
    cpu_affinity: str = ""
    high_priority: bool = False   # lowest permitted nice value and realtime I/O priority for this process
    prefetch_factor: int = 2
    print_freq: int = 100
    seed: int = 42
    amp: bool = True
    progress_bar: bool = True
    compile_mode: str = "selective"
    # distributed worker plumbing (set by the launcher)
    dist_worker: bool = False
    dist_rank: int = 0
    dist_world_size: int = 1
    dist_store_file: str = ""
    # B200 framework switches
    ddp_backend: str = "fused"        # "fused" (in-kernel NVSwitch RS/AG + AdamW + EMA) | "nccl" (baseline)
    cuda_graph: bool = True
    overrides: set = dataclasses.field(default_factory=set)

    def micro_batches_per_step(self) -> int:
        """Batches whose gradients make one optimizer step: grad_accum_steps x lanes (reference
        `train.cpp:2459-2511`: a wave of ``lanes`` batches, every ``grad_accum_steps`` waves)."""
        return max(1, int(self.grad_accum_steps)) * max(1, int(self.lanes))

    def validate(self) -> None:
        if self.optimizer not in RECIPES:
            raise ValueError(f"unknown optimizer {self.optimizer}")
        if self.lr_scheduler not in ("step", "cosine"):
            raise ValueError(f"unknown lr scheduler {self.lr_scheduler}")
        if self.compile_mode not in ("none", "selective", "full"):
            raise ValueError(f"unknown compile mode {self.compile_mode}")
        if self.batch_size < 1 or self.grad_accum_steps < 1 or self.epochs < 1:
            raise ValueError("batch size, grad accumulation steps and epochs must be positive")
        if not self.augmentation.valid():
            raise ValueError("invalid augmentation configuration")


def apply_recipe(opts: TrainOptions, optimizer: Optional[str] = None) -> TrainOptions:
    """Apply the optimizer recipe to every field the user did not set explicitly."""
    recipe = RECIPES[optimizer or opts.optimizer]
    for field in RECIPE_FIELDS:
        if field not in opts.overrides:
            setattr(opts, field, recipe[field])
    return opts


def lr_scale(opts: TrainOptions, step: int, steps_per_epoch: int, total_steps: int) -> float:
    """LR multiplier (reference `include/mmltk/rfdetr/training_ops.h:239-255`)."""
    warm = float(steps_per_epoch) * opts.warmup_epochs
    if warm > 0 and step < warm:
        return step / max(1.0, warm)
    if opts.lr_scheduler == "cosine":
        progress = step - warm
        denom = max(1.0, total_steps - warm)
        return opts.lr_min_factor + (1 - opts.lr_min_factor) * 0.5 * (1 + math.cos(math.pi * progress / denom))
    return 1.0 if step < opts.lr_drop * steps_per_epoch else 0.1


def warmup_momentum(opts: TrainOptions, step: int, steps_per_epoch: int, target: float) -> float:
    warm = float(steps_per_epoch) * opts.warmup_epochs
    if warm <= 0 or opts.warmup_momentum <= 0 or step >= warm:
        return target
    a = step / max(1.0, warm)
    return opts.warmup_momentum + (target - opts.warmup_momentum) * a
