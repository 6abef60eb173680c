"""RF-DETR preset catalog, weight catalog and path -> preset inference.

The preset values are the model hyper-parameters of the reference
(`src/rfdetr/layers/model_config.cpp:91-313`, display metadata
`include/mmltk/rfdetr/preset_catalog.h:24-35`, weight assets
`src/rfdetr/weight_catalog.cpp:10-33`).  They have to be identical because
the official `.pth` checkpoints only load into a model of the same shape.

Three presets have no counterpart in the reference and exist for the
benchmark configurations of this framework:

* ``rf-detr-base``: 560x560, patch 14 (40x40 tokens, 20x20 per window), ViT-S,
  single P4 level.  560 is not divisible into 2 windows at patch 16.
* ``rf-detr-large-vitb``: 704x704, patch 16, a ViT-B backbone (768 wide, 12
  heads) and a two-level projector (P3 + P5).
* ``rf-detr-tiny-test``: a 32x32 model used by unit tests only.
"""
from __future__ import annotations

import dataclasses
import os
import re
from typing import Optional

__all__ = [
    "PresetSpec",
    "PRESETS",
    "WEIGHT_CATALOG",
    "find_preset",
    "preset_names",
    "find_preset_by_weight_filename",
    "infer_preset_from_path",
]


@dataclasses.dataclass(frozen=True)
class PresetSpec:
    name: str
    display_name: str
    size_label: str
    encoder: str
    weight_filename: str
    resolution: int
    patch_size: int
    num_windows: int
    positional_encoding_size: int
    dec_layers: int
    num_queries: int
    num_select: int
    num_classes: int = 91
    hidden_dim: int = 256
    group_detr: int = 13
    two_stage: bool = True
    segmentation: bool = False
    cls_loss_coef: float = 1.0
    bbox_loss_coef: float = 5.0
    giou_loss_coef: float = 2.0
    mask_ce_loss_coef: float = 1.0
    mask_dice_loss_coef: float = 1.0
    # backbone shape (the reference hard-wires ViT-S: 384 / 12 layers / 6 heads)
    vit_width: int = 384
    vit_depth: int = 12
    vit_heads: int = 6
    out_feature_indexes: tuple = (3, 6, 9, 12)
    projector_levels: tuple = ("P4",)
    in_reference: bool = True

    @property
    def task(self) -> str:
        return "segmentation" if self.segmentation else "detection"


def _det(name, display, label, weights, res, dec_layers, pos):
    return PresetSpec(name, display, label, "dinov2_windowed_small", weights, res, 16, 2, pos, dec_layers, 300, 300)


def _seg(name, display, label, weights, res, windows, pos, dec_layers, queries):
    return PresetSpec(
        name, display, label, "dinov2_windowed_small", weights, res, 12, windows, pos, dec_layers, queries, queries,
        segmentation=True, cls_loss_coef=5.0, bbox_loss_coef=5.0, giou_loss_coef=2.0,
        mask_ce_loss_coef=5.0, mask_dice_loss_coef=5.0,
    )


_PRESET_LIST = [
    _det("rf-detr-nano", "RF-DETR Nano", "N", "rf-detr-nano.pth", 384, 2, 24),
    _det("rf-detr-small", "RF-DETR Small", "S", "rf-detr-small.pth", 512, 3, 32),
    _det("rf-detr-medium", "RF-DETR Medium", "M", "rf-detr-medium.pth", 576, 4, 36),
    _det("rf-detr-large", "RF-DETR Large", "L", "rf-detr-large-2026.pth", 704, 4, 44),
    _seg("rf-detr-seg-nano", "RF-DETR Seg Nano", "N", "rf-detr-seg-nano.pt", 312, 1, 26, 4, 100),
    _seg("rf-detr-seg-small", "RF-DETR Seg Small", "S", "rf-detr-seg-small.pt", 384, 2, 32, 4, 100),
    _seg("rf-detr-seg-medium", "RF-DETR Seg Medium", "M", "rf-detr-seg-medium.pt", 432, 2, 36, 5, 200),
    _seg("rf-detr-seg-large", "RF-DETR Seg Large", "L", "rf-detr-seg-large.pt", 504, 2, 42, 5, 200),
    _seg("rf-detr-seg-xlarge", "RF-DETR Seg XLarge", "XL", "rf-detr-seg-xlarge.pt", 624, 2, 52, 6, 300),
    _seg("rf-detr-seg-xxlarge", "RF-DETR Seg 2XLarge", "2XL", "rf-detr-seg-xxlarge.pt", 768, 2, 64, 6, 300),
    # framework-only presets (benchmark configurations; no reference counterpart)
    PresetSpec("rf-detr-base", "RF-DETR Base", "B", "dinov2_windowed_small", "rf-detr-base.pth", 560, 14, 2, 40,
               3, 300, 300, in_reference=False),
    PresetSpec("rf-detr-large-vitb", "RF-DETR Large (ViT-B, P3+P5)", "L", "dinov2_windowed_base",
               "rf-detr-large-vitb.pth", 704, 16, 2, 44, 4, 300, 300, vit_width=768, vit_heads=12,
               out_feature_indexes=(2, 5, 8, 11), projector_levels=("P3", "P5"), in_reference=False),
    PresetSpec("rf-detr-tiny-test", "RF-DETR tiny (tests)", "T", "dinov2_windowed_small", "rf-detr-tiny-test.pth",
               32, 16, 1, 2, 2, 10, 10, group_detr=1, vit_width=64, vit_depth=4, vit_heads=2,
               out_feature_indexes=(1, 2, 3, 4), in_reference=False),
]

PRESETS = {p.name: p for p in _PRESET_LIST}

# canonical filename -> (download url, md5); reference `src/rfdetr/weight_catalog.cpp:10-33`
WEIGHT_CATALOG = {
    "rf-detr-large-2026.pth": ("https://storage.googleapis.com/rfdetr/rf-detr-large-2026.pth",
                               "5cb72153541cbcb9aa6efa26222acc75"),
    "rf-detr-nano.pth": ("https://storage.googleapis.com/rfdetr/nano_coco/checkpoint_best_regular.pth",
                         "fb6504cce7fbdc783f7a46991f07639f"),
    "rf-detr-small.pth": ("https://storage.googleapis.com/rfdetr/small_coco/checkpoint_best_regular.pth",
                          "fb37061c1af7bace359c91b723a8d5c1"),
    "rf-detr-medium.pth": ("https://storage.googleapis.com/rfdetr/medium_coco/checkpoint_best_regular.pth",
                           "7223f764a87b863f02eb8d52bf0ce2ee"),
    "rf-detr-seg-nano.pt": ("https://storage.googleapis.com/rfdetr/rf-detr-seg-n-ft.pth",
                            "9995497791d0ff1664a1d9ddee9cfd20"),
    "rf-detr-seg-small.pt": ("https://storage.googleapis.com/rfdetr/rf-detr-seg-s-ft.pth",
                             "0a2a3006381d0c42853907e700eadd08"),
    "rf-detr-seg-medium.pt": ("https://storage.googleapis.com/rfdetr/rf-detr-seg-m-ft.pth",
                              "a49af1562c3719227ad43d0ca53b4c7a"),
    "rf-detr-seg-large.pt": ("https://storage.googleapis.com/rfdetr/rf-detr-seg-l-ft.pth",
                             "275f7b094909544ed2841c94a677d07e"),
    "rf-detr-seg-xlarge.pt": ("https://storage.googleapis.com/rfdetr/rf-detr-seg-xl-ft.pth",
                              "3693b35d0eea86ebb3e0444f4a611fba"),
    "rf-detr-seg-xxlarge.pt": ("https://storage.googleapis.com/rfdetr/rf-detr-seg-2xl-ft.pth",
                               "040bc3412af840fa8a47e0ff69b552ba"),
}

# extra short aliases per preset and their scores (reference `model_config.cpp:65-89`)
_ALIASES = {
    "seg-nano": [("seg-n", 1400)],
    "seg-small": [("seg-s", 1400)],
    "seg-medium": [("seg-med", 1400), ("seg-m", 1390)],
    "seg-large": [("seg-l", 1400)],
    "seg-xlarge": [("seg-xl", 1400)],
    "seg-xxlarge": [("seg-2xl", 1400), ("seg-xxl", 1390)],
}


def preset_names(reference_only: bool = False):
    return [p.name for p in _PRESET_LIST if p.in_reference or not reference_only]


def find_preset(name: str) -> Optional[PresetSpec]:
    return PRESETS.get(name)


def find_preset_by_weight_filename(filename: str) -> Optional[PresetSpec]:
    for p in _PRESET_LIST:
        if p.weight_filename == filename:
            return p
    return None


def _has_token(haystack: str, needle: str) -> bool:
    """True if ``needle`` occurs in ``haystack`` bounded by non-alphanumerics."""
    if not needle:
        return False
    for m in re.finditer(re.escape(needle), haystack):
        s, e = m.start(), m.end()
        left = s == 0 or not haystack[s - 1].isalnum()
        right = e == len(haystack) or not haystack[e].isalnum()
        if left and right:
            return True
    return False


def infer_preset_from_path(path) -> Optional[PresetSpec]:
    """Score every preset against a weights/engine path (reference `model_config.cpp:17-89,332-395`).

    Exact canonical filenames win; then full preset names, upstream URL
    basenames, preset suffixes ("medium", "seg-xl", ...) and aliases.  The
    longest, highest-scoring token match is returned.
    """
    text = os.fspath(path).replace("\\", "/").lower()
    base = os.path.basename(text)
    exact = find_preset_by_weight_filename(os.path.basename(os.fspath(path)))
    if exact is not None:
        return exact
    best, best_score = None, 0
    for p in _PRESET_LIST:
        if not p.in_reference:
            continue
        cands = [(p.name, 3000), (p.weight_filename.rsplit(".", 1)[0], 2500)]
        url = WEIGHT_CATALOG.get(p.weight_filename, ("", ""))[0]
        ub = url.rsplit("/", 1)[-1].rsplit(".", 1)[0].lower()
        if ub and ub != "checkpoint_best_regular":
            cands.append((ub, 2000))
        suffix = p.name[len("rf-detr-"):]
        cands.append((suffix, 1500))
        cands.extend(_ALIASES.get(suffix, []))
        for cand, score in cands:
            if _has_token(text, cand.lower()) or _has_token(base, cand.lower()):
                s = score + len(cand)
                if s > best_score:
                    best, best_score = p, s
    return best
