"""Native checkpoint files (``.pt``): model state + metadata, optionally the
resume state.

Container: a libtorch serialize archive, read and written through the same
libtorch classes as the reference (bridge in ``csrc/host/archive_io.cpp``), so
files are interchangeable with it.  Key layout (reference
`include/mmltk/rfdetr/checkpoint.h:14-64`, `src/rfdetr/checkpoint.cpp:26-106`,
`src/rfdetr/archive_utils.h`):

* ``format = "mmltk.rfdetr.native_checkpoint"``, ``format_version = 1``;
* metadata: ``preset_name``, ``source_kind``, ``source_path``, ``num_classes``
  and the optional loss / matcher fields of :data:`OPTIONAL_FIELDS`;
* ``state``: ``entry_count`` and one sub-archive ``entry_%06d`` per tensor with
  ``name`` and ``tensor``;
* resume checkpoints add ``optimizer_kind`` / ``optimizer`` / ``ema_state`` /
  ``epoch`` / scheduler and augmentation settings / best metrics / grad-scaler
  state (reference `src/rfdetr/training/train.cpp:1154-1245`); see
  :mod:`mmltk_b200.ckpt.resume`.
"""
from __future__ import annotations

import dataclasses
import os
import zipfile
from collections import OrderedDict
from typing import Dict, Optional

import torch

from ..ops._ext import native

__all__ = ["FORMAT", "FORMAT_VERSION", "OPTIONAL_FIELDS", "CheckpointMetadata", "NativeCheckpoint",
           "save_native_checkpoint", "load_native_checkpoint", "is_native_checkpoint", "state_to_archive",
           "state_from_archive"]

FORMAT = "mmltk.rfdetr.native_checkpoint"
FORMAT_VERSION = 1

OPTIONAL_FIELDS = {
    "sum_group_losses": bool, "use_varifocal_loss": bool, "use_position_supervised_loss": bool,
    "ia_bce_loss": bool, "aux_loss": bool, "mask_point_sample_ratio": int, "focal_alpha": float,
    "cls_loss_coef": float, "bbox_loss_coef": float, "giou_loss_coef": float, "mask_ce_loss_coef": float,
    "mask_dice_loss_coef": float, "set_cost_class": float, "set_cost_bbox": float, "set_cost_giou": float,
}


@dataclasses.dataclass
class CheckpointMetadata:
    preset_name: str = ""
    source_kind: str = "native"
    source_path: str = ""
    num_classes: int = 0
    optional: Dict[str, object] = dataclasses.field(default_factory=dict)

    def to_archive(self) -> dict:
        d = {"format": FORMAT, "format_version": FORMAT_VERSION, "preset_name": self.preset_name,
             "source_kind": self.source_kind, "source_path": self.source_path, "num_classes": int(self.num_classes)}
        for k, v in self.optional.items():
            if k in OPTIONAL_FIELDS and v is not None:
                d[k] = OPTIONAL_FIELDS[k](v)
        return d

    @classmethod
    def from_archive(cls, d: dict, path: str = "") -> "CheckpointMetadata":
        opt = {}
        for k, t in OPTIONAL_FIELDS.items():
            if k in d:
                v = d[k]
                if t is float and isinstance(v, bool):
                    raise ValueError(f"checkpoint key {k} is not numeric")
                opt[k] = t(v)
        return cls(str(d.get("preset_name", "")), str(d.get("source_kind", "native")),
                   str(d.get("source_path", path)), int(d.get("num_classes", 0)), opt)

    @classmethod
    def from_config(cls, cfg, source_kind: str = "native", source_path: str = "") -> "CheckpointMetadata":
        opt = {k: getattr(cfg, k) for k in OPTIONAL_FIELDS if hasattr(cfg, k)}
        return cls(getattr(cfg, "preset_name", ""), source_kind, source_path, int(cfg.num_classes), opt)


@dataclasses.dataclass
class NativeCheckpoint:
    metadata: CheckpointMetadata
    state_dict: "OrderedDict[str, torch.Tensor]"
    extra: dict = dataclasses.field(default_factory=dict)   # resume fields (everything not above)


def state_to_archive(state: Dict[str, torch.Tensor]) -> dict:
    d = {"entry_count": len(state)}
    for i, (k, v) in enumerate(state.items()):
        d[f"entry_{i:06d}"] = {"name": str(k), "tensor": v.detach().cpu().contiguous()}
    return d


def state_from_archive(d: dict) -> "OrderedDict[str, torch.Tensor]":
    n = int(d["entry_count"])
    if n < 0:
        raise ValueError("checkpoint entry_count is negative")
    out = OrderedDict()
    for i in range(n):
        e = d[f"entry_{i:06d}"]
        out[e["name"]] = e["tensor"]
    return out


def save_native_checkpoint(path: str, state_dict: Dict[str, torch.Tensor], metadata: CheckpointMetadata,
                           extra: Optional[dict] = None) -> None:
    d = metadata.to_archive()
    d["state"] = state_to_archive(state_dict)
    if extra:
        d.update(extra)
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    tmp = path + ".tmp"
    native().archive_save(tmp, d)
    os.replace(tmp, path)   # readers never see a half-written file


def is_native_checkpoint(path: str) -> bool:
    if not zipfile.is_zipfile(path):
        return False
    try:
        return native().archive_load(path).get("format") == FORMAT
    except Exception:
        return False


def load_native_checkpoint(path: str) -> NativeCheckpoint:
    d = native().archive_load(path)
    if d.get("format") != FORMAT:
        raise ValueError(f"not a native RF-DETR checkpoint: {path}")
    if int(d.get("format_version", -1)) != FORMAT_VERSION:
        raise ValueError(f"unsupported native checkpoint format version {d.get('format_version')}: {path}")
    meta = CheckpointMetadata.from_archive(d, os.path.abspath(path))
    state = state_from_archive(d["state"])
    known = set(meta.to_archive()) | {"state"} | set(OPTIONAL_FIELDS)
    extra = {k: v for k, v in d.items() if k not in known}
    return NativeCheckpoint(meta, state, extra)
