"""Loading checkpoints into a model.

* :func:`load_checkpoint` -- native archive or upstream ``.pth``, by content;
* :func:`prepare_for_module` -- encoder-head names of upstream exports
  (``enc_output.*``, ``enc_output_norm.*``, ``enc_out_class_embed.*``,
  ``enc_out_bbox_embed.*``) get the ``transformer.`` prefix and group 0 is
  copied to every further group the model has; query / refpoint tables are
  narrowed to the model's rows (reference `src/rfdetr/layers/model.cpp:1423-1469`);
* :func:`apply_to_module` -- name / shape matched copy with a
  loaded / missing / unexpected / incompatible summary, strict or not
  (`src/rfdetr/checkpoint.cpp:203-286`);
* :func:`load_weights` -- the above plus the class-count bridge: when the
  checkpoint's class head differs, the model's heads are resized to it, loaded,
  then resized back by repeating rows (`model.cpp:1943-1986`), restoring the
  original heads if loading fails.
"""
from __future__ import annotations

import dataclasses
import os
from collections import OrderedDict
from typing import Dict, List, Optional

import torch

from ..config.presets import find_preset_by_weight_filename, infer_preset_from_path
from .native import CheckpointMetadata, NativeCheckpoint, is_native_checkpoint, load_native_checkpoint, \
    save_native_checkpoint
from .upstream import load_upstream_checkpoint

__all__ = ["LoadSummary", "load_checkpoint", "prepare_for_module", "apply_to_module", "load_weights",
           "checkpoint_class_count", "normalize_checkpoint"]

_ENC = ("enc_output.", "enc_output_norm.", "enc_out_class_embed.", "enc_out_bbox_embed.")


@dataclasses.dataclass
class LoadSummary:
    loaded: List[str] = dataclasses.field(default_factory=list)
    missing: List[str] = dataclasses.field(default_factory=list)
    unexpected: List[str] = dataclasses.field(default_factory=list)
    incompatible: List[str] = dataclasses.field(default_factory=list)

    def ok(self) -> bool:
        return not (self.missing or self.unexpected or self.incompatible)


def load_checkpoint(path: str) -> NativeCheckpoint:
    if not os.path.exists(path):
        raise FileNotFoundError(path)
    if is_native_checkpoint(path):
        return load_native_checkpoint(path)
    state, opt = load_upstream_checkpoint(path)
    meta = CheckpointMetadata(source_kind="upstream-python", source_path=os.path.abspath(path), optional=opt)
    spec = find_preset_by_weight_filename(os.path.basename(path)) or infer_preset_from_path(path)
    if spec is not None:
        meta.preset_name = spec.name
        meta.num_classes = spec.num_classes
    n = checkpoint_class_count(state)
    if n is not None:
        meta.num_classes = n
    return NativeCheckpoint(meta, state)


def checkpoint_class_count(state: Dict[str, torch.Tensor]) -> Optional[int]:
    for k in ("class_embed.bias", "class_embed.weight"):
        if k in state and state[k].dim() >= 1:
            return int(state[k].shape[0])
    return None


def prepare_for_module(state: Dict[str, torch.Tensor], target: Dict[str, torch.Tensor]) -> "OrderedDict[str, torch.Tensor]":
    out = OrderedDict()
    extra = OrderedDict()
    for name, t in state.items():
        if name.startswith(_ENC):
            orig = name
            name = "transformer." + name
            if ".0." in orig:
                for g in range(1, 32):
                    cand = "transformer." + orig.replace(".0.", f".{g}.", 1)
                    if cand in target:
                        extra[cand] = t.clone()
        if name in ("refpoint_embed.weight", "query_feat.weight") and name in target:
            rows = target[name].shape[0]
            if t.dim() == target[name].dim() and t.shape[0] >= rows:
                t = t[:rows].contiguous()
        out[name] = t
    for k, v in extra.items():
        out.setdefault(k, v)
    return out


def apply_to_module(model: torch.nn.Module, state: Dict[str, torch.Tensor], strict: bool = True) -> LoadSummary:
    own = model.state_dict()
    s = LoadSummary()
    good = OrderedDict()
    for k, v in state.items():
        if k not in own:
            s.unexpected.append(k)
        elif tuple(own[k].shape) != tuple(v.shape):
            s.incompatible.append(k)
        else:
            good[k] = v.to(own[k].dtype)
            s.loaded.append(k)
    s.missing = [k for k in own if k not in state]
    if strict and not s.ok():
        def few(x):
            return ", ".join(x[:5]) + (" ..." if len(x) > 5 else "")
        raise RuntimeError(f"checkpoint does not match the model: missing [{few(s.missing)}] unexpected "
                           f"[{few(s.unexpected)}] incompatible [{few(s.incompatible)}]")
    merged = OrderedDict((k, good.get(k, own[k])) for k in own)
    model.load_state_dict(merged, strict=True)
    return s


def load_weights(model, path_or_ckpt, strict: bool = True) -> LoadSummary:
    ckpt = load_checkpoint(path_or_ckpt) if isinstance(path_or_ckpt, str) else path_or_ckpt
    orig = model.class_embed.weight.shape[0]
    n = checkpoint_class_count(ckpt.state_dict)
    resized = n is not None and n != orig
    saved = None
    if resized:
        saved = {k: v.detach().clone() for k, v in model.state_dict().items()
                 if k.startswith(("class_embed.", "transformer.enc_out_class_embed."))}
        model.reinitialize_detection_head(n)
    try:
        prepared = prepare_for_module(ckpt.state_dict, model.state_dict())
        summary = apply_to_module(model, prepared, strict)
    except Exception:
        if resized:
            model.reinitialize_detection_head(orig)
            model.load_state_dict(saved, strict=False)
        raise
    if resized:
        model.reinitialize_detection_head(orig)
    return summary


def normalize_checkpoint(src: str, dst: str) -> NativeCheckpoint:
    """Any supported checkpoint -> native archive (``mmltk rfdetr normalize-weights``)."""
    ckpt = load_checkpoint(src)
    save_native_checkpoint(dst, ckpt.state_dict, ckpt.metadata, ckpt.extra)
    return ckpt
