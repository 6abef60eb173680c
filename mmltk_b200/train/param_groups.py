"""Per-parameter learning rate / weight decay (reference
`src/rfdetr/training/train.cpp:889-955`).

encoder (``backbone.0.encoder``): lr_encoder * encoder_layer_decay^(L+1-layer_id) * lr_component_decay^2,
    layer_id 0 for embeddings, i+1 for ``.layer.<i>.``, L+1 otherwise (L = 13 for the 12-layer ViT);
    zero weight decay for names containing gamma / bias / norm / embeddings / rel_pos;
decoder (``transformer.decoder``): lr * lr_component_decay;  everything else: lr.
"""
from __future__ import annotations

import re
from typing import Dict, List, Tuple

__all__ = ["parameter_lr", "parameter_weight_decay", "is_muon_hidden_weight", "build_param_groups"]

_LAYER_RE = re.compile(r"\.layer\.(\d+)")


def is_encoder_param(name: str) -> bool:
    return "backbone.0.encoder" in name


def encoder_layer_id(name: str, num_vit_layers: int = 13) -> int:
    if "embeddings" in name:
        return 0
    m = _LAYER_RE.search(name)
    if m and ".residual." not in name:
        return int(m.group(1)) + 1
    return num_vit_layers + 1


def parameter_lr(name: str, opts, num_vit_layers: int = 13) -> float:
    if is_encoder_param(name):
        lid = encoder_layer_id(name, num_vit_layers)
        return (opts.lr_encoder * opts.encoder_layer_decay ** (num_vit_layers + 1 - lid)
                * opts.lr_component_decay ** 2)
    if "transformer.decoder" in name:
        return opts.lr * opts.lr_component_decay
    return opts.lr


def parameter_weight_decay(name: str, opts) -> float:
    if is_encoder_param(name):
        if any(k in name for k in ("gamma", "bias", "norm", "embeddings", "rel_pos")):
            return 0.0
    return opts.weight_decay


def is_muon_hidden_weight(name: str, ndim: int) -> bool:
    if ndim not in (2, 4) or "weight" not in name:
        return False
    excluded = ("embeddings", "cls_token", "mask_token", "query_feat", "refpoint_embed", "class_embed", "bbox_embed",
                "segmentation_head")
    return not any(k in name for k in excluded)


def build_param_groups(named_params, opts, num_vit_layers: int = 13) -> Tuple[List[Dict], List[int]]:
    """Returns (groups [{lr, weight_decay, muon, names}], group index per parameter) in
    first-seen order of (kind, lr, wd), like the reference."""
    groups: List[Dict] = []
    index: Dict[tuple, int] = {}
    assign: List[int] = []
    muon = getattr(opts, "optimizer", "adamw") == "muon"
    for name, p in named_params:
        lr = parameter_lr(name, opts, num_vit_layers)
        wd = parameter_weight_decay(name, opts)
        use_muon = muon and is_muon_hidden_weight(name, p.dim())
        key = (use_muon, lr, wd)
        if key not in index:
            index[key] = len(groups)
            groups.append({"lr": lr, "weight_decay": wd, "muon": use_muon, "names": []})
        groups[index[key]]["names"].append(name)
        assign.append(index[key])
    return groups, assign
