"""Upstream RF-DETR ``.pth`` checkpoints (the official Python package's files).

Reading: ``{"model": state_dict, "args": Namespace}`` (also a bare state dict,
``{"state_dict": ...}`` or a module with ``state_dict()``), tensors kept under
their upstream names; 15 loss/matcher fields are taken from ``args``.
Writing: ``{"model": OrderedDict, "args": Namespace(...)}``.  Reference:
`utilities/rfdetr_checkpoint_bridge.py:46-238` (run there as a helper process
from C++; here it is plain Python in-process) and
`src/rfdetr/checkpoint/python_checkpoint_bridge.cpp:181-381`.

Loading uses ``torch.load(weights_only=True)`` with ``argparse.Namespace`` as
the only extra allowed global, so a checkpoint cannot run code on load.
"""
from __future__ import annotations

import argparse
import os
from collections import OrderedDict
from typing import Dict, Optional, Tuple

import torch

from .native import OPTIONAL_FIELDS

__all__ = ["load_upstream_checkpoint", "write_upstream_checkpoint", "upstream_metadata"]


def _coerce(kind, v):
    if kind is bool:
        return bool(v) if isinstance(v, bool) else None
    if isinstance(v, bool):
        return None
    if kind is int:
        if isinstance(v, int) or (isinstance(v, float) and float(v).is_integer()):
            return int(v)
        return None
    if isinstance(v, (int, float)):
        return float(v)
    return None


def upstream_metadata(args) -> Dict[str, object]:
    if args is None:
        return {}
    get = (lambda k: args.get(k)) if isinstance(args, dict) else (lambda k: getattr(args, k, None))
    out = {}
    for k, kind in OPTIONAL_FIELDS.items():
        v = _coerce(kind, get(k))
        if v is not None:
            out[k] = v
    return out


def load_upstream_checkpoint(path: str) -> Tuple["OrderedDict[str, torch.Tensor]", Dict[str, object]]:
    with torch.serialization.safe_globals([argparse.Namespace]):
        root = torch.load(path, map_location="cpu", weights_only=True)
    args = None
    if isinstance(root, dict):
        args = root.get("args")
        if isinstance(root.get("model"), dict):
            state = root["model"]
        elif isinstance(root.get("state_dict"), dict):
            state = root["state_dict"]
        elif root and all(isinstance(k, str) and isinstance(v, torch.Tensor) for k, v in root.items()):
            state = root
        else:
            raise ValueError(f"upstream checkpoint has neither 'model' nor 'state_dict': {path}")
    elif hasattr(root, "state_dict"):
        state = root.state_dict()
    else:
        raise ValueError(f"upstream checkpoint root is {type(root).__name__}: {path}")
    out = OrderedDict()
    for k, v in state.items():
        if not isinstance(v, torch.Tensor):
            raise ValueError(f"upstream checkpoint entry is not a tensor: {k}")
        out[str(k)] = v.detach().cpu().contiguous()
    if not out:
        raise ValueError(f"upstream checkpoint state dict is empty: {path}")
    return out, upstream_metadata(args)


def write_upstream_checkpoint(path: str, state: Dict[str, torch.Tensor], metadata: Optional[dict] = None) -> None:
    model = OrderedDict((k, v.detach().cpu().contiguous()) for k, v in state.items())
    args = argparse.Namespace(**(metadata or {}))
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    torch.save({"model": model, "args": args}, path)
