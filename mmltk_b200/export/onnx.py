"""ONNX export and inspection.

Export (reference `src/rfdetr/layers/model.cpp:2141-2244`): eval mode, fp32 on
the CPU path (so MSDeformAttn is the grid-sample statement and attention the
plain SDPA), traced with torch's TorchScript-based exporter at opset 19 (the
only opset the reference accepts), batch size fixed at export.  Graph
inputs/outputs: ``input`` [B,3,H,W] (normalised pixels) -> ``dets``
[B,Q,4] (cxcywh), ``labels`` [B,Q,C] (logits) and, for segmentation presets,
``masks`` [B,Q,H/4,W/4].

The exporter builds the ModelProto in C++; torch only imports the ``onnx``
package afterwards to splice in onnxscript-defined custom functions, of which
this model has none.  When ``onnx`` is not installed that step is skipped.

:func:`onnx_info` reads a model's graph inputs / outputs with a small
protobuf wire-format reader (no ``onnx`` dependency), like the reference's
``mmltk-rfdetr-onnx-info`` tool (`src/rfdetr/onnx_model_info.cpp:63-113`).
"""
from __future__ import annotations

import contextlib
import io
import os
from typing import Dict, List, Optional, Tuple

import torch

__all__ = ["export_onnx", "onnx_info", "SUPPORTED_OPSETS"]

SUPPORTED_OPSETS = (19,)


class _Wrapper(torch.nn.Module):
    def __init__(self, model, masks: bool):
        super().__init__()
        self.model = model
        self.masks = masks

    def forward(self, x):
        out = self.model(x, include_masks=self.masks)
        if self.masks and "pred_masks" in out:
            return out["pred_boxes"], out["pred_logits"], out["pred_masks"]
        return out["pred_boxes"], out["pred_logits"]


@contextlib.contextmanager
def _without_onnx_package():
    try:
        import onnx  # noqa: F401
        yield
        return
    except ImportError:
        pass
    from torch.onnx._internal.torchscript_exporter import onnx_proto_utils, utils
    orig = onnx_proto_utils._add_onnxscript_fn

    def passthrough(model_bytes, custom_opsets):
        return model_bytes

    onnx_proto_utils._add_onnxscript_fn = passthrough
    try:
        yield
    finally:
        onnx_proto_utils._add_onnxscript_fn = orig


def export_onnx(model, path: str, opset_version: int = 19, batch_size: int = 1) -> Dict:
    if opset_version not in SUPPORTED_OPSETS:
        raise ValueError(f"ONNX export supports opset {SUPPORTED_OPSETS} only (got {opset_version})")
    import copy
    m = copy.deepcopy(model).to("cpu", torch.float32).eval().requires_grad_(False)
    res = m.cfg.resolution
    masks = bool(m.cfg.segmentation)
    w = _Wrapper(m, masks).eval()
    x = torch.zeros(batch_size, 3, res, res)
    names = ["dets", "labels"] + (["masks"] if masks else [])
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    with torch.no_grad(), _without_onnx_package():
        torch.onnx.export(w, (x,), path, dynamo=False, opset_version=opset_version, input_names=["input"],
                          output_names=names, do_constant_folding=True)
    return onnx_info(path)


# ------------------------------------------------------------------ minimal protobuf reader

def _varint(b: bytes, i: int) -> Tuple[int, int]:
    v, s = 0, 0
    while True:
        c = b[i]
        i += 1
        v |= (c & 0x7F) << s
        s += 7
        if c < 0x80:
            return v, i


def _fields(b: bytes):
    i = 0
    while i < len(b):
        key, i = _varint(b, i)
        f, wt = key >> 3, key & 7
        if wt == 0:
            v, i = _varint(b, i)
        elif wt == 1:
            v, i = b[i:i + 8], i + 8
        elif wt == 2:
            n, i = _varint(b, i)
            v, i = b[i:i + n], i + n
        elif wt == 5:
            v, i = b[i:i + 4], i + 4
        else:
            raise ValueError(f"unsupported protobuf wire type {wt}")
        yield f, wt, v


_ELEM = {1: "float32", 2: "uint8", 3: "int8", 5: "int16", 6: "int32", 7: "int64", 9: "bool", 10: "float16",
         11: "float64", 16: "bfloat16"}


def _value_info(b: bytes) -> Dict:
    name, elem, dims = "", None, []
    for f, _, v in _fields(b):
        if f == 1:
            name = v.decode()
        elif f == 2:                                   # TypeProto
            for f2, _, v2 in _fields(v):
                if f2 == 1:                            # tensor_type
                    for f3, _, v3 in _fields(v2):
                        if f3 == 1:
                            elem = _ELEM.get(v3, str(v3))
                        elif f3 == 2:                  # TensorShapeProto
                            for f4, _, v4 in _fields(v3):
                                if f4 == 1:
                                    d = None
                                    for f5, _, v5 in _fields(v4):
                                        d = v5 if f5 == 1 else (v5.decode() if f5 == 2 else d)
                                    dims.append(d)
    return {"name": name, "dtype": elem, "shape": dims}


def onnx_info(path: str) -> Dict:
    data = open(path, "rb").read()
    info = {"path": os.path.abspath(path), "inputs": [], "outputs": [], "opset": None, "initializers": 0,
            "nodes": 0}
    for f, _, v in _fields(data):
        if f == 8:                                     # opset_import
            for f2, _, v2 in _fields(v):
                if f2 == 2:
                    info["opset"] = v2
        elif f == 7:                                   # graph
            inits = set()
            ins = []
            for f2, _, v2 in _fields(v):
                if f2 == 1:
                    info["nodes"] += 1
                elif f2 == 5:
                    info["initializers"] += 1
                    for f3, _, v3 in _fields(v2):
                        if f3 == 8:
                            inits.add(v3.decode())
                elif f2 == 11:
                    ins.append(_value_info(v2))
                elif f2 == 12:
                    info["outputs"].append(_value_info(v2))
            info["inputs"] = [i for i in ins if i["name"] not in inits]
    outs = {o["name"]: o for o in info["outputs"]}
    if "labels" in outs and len(outs["labels"]["shape"]) == 3:
        info["num_queries"], info["num_classes"] = outs["labels"]["shape"][1], outs["labels"]["shape"][2]
    info["has_masks"] = "masks" in outs
    return info
