"""Dataset compiler front-end: source tree -> compiled ``<split>.bin``.

Source layout (reference `README.md:293-360`): ``categories.json`` with a
``classes`` table (dense ids starting at 0 or 1, unique names) and one
directory per split holding ``000001.png`` + ``000001.jsonl`` pairs (six-digit
sequential names).  Each JSONL line is one instance: ``class`` (name),
``bbox_xyxy`` (absolute pixels), optional ``mask_rle`` ("start:length ..."
row-major runs) and optional ``image_size_wh``.  Background images have an
empty JSONL file.

Class ids are stored as given by ``categories.json`` (the model then gets
``num_classes = max id + 1``, reference `src/rfdetr/training/train.cpp:107-109`).
The parsing happens here; image decode, resize, mask re-encoding and the file
layout are done by the native compiler (``csrc/host/dataset.cpp``) on a thread pool.
"""
from __future__ import annotations

import json
import os
import re
from typing import Dict, List, Optional, Tuple

import torch

from ..ops._ext import native

__all__ = ["load_categories", "scan_split", "compile_split", "compile_dataset", "CompileError"]

_NAME = re.compile(r"^(\d{6})\.png$")


class CompileError(RuntimeError):
    pass


def load_categories(source_dir: str) -> Tuple[Dict[str, int], List[str], dict]:
    path = os.path.join(source_dir, "categories.json")
    try:
        with open(path) as f:
            meta = json.load(f)
    except FileNotFoundError:
        raise CompileError(f"missing {path}")
    classes = meta.get("classes", [])
    if not classes:
        raise CompileError("categories.json has no classes")
    ids = sorted(int(c["id"]) for c in classes)
    if ids[0] not in (0, 1) or ids != list(range(ids[0], ids[0] + len(ids))):
        raise CompileError("class ids must be dense and start at 0 or 1")
    names = [str(c["name"]) for c in classes]
    if len(set(names)) != len(names):
        raise CompileError("class names must be unique")
    if ids[-1] >= 256:
        raise CompileError("at most 256 classes are supported")
    by_name = {str(c["name"]): int(c["id"]) for c in classes}
    table = [""] * (ids[-1] + 1)
    for n, i in by_name.items():
        table[i] = n
    return by_name, table, meta


def scan_split(source_dir: str, split: str) -> List[str]:
    d = os.path.join(source_dir, split)
    if not os.path.isdir(d):
        raise CompileError(f"missing split directory {d}")
    stems = sorted(m.group(1) for f in os.listdir(d) if (m := _NAME.match(f)))
    for i, s in enumerate(stems):
        if int(s) != i + 1:
            raise CompileError(f"{split}: image names must be sequential from 000001 (found {s} at position {i + 1})")
        if not os.path.exists(os.path.join(d, s + ".jsonl")):
            raise CompileError(f"{split}: {s}.png has no {s}.jsonl")
    return [os.path.join(d, s) for s in stems]


def _parse_rle(text: str) -> List[int]:
    out = []
    for tok in text.split():
        a, b = tok.split(":")
        out += [int(a), int(b)]
    return out


def compile_split(source_dir: str, output_dir: str, split: str, width: int = 432, height: int = 432,
                  workers: int = 0) -> dict:
    by_name, table, _ = load_categories(source_dir)
    stems = scan_split(source_dir, split)
    paths, counts, classes, boxes, rb, rc, rle = [], [], [], [], [], [], []
    for stem in stems:
        n = 0
        with open(stem + ".jsonl") as f:
            for lineno, line in enumerate(f, 1):
                line = line.strip()
                if not line:
                    continue
                obj = json.loads(line)
                name = obj.get("class")
                if name not in by_name:
                    raise CompileError(f"{stem}.jsonl:{lineno}: unknown class {name!r}")
                bb = obj.get("bbox_xyxy")
                if not bb or len(bb) != 4:
                    raise CompileError(f"{stem}.jsonl:{lineno}: bbox_xyxy must have 4 numbers")
                classes.append(by_name[name])
                boxes.append([float(v) for v in bb])
                runs = _parse_rle(obj["mask_rle"]) if obj.get("mask_rle") else []
                rb.append(len(rle) // 2)
                rc.append(len(runs) // 2)
                rle += runs
                n += 1
        paths.append(stem + ".png")
        counts.append(n)
    os.makedirs(output_dir, exist_ok=True)
    out = os.path.join(output_dir, f"{split}.bin")
    stats = native().compile_dataset(
        out, paths, torch.tensor(counts, dtype=torch.int32), torch.tensor(classes, dtype=torch.uint8),
        torch.tensor(boxes, dtype=torch.float32).reshape(-1, 4), torch.tensor(rb, dtype=torch.int64),
        torch.tensor(rc, dtype=torch.int64), torch.tensor(rle, dtype=torch.int64), table, width, height, workers)
    stats["path"] = out
    stats["split"] = split
    return stats


def compile_dataset(source_dir: str, output_dir: str, splits: Optional[List[str]] = None, width: int = 432,
                    height: int = 432, workers: int = 0) -> List[dict]:
    if splits is None:
        splits = sorted(d for d in os.listdir(source_dir) if os.path.isdir(os.path.join(source_dir, d)))
    return [compile_split(source_dir, output_dir, s, width, height, workers) for s in splits]
