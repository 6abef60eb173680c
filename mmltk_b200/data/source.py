"""Writes a small synthetic source dataset (categories.json + PNG/JSONL
pairs) in the compiler's input layout -- the fixture the reference's tests
build (`tests/support/test_fixture.cpp:52-108`), used by tests and demos."""
from __future__ import annotations

import json
import os

import torch

from ..ops._ext import native

__all__ = ["write_synthetic_source"]


def _rle(mask: torch.Tensor) -> str:
    flat = mask.flatten().to(torch.int8)
    runs = []
    i, n = 0, flat.numel()
    d = torch.diff(torch.cat([torch.zeros(1, dtype=torch.int8), flat, torch.zeros(1, dtype=torch.int8)]))
    starts = (d == 1).nonzero().flatten().tolist()
    ends = (d == -1).nonzero().flatten().tolist()
    for s, e in zip(starts, ends):
        runs.append(f"{s}:{e - s}")
    return " ".join(runs)


def write_synthetic_source(root: str, splits=("train", "val"), images: int = 8, size=(96, 80), classes: int = 3,
                           max_instances: int = 4, seed: int = 0, masks: bool = True, min_instances: int = 0) -> str:
    g = torch.Generator().manual_seed(seed)
    w, h = size
    os.makedirs(root, exist_ok=True)
    cats = {"meta": {"dataset_name": "synthetic", "version": "1.0", "image_format": "png", "image_size_wh": [w, h],
                     "bbox_format": "xyxy_absolute_pixels", "mask_format": "rle_row_major_start_length"},
            "classes": [{"id": i + 1, "name": f"class_{i + 1}"} for i in range(classes)], "splits": {}}
    for split in splits:
        d = os.path.join(root, split)
        os.makedirs(d, exist_ok=True)
        for k in range(1, images + 1):
            img = (torch.rand(h, w, 3, generator=g) * 255).to(torch.uint8)
            lines = []
            for _ in range(int(torch.randint(min_instances, max_instances + 1, (1,), generator=g))):
                x1 = int(torch.randint(0, w - 12, (1,), generator=g))
                y1 = int(torch.randint(0, h - 12, (1,), generator=g))
                x2 = min(w, x1 + int(torch.randint(8, w // 2, (1,), generator=g)))
                y2 = min(h, y1 + int(torch.randint(8, h // 2, (1,), generator=g)))
                c = int(torch.randint(1, classes + 1, (1,), generator=g))
                rec = {"class": f"class_{c}", "bbox_xyxy": [x1, y1, x2, y2], "image_size_wh": [w, h]}
                if masks:
                    m = torch.zeros(h, w, dtype=torch.bool)
                    m[y1:y2, x1:x2] = True
                    rec["mask_rle"] = _rle(m)
                img[y1:y2, x1:x2] = torch.tensor([(40 * c) % 256, 255 - (40 * c) % 256, 128], dtype=torch.uint8)
                lines.append(json.dumps(rec))
            with open(os.path.join(d, f"{k:06d}.png"), "wb") as f:
                f.write(native().encode_png(img))
            with open(os.path.join(d, f"{k:06d}.jsonl"), "w") as f:
                f.write("\n".join(lines) + ("\n" if lines else ""))
        cats["splits"][split] = {"total": images}
    with open(os.path.join(root, "categories.json"), "w") as f:
        json.dump(cats, f, indent=1)
    return root
