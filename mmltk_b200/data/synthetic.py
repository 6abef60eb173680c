"""Synthetic batches with the BASELINE shapes: images drawn i.i.d. N(0,1) per
pixel (already normalised), K ~ U{kmin..kmax} boxes per image in normalised
cxcywh with centres U(0.1, 0.9) and w, h U(0.02, 0.4), labels uniform over
``num_labels`` class ids.  Used by the benchmark, the smoke test and the tests
(there is no dataset download on the build machines)."""
from __future__ import annotations

from typing import List, Tuple

import torch

from ..criterion.targets import Targets, pad_targets

__all__ = ["synthetic_batch", "synthetic_targets"]


def synthetic_targets(batch: int, gen: torch.Generator, kmin: int = 1, kmax: int = 10, num_labels: int = 80,
                      slots: int = None) -> Targets:
    per = []
    for _ in range(batch):
        k = int(torch.randint(kmin, kmax + 1, (1,), generator=gen))
        c = torch.rand(k, 2, generator=gen) * 0.8 + 0.1
        wh = torch.rand(k, 2, generator=gen) * 0.38 + 0.02
        per.append({"boxes": torch.cat([c, wh], 1), "labels": torch.randint(0, num_labels, (k,), generator=gen)})
    return pad_targets(per, slots=slots if slots is not None else kmax)


def synthetic_batch(batch: int, resolution: int, seed: int = 0, kmin: int = 1, kmax: int = 10,
                    num_labels: int = 80, slots: int = None, dtype=torch.float32) -> Tuple[torch.Tensor, Targets]:
    gen = torch.Generator().manual_seed(seed)
    images = torch.randn(batch, 3, resolution, resolution, generator=gen).to(dtype)
    return images, synthetic_targets(batch, gen, kmin, kmax, num_labels, slots)
