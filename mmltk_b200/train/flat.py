"""Flat parameter / gradient storage.

All trainable parameters live in ONE bf16 buffer (each parameter a 64-element
aligned view), and their ``.grad`` tensors are views into ONE bf16 gradient
buffer, so the optimizer, the gradient norm, the DDP reduce-scatter /
all-gather and the EMA each touch memory with a single launch instead of one
per tensor.  fp32 master weights, Adam moments and the EMA shadow are flat
fp32 buffers with the same layout.  Parameters of one optimizer group are
contiguous, and the group boundaries are described by a chunk table
(offset, length, group) consumed by the fused kernels.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Tuple

import torch

__all__ = ["FlatParams", "ALIGN"]

ALIGN = 64          # elements (128 bytes of bf16)
CHUNK = 1 << 13     # max elements per chunk-table entry (small: the optimizer's blocks stride over
                    # chunks, so large tensors split into many chunks keep the blocks balanced)


def _round(n: int, a: int = ALIGN) -> int:
    return (n + a - 1) // a * a


class FlatParams:
    def __init__(self, named_params: Sequence[Tuple[str, torch.nn.Parameter]], group_of: Sequence[int],
                 device, dtype=torch.bfloat16, pad_to: int = 1, alloc=None, stage=None):
        # order parameters by group so every group is one contiguous range; with ``stage(name)``
        # (backward-completion stage, larger = complete earlier) by stage first, so the gradients
        # the backward pass completes together are one contiguous range (a data-parallel bucket)
        if stage is None:
            order = sorted(range(len(named_params)), key=lambda i: (group_of[i], i))
        else:
            order = sorted(range(len(named_params)), key=lambda i: (stage(named_params[i][0]), group_of[i], i))
        self.names: List[str] = []
        self.params: List[torch.nn.Parameter] = []
        self.offsets: List[int] = []
        self.numels: List[int] = []
        self.group_of: List[int] = []
        off = 0
        for i in order:
            name, p = named_params[i]
            self.names.append(name)
            self.params.append(p)
            self.offsets.append(off)
            self.numels.append(p.numel())
            self.group_of.append(group_of[i])
            off += _round(p.numel())
        self.total = _round(off, max(ALIGN, pad_to))
        self.device = torch.device(device)
        self.dtype = dtype
        # `alloc(numel, dtype)` lets a gradient-sync backend place both buffers in
        # peer-visible memory (zero-initialised)
        if alloc is None:
            alloc = lambda n, dt: torch.zeros(n, dtype=dt, device=self.device)  # noqa: E731
        self.param_buf = alloc(self.total, dtype)
        self.grad_buf = alloc(self.total, dtype)
        with torch.no_grad():
            for p, o, n in zip(self.params, self.offsets, self.numels):
                self.param_buf[o:o + n].copy_(p.detach().reshape(-1))
        self.bind()

    def view(self, buf: torch.Tensor, i: int) -> torch.Tensor:
        o, n = self.offsets[i], self.numels[i]
        return buf[o:o + n].view(self.params[i].shape)

    def bind(self) -> None:
        """Point every parameter's data and grad at the flat buffers."""
        for i, p in enumerate(self.params):
            p.data = self.view(self.param_buf, i)
            p.grad = self.view(self.grad_buf, i)

    def zero_grad(self) -> None:
        self.grad_buf.zero_()

    def chunk_table(self) -> torch.Tensor:
        """int64 [n,3] (offset, padded length, group) covering every parameter slot."""
        rows = []
        for o, n, g in zip(self.offsets, self.numels, self.group_of):
            L = _round(n)
            s = 0
            while s < L:
                ln = min(CHUNK, L - s)
                rows.append((o + s, ln, g))
                s += ln
        return torch.tensor(rows, dtype=torch.int64)

    def group_ranges(self) -> Dict[int, Tuple[int, int]]:
        out: Dict[int, Tuple[int, int]] = {}
        for o, n, g in zip(self.offsets, self.numels, self.group_of):
            a, b = out.get(g, (o, o + _round(n)))
            out[g] = (min(a, o), max(b, o + _round(n)))
        return out

    def master_fp32(self) -> torch.Tensor:
        return self.param_buf.float()

    def state_dict_tensors(self, buf: torch.Tensor) -> Dict[str, torch.Tensor]:
        return {n: self.view(buf, i) for i, n in enumerate(self.names)}
