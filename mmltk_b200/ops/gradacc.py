"""In-place parameter-gradient accumulation for the framework's backward kernels.

When a parameter's ``.grad`` is already allocated -- the training engine binds
every ``.grad`` to a view of one flat gradient buffer -- a backward kernel can
add its result straight into it (GEMM with beta = 1, column reductions with an
accumulate flag) and return ``None`` to autograd.  That removes autograd's
separate AccumulateGrad add (one extra read + write of every gradient, and a
launch per parameter) from every step.  Semantics are those of AccumulateGrad:
the gradient is summed into ``.grad``.
"""
from __future__ import annotations

import torch

__all__ = ["grad_target"]


def grad_target(p) -> "torch.Tensor | None":
    """``p.grad`` when a backward kernel may accumulate into it in place, else None."""
    if p is None or not isinstance(p, torch.nn.Parameter) or not p.requires_grad:
        return None
    g = p.grad
    if g is None or g.dtype != p.dtype or g.shape != p.shape or not g.is_contiguous() or not g.is_cuda:
        return None
    return g
