"""Data-parallel gradient synchronisation.

Two interchangeable ``GradSync`` implementations plug into ``TrainEngine``:

* ``NcclGradSync`` -- the baseline with the reference's semantics
  (`src/rfdetr/training/train.cpp:876-887,1389-1410`): one all-reduce of every
  gradient after the full backward, then the (replicated) optimizer.  Here the
  all-reduce runs over the flat bf16 gradient buffer in one NCCL call.
* ``FusedGradSync`` (``mmltk_b200.parallel.fused``) -- the product path: an
  in-kernel reduce-scatter over NVSwitch peer memory fused with the gradient
  average, the global-norm clip, the sharded AdamW update and the EMA update,
  followed by an in-kernel all-gather of the updated bf16 parameters.

Both also provide the small all-reduce the criterion uses for ``num_boxes``
(device tensor, no host sync; reference `detection_ops.cpp:1501-1510`).
"""
from __future__ import annotations

from typing import List

import torch
import torch.distributed as dist

from ..ops._ext import kernels

__all__ = ["NcclGradSync"]


class NcclGradSync:
    pad_multiple = 1

    def __init__(self, group=None):
        self.group = group
        self.world_size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def setup(self, engine) -> None:
        k = kernels()
        engine.m = torch.zeros_like(engine.master)
        engine.v = torch.zeros_like(engine.master)
        engine.ema_buf = engine.master.clone() if engine.opts.use_ema else None
        engine.scratch = torch.zeros(k.optim_num_partials(), dtype=torch.float32, device=engine.device)

    def all_reduce_small(self, t: torch.Tensor) -> torch.Tensor:
        dist.all_reduce(t, group=self.group)
        return t

    def step(self, engine) -> None:
        dist.all_reduce(engine.flat.grad_buf, group=self.group)
        kernels().adamw_ema_step(engine.chunks, engine.group_hyper, engine.scalars, engine.flat.grad_buf,
                                 engine.master, engine.m, engine.v, engine.ema_buf, engine.flat.param_buf,
                                 engine.scratch, engine.flags)

    def after_step(self, engine) -> None:
        pass

    def gather_ema(self, engine):
        return engine.ema_buf

    def cpu_average(self, params: List[torch.Tensor]) -> None:
        grads = [p.grad for p in params if p.grad is not None]
        if not grads:
            return
        flat = torch.cat([g.reshape(-1) for g in grads])
        dist.all_reduce(flat, group=self.group)
        flat /= self.world_size
        o = 0
        for g in grads:
            n = g.numel()
            g.copy_(flat[o:o + n].view_as(g))
            o += n
