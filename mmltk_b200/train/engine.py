"""One training step on one device: forward, matcher, losses, backward and the
optimizer update -- eager or replayed from a CUDA graph.

Reference step (`src/rfdetr/training/train.cpp:2287-2458`): autocast forward,
`detection_loss_dict`, `backward`, `average_gradients` (NCCL), finite check,
`clip_grad_norm_(0.1)`, fused AdamW, EMA update, with one host sync per
optimizer step for the metrics.

B200 design:
* parameters are bf16 views into one flat buffer; fp32 master weights, Adam
  moments and the EMA shadow are flat fp32 buffers; gradients accumulate in
  place into one flat bf16 buffer;
* the matcher and every loss stay on the device, so the whole step (including
  the optimizer kernels and, for DDP, the gradient collective) is captured once
  into a CUDA graph and replayed; the host only refreshes the per-step
  scalars (lr scale, bias corrections, EMA decay) with one async copy and reads
  back the loss + status flags once per step;
* the optimizer is the fused grad-norm + AdamW + EMA kernel pair (one pass
  over memory).  With DDP the gradient reduction is delegated to a
  ``GradientSync`` (fused in-kernel NVSwitch reduce-scatter/all-gather, or the
  NCCL baseline).
"""
from __future__ import annotations

import math
import time
from typing import Callable, Dict, List, Optional

import torch

from ..config import TrainOptions, lr_scale
from ..criterion import SetCriterion, Targets
from ..ops._ext import kernels
from .flat import FlatParams
from .param_groups import build_param_groups

__all__ = ["TrainEngine", "StepResult", "PendingStep"]


class StepResult:
    __slots__ = ("loss", "losses", "grad_norm", "nonfinite")

    def __init__(self, loss, losses, grad_norm, nonfinite):
        self.loss, self.losses, self.grad_norm, self.nonfinite = loss, losses, grad_norm, nonfinite


class PendingStep:
    """Handle of a step queued by ``TrainEngine.step_async``."""
    __slots__ = ("engine", "rb", "event", "partial", "step", "_done", "_slot", "_gen")

    def __init__(self, engine, rb, event, partial: StepResult):
        self.engine, self.rb, self.event, self.partial = engine, rb, event, partial
        self.step = engine.step_count
        self._done = partial if rb is None else None
        # which pinned readback slot holds this step's values, and that slot's use count then
        self._slot, self._gen = (engine._rb_last if rb is not None else (None, None))

    def ready(self) -> bool:
        return self._done is not None or self.event.query()

    def result(self) -> StepResult:
        if self._done is None:
            self.event.synchronize()
            if self.engine._rb_gen[self._slot] != self._gen:
                raise RuntimeError(
                    f"step {self.step}'s readback slot was reused by a later step: at most "
                    f"{len(self.engine._readbacks) - 1} more steps may be queued before result() is called")
            self._done = self.engine._read_result(self.rb, self.partial.losses, self.step)
        return self._done


class TrainEngine:
    def __init__(self, model: torch.nn.Module, opts: TrainOptions, device, grad_sync=None,
                 max_targets: int = 100, steps_per_epoch: int = 1, total_steps: int = 1):
        self.model = model
        self.cfg = model.cfg
        self.opts = opts
        self.device = torch.device(device)
        self.cuda = self.device.type == "cuda"
        self.grad_sync = grad_sync
        self.world = grad_sync.world_size if grad_sync is not None else 1
        self.max_targets = max_targets
        self.steps_per_epoch = max(1, steps_per_epoch)
        self.total_steps = max(1, total_steps)
        self.step_count = 0
        if opts.freeze_encoder:
            for n, p in model.named_parameters():
                if "backbone.0.encoder" in n:
                    p.requires_grad_(False)
        named = [(n, p) for n, p in model.named_parameters() if p.requires_grad]
        nvit = getattr(self.cfg, "vit_depth", 12) + 1
        self.groups, assign = build_param_groups(named, opts, nvit)
        self.criterion = SetCriterion(self.cfg, self.world,
                                      grad_sync.all_reduce_small if grad_sync is not None else None)
        if self.cuda:
            self._init_cuda(named, assign)
        else:
            self._init_cpu(named, assign)
        self.graph = None
        self._graph_warmup = 0
        # micro-batches per optimizer step: --grad-accum-steps x --lanes (the reference's lanes are
        # that many batches whose gradients are summed before one step, each loss scaled by
        # 1/(lanes * accum); here they run one after another on one stream, each a graph replay)
        self.accum = opts.micro_batches_per_step()
        self._micro = 0
        self._acc_graphs = {}      # "first" / "mid" / "last" micro-batch graphs (accumulation)
        self._pool = None

    # ------------------------------------------------------------------ setup
    def _init_cpu(self, named, assign):
        self.model.to(self.device)
        pgs = [{"params": [], "lr": g["lr"], "weight_decay": g["weight_decay"]} for g in self.groups]
        for (n, p), gi in zip(named, assign):
            pgs[gi]["params"].append(p)
        self.optimizer = torch.optim.AdamW(pgs, betas=(0.9, 0.999), eps=1e-8)
        self.base_lrs = [g["lr"] for g in self.groups]
        self.muon = None
        if self.opts.optimizer == "muon":
            from .muon import MuonAux
            self.muon = MuonAux([n for n, _ in named], [p.data for _, p in named], assign, self.groups,
                                self.opts.momentum)
        self.ema = [p.detach().clone() for _, p in named] if self.opts.use_ema else None
        self.ema_named = [n for n, _ in named]
        self.params = [p for _, p in named]

    def _init_cuda(self, named, assign):
        k = kernels()
        pad = self.grad_sync.pad_multiple if self.grad_sync is not None else 1
        fp32 = {n: p.detach().float().clone() for n, p in named}
        self.model.to(self.device, torch.bfloat16)
        named_dev = [(n, p) for n, p in self.model.named_parameters() if p.requires_grad]
        alloc = getattr(self.grad_sync, "alloc", None) if self.grad_sync is not None else None
        # a bucketed gradient sync wants the flat layout in backward-completion order
        stage = (getattr(self.model, "grad_stage", None)
                 if getattr(self.grad_sync, "bucketed", False) and self.opts.optimizer != "muon" else None)
        self.flat = FlatParams(named_dev, assign, self.device, torch.bfloat16, pad_to=pad, alloc=alloc, stage=stage)
        master = torch.zeros(self.flat.total, dtype=torch.float32, device=self.device)
        for i, n in enumerate(self.flat.names):
            o, c = self.flat.offsets[i], self.flat.numels[i]
            master[o:o + c].copy_(fp32[n].reshape(-1))
        self.master = master
        self.chunks = self.flat.chunk_table().to(self.device)
        self.group_hyper = torch.tensor([[g["lr"], g["weight_decay"]] for g in self.groups], dtype=torch.float32,
                                        device=self.device)
        nsc = k.step_scalar_floats()
        self.scalars_host = torch.zeros(nsc, dtype=torch.float32).pin_memory()
        self.scalars = torch.zeros(nsc, dtype=torch.float32, device=self.device)
        # per-step status words: [0] non-finite gradients, [1] gradient norm (fp32 bits),
        # [2] GPU assignment-solver status (non-zero: a bounded search gave up)
        self.flags = torch.zeros(3, dtype=torch.int32, device=self.device)
        self.criterion.match_status = self.flags[2:3]
        self.muon = None
        if self.opts.optimizer == "muon":
            # Muon runs eagerly on the master weights (fp32 views into the flat buffer)
            from .muon import MuonAux
            shapes = dict((n, p.shape) for n, p in named_dev)
            self.muon = MuonAux(self.flat.names, [self.flat.view(master, i).view(shapes[n])
                                                  for i, n in enumerate(self.flat.names)],
                                self.flat.group_of, self.groups, self.opts.momentum)
            self.m = self.v = None
            self.ema_buf = master.clone() if self.opts.use_ema else None
            self._alloc_readback()
            if self.grad_sync is not None:
                self.grad_sync.muon_mode = True
                if hasattr(self.grad_sync, "setup_replicated"):
                    # the fused sync as a gradient all-reduce over peer memory (replicated Muon)
                    self.grad_sync.setup_replicated(self)
            return
        if self.grad_sync is not None:
            self.grad_sync.setup(self)
        else:
            self.m = torch.zeros_like(master)
            self.v = torch.zeros_like(master)
            self.ema_buf = master.clone() if self.opts.use_ema else None
            self.scratch = torch.zeros(k.optim_num_partials(), dtype=torch.float32, device=self.device)
        self._alloc_readback()

    def _alloc_readback(self) -> None:
        # a ring of pinned readback slots: a deferred step's values stay readable while up to
        # three more steps are queued behind it
        self._readbacks = [torch.zeros(5, dtype=torch.float32).pin_memory() for _ in range(4)]
        self._rb_gen = [0] * len(self._readbacks)
        self._rb_last = (0, 0)
        self._rb_turn = 0
        self.readback = self._readbacks[0]

    # ------------------------------------------------------------------ scalars
    def _host_scalars(self, step: int):
        o = self.opts
        t = step + 1
        s = lr_scale(o, step, self.steps_per_epoch, self.total_steps)
        d = o.ema_decay * (1 - math.exp(-(step + 1) / o.ema_tau)) if o.ema_tau > 0 else o.ema_decay
        return [s, 0.9, 0.999, 1e-8, 1 - 0.9 ** t, 1 - 0.999 ** t, o.clip_max_norm, d,
                1.0 if o.use_ema else 0.0, 1.0 / self.world]

    # ------------------------------------------------------------------ body
    def _forward_loss(self, images: torch.Tensor, targets: Targets):
        out = self.model(images)
        losses, _ = self.criterion(out, targets, training=True)
        total = self.criterion.weighted(losses)
        return total, losses

    def _cuda_body(self, images, targets, first: bool = True, last: bool = True):
        if first:
            self.flags.zero_()
            self.flat.zero_grad()
        total, losses = self._forward_loss(images, targets)
        if last and self.muon is None and hasattr(self.grad_sync, "arm"):
            self.grad_sync.arm()     # this backward's gradient marks start the bucket reduce-scatters
        (total / self.accum if self.accum > 1 else total).backward()
        if not last:
            return total.detach(), {k: v.detach() for k, v in losses.items()}
        if self.muon is not None:
            self._muon_update()
        elif self.grad_sync is not None:
            self.grad_sync.step(self)
        else:
            kernels().adamw_ema_step(self.chunks, self.group_hyper, self.scalars, self.flat.grad_buf, self.master,
                                     self.m, self.v, self.ema_buf, self.flat.param_buf, self.scratch, self.flags)
        return total.detach(), {k: v.detach() for k, v in losses.items()}

    def _muon_update(self) -> None:
        """Eager Muon step on the flat buffers: all-reduce, clip, Muon/AdamW on the fp32
        master, bf16 parameter refresh, EMA."""
        from ..config import warmup_momentum
        o = self.opts
        g = self.flat.grad_buf
        if self.grad_sync is not None:
            if hasattr(self.grad_sync, "all_reduce_grads"):
                self.grad_sync.all_reduce_grads(self)      # in-kernel, over NVSwitch peer memory
            else:
                torch.distributed.all_reduce(g, group=self.grad_sync.group)
        gf = g.float()
        if self.world > 1:
            gf.div_(self.world)
        norm = gf.norm()
        self.flags[0:1].copy_((~torch.isfinite(norm)).to(torch.int32).reshape(1))
        self.flags[1:2].copy_(norm.reshape(1).view(torch.int32))
        if o.clip_max_norm > 0:
            gf.mul_((o.clip_max_norm / (norm + 1e-6)).clamp(max=1.0))
        grads = [self.flat.view(gf, i) for i in range(len(self.flat.names))]
        s = lr_scale(o, self.step_count, self.steps_per_epoch, self.total_steps)
        mom = warmup_momentum(o, self.step_count, self.steps_per_epoch, o.momentum)
        self.muon.step(grads, s, mom)
        self.flat.param_buf.copy_(self.master)
        if self.ema_buf is not None:
            d = o.ema_decay * (1 - math.exp(-(self.step_count + 1) / o.ema_tau)) if o.ema_tau > 0 else o.ema_decay
            self.ema_buf.mul_(d).add_(self.master, alpha=1 - d)

    # ------------------------------------------------------------------ public
    def bind_static_inputs(self, batch: int, channels: int, height: int, width: int) -> None:
        dev = self.device
        self.in_images = torch.zeros(batch, channels, height, width, dtype=torch.bfloat16, device=dev)
        T = self.max_targets
        self.in_targets = Targets(torch.full((batch, T, 4), 0.5, device=dev), torch.zeros(batch, T, dtype=torch.int64,
                                  device=dev), torch.ones(batch, dtype=torch.int32, device=dev), [1] * batch)

    def load_inputs(self, images: torch.Tensor, targets: Targets) -> None:
        """Copy one batch (pinned host or device tensors) into the static input buffers."""
        self.in_images.copy_(images, non_blocking=True)
        t = self.in_targets
        T = targets.slots
        if T > t.slots:
            raise ValueError(f"batch has {T} target slots, engine was built for {t.slots}")
        t.boxes[:, :T].copy_(targets.boxes, non_blocking=True)
        t.labels[:, :T].copy_(targets.labels, non_blocking=True)
        if T < t.slots:
            t.boxes[:, T:].fill_(0.5)
            t.labels[:, T:].zero_()
        t.counts.copy_(targets.counts, non_blocking=True)
        t.counts_host = list(targets.counts_host)
        # segmentation targets: the mask rows change size with every batch, so they are
        # passed through (and such steps run eagerly, outside the captured graph)
        t.masks = None if targets.masks is None else targets.masks.to(self.device, non_blocking=True)
        t.mask_offsets = targets.mask_offsets

    def step(self, images: Optional[torch.Tensor] = None, targets: Optional[Targets] = None,
             sync: bool = True) -> StepResult:
        """One optimizer step.  On CUDA, inputs are copied into the static buffers first
        (pass None to reuse what is already there)."""
        if not self.cuda:
            return self._cpu_step(images, targets)
        if images is not None:
            self.load_inputs(images, targets)
        if self.accum > 1:
            # micro-batch: forward + backward into the flat gradient, optimizer on the last one;
            # after three eager optimizer steps each micro-batch kind is a graph replay
            first, last = self._micro == 0, self._micro == self.accum - 1
            self._micro = 0 if last else self._micro + 1
            if last:
                sc = self._host_scalars(self.step_count)
                self.scalars_host[:len(sc)] = torch.tensor(sc)
                self.scalars.copy_(self.scalars_host, non_blocking=True)
            if (self.opts.cuda_graph and self._graph_warmup >= 3 and self.in_targets.masks is None
                    and self.muon is None):
                kind = "last" if last else ("first" if first else "mid")
                g = self._acc_graphs.get(kind)
                if g is None:
                    g = self._capture_micro(first, last)
                    self._acc_graphs[kind] = g
                g[0].replay()
                total, losses = g[1], g[2]
            else:
                total, losses = self._cuda_body(self.in_images, self.in_targets, first=first, last=last)
                if last:
                    self._graph_warmup += 1
            if not last:
                return StepResult(total, losses, None, None)
            return self._finish(total, losses, sync)
        sc = self._host_scalars(self.step_count)
        self.scalars_host[:len(sc)] = torch.tensor(sc)
        self.scalars.copy_(self.scalars_host, non_blocking=True)
        if (self.opts.cuda_graph and self._graph_warmup >= 3 and self.in_targets.masks is None
                and self.muon is None):
            if self.graph is None:
                self._capture()
            self.graph.replay()
            total, losses = self.static_total, self.static_losses
        else:
            total, losses = self._cuda_body(self.in_images, self.in_targets)
            self._graph_warmup += 1
        return self._finish(total, losses, sync)

    def step_async(self, images: Optional[torch.Tensor] = None, targets: Optional[Targets] = None) -> "PendingStep":
        """Queue one optimizer step and its loss/flag readback without waiting; ``.result()`` on the
        returned handle waits for that step only.  The host can prepare the next batch meanwhile.
        (The reference trainer reads its loss synchronously every step: rfdetr/src/engine.cpp.)"""
        if not self.cuda:
            return PendingStep(self, None, None, self.step(images, targets))
        r = self.step(images, targets, sync=False)
        if self.accum > 1 and self._micro != 0:
            return PendingStep(self, None, None, r)        # a micro-batch: nothing to read yet
        rb = self._queue_readback(r.loss)
        ev = torch.cuda.Event()
        ev.record()
        return PendingStep(self, rb, ev, StepResult(None, r.losses, None, None))

    def _queue_readback(self, total) -> torch.Tensor:
        slot = self._rb_turn
        rb = self._readbacks[slot]
        self._rb_gen[slot] += 1
        self._rb_last = (slot, self._rb_gen[slot])
        self._rb_turn = (self._rb_turn + 1) % len(self._readbacks)
        rb[0:1].copy_(total.reshape(1), non_blocking=True)
        rb[1:4].copy_(self.flags.view(torch.float32), non_blocking=True)
        sync_status = getattr(self.grad_sync, "status_tensor", None)
        if sync_status is not None:
            rb[4:5].copy_(sync_status().view(torch.float32), non_blocking=True)
        return rb

    def _read_result(self, rb: torch.Tensor, losses, step: int) -> StepResult:
        if getattr(self.grad_sync, "status_tensor", None) is not None:
            self.grad_sync.check(self.flags_host_bits(rb[4]))
        loss = float(rb[0])
        nonfinite = int(self.flags_host_bits(rb[1]))
        norm = float(rb[2])
        match_status = int(self.flags_host_bits(rb[3]))
        if self.cuda and kernels().debug_build():
            # debug-bounds build: the step's index checks (one read of the status words per step)
            code = int(kernels().debug_status())
            if code:
                raise RuntimeError(f"debug bounds check failed at step {step}: code {code:#x} "
                                   "(an input index outside its table; see MMLTK_DEBUG_CHECK codes)")
        if match_status:
            raise RuntimeError(f"GPU Hungarian matcher gave up on a bounded search at step {step} "
                               f"(status {match_status}); the assignment would be partial")
        if nonfinite or not math.isfinite(loss):
            raise FloatingPointError(f"non-finite RF-DETR loss ({loss}) or gradients (norm {norm}) at step {step}")
        return StepResult(loss, losses, norm, nonfinite)

    def _finish(self, total, losses, sync: bool) -> StepResult:
        self.step_count += 1
        if self.grad_sync is not None:
            self.grad_sync.after_step(self)
        if not sync:
            return StepResult(total, losses, None, None)
        rb = self._queue_readback(total)
        torch.cuda.current_stream().synchronize()
        return self._read_result(rb, losses, self.step_count)

    @staticmethod
    def flags_host_bits(x: torch.Tensor) -> int:
        return int(x.view(torch.int32).item())

    def release_graph(self) -> None:
        """Drop the captured graphs (required before destroying a process group they use)."""
        if self.graph is not None or self._acc_graphs:
            torch.cuda.synchronize()
        if self.graph is not None:
            self.graph.reset()
            self.graph = None
            self.static_total = self.static_losses = None
            self._graph_warmup = 0
        for g in self._acc_graphs.values():
            g[0].reset()
        self._acc_graphs = {}

    def _capture(self):
        stream = torch.cuda.current_stream()
        self.graph = torch.cuda.CUDAGraph()
        torch.cuda.synchronize()
        with torch.cuda.graph(self.graph, stream=torch.cuda.Stream()):
            self.static_total, self.static_losses = self._cuda_body(self.in_images, self.in_targets)
        stream.wait_stream(stream)

    def _capture_micro(self, first: bool, last: bool):
        """One accumulation micro-batch kind as a graph.  The kinds never run concurrently, so they
        share one memory pool: their activations reuse the same memory."""
        if self._pool is None:
            self._pool = torch.cuda.graph_pool_handle()
        g = torch.cuda.CUDAGraph()
        torch.cuda.synchronize()
        with torch.cuda.graph(g, pool=self._pool, stream=torch.cuda.Stream()):
            total, losses = self._cuda_body(self.in_images, self.in_targets, first=first, last=last)
        return g, total, losses

    def _cpu_step(self, images, targets) -> StepResult:
        o = self.opts
        s = lr_scale(o, self.step_count, self.steps_per_epoch, self.total_steps)
        for g, base in zip(self.optimizer.param_groups, self.base_lrs):
            g["lr"] = base * s
        first, last = self._micro == 0, self._micro == self.accum - 1
        self._micro = 0 if last else self._micro + 1
        if first:
            self.optimizer.zero_grad(set_to_none=True)
        total, losses = self._forward_loss(images, targets)
        if last and self.muon is None and hasattr(self.grad_sync, "arm"):
            self.grad_sync.arm()     # this backward's gradient marks start the bucket reduce-scatters
        (total / self.accum if self.accum > 1 else total).backward()
        if not last:
            return StepResult(float(total.detach()),{k: v.detach() for k, v in losses.items()}, None, 0)
        if self.grad_sync is not None:
            self.grad_sync.cpu_average(self.params)
        norm = torch.nn.utils.clip_grad_norm_(self.params, o.clip_max_norm) if o.clip_max_norm > 0 else None
        if not torch.isfinite(total) or (norm is not None and not torch.isfinite(norm)):
            raise FloatingPointError(f"non-finite RF-DETR loss or gradients at step {self.step_count}")
        if self.muon is not None:
            from ..config import warmup_momentum
            zeros = [torch.zeros_like(p) for p in self.params]
            self.muon.step([p.grad if p.grad is not None else z for p, z in zip(self.params, zeros)], s,
                           warmup_momentum(o, self.step_count, self.steps_per_epoch, o.momentum))
        else:
            self.optimizer.step()
        if self.ema is not None:
            d = o.ema_decay * (1 - math.exp(-(self.step_count + 1) / o.ema_tau)) if o.ema_tau > 0 else o.ema_decay
            with torch.no_grad():
                torch._foreach_mul_(self.ema, d)
                torch._foreach_add_(self.ema, [p.detach() for p in self.params], alpha=1 - d)
        self.step_count += 1
        return StepResult(float(total.detach()),{k: v.detach() for k, v in losses.items()},
                          None if norm is None else float(norm), 0)

    # ------------------------------------------------------------------ state
    def ema_state(self) -> Optional[Dict[str, torch.Tensor]]:
        if not self.cuda:
            return None if self.ema is None else {n: t for n, t in zip(self.ema_named, self.ema)}
        buf = self.grad_sync.gather_ema(self) if self.grad_sync is not None else self.ema_buf
        return None if buf is None else self.flat.state_dict_tensors(buf)

    # flat fp32 buffers, full length, on this device ("master", "m", "v", "ema"); sharded copies are gathered
    def _full(self, which: str) -> Optional[torch.Tensor]:
        sharded = getattr(self, "master_shard", None) is not None and self.master is None
        local = {"master": self.master_shard if sharded else self.master, "m": self.m, "v": self.v,
                 "ema": self.ema_buf}[which]
        if local is None:
            return None
        return self.grad_sync.gather_full(local) if sharded else local

    def export_model(self, which: str = "master") -> torch.nn.Module:
        """An fp32 CPU copy of the model holding the master (or EMA) weights -- for checkpoints
        and evaluation; its ``state_dict()`` has the checkpoint key layout."""
        import copy
        if not self.cuda:
            m = copy.deepcopy(self.model).float()
            if which == "ema" and self.ema is not None:
                named = dict(m.named_parameters())
                with torch.no_grad():
                    for n, t in zip(self.ema_named, self.ema):
                        named[n].copy_(t)
            return m
        buf = self._full("ema" if which == "ema" else "master")
        if buf is None:
            raise ValueError(f"no {which} weights (EMA disabled?)")
        host = buf.float().cpu()
        m = copy.deepcopy(self.model).to("cpu", torch.float32)
        named = dict(m.named_parameters())
        with torch.no_grad():
            for i, n in enumerate(self.flat.names):
                o, c = self.flat.offsets[i], self.flat.numels[i]
                named[n].copy_(host[o:o + c].view_as(named[n]))
        return m

    def optimizer_state(self) -> dict:
        """Per-parameter optimizer state in a world-size independent layout (archive-ready dict)."""
        if self.muon is not None:
            d = self.muon.state_dict()
            d["step"] = int(self.step_count)
            return d
        d = {"kind": "adamw", "step": int(self.step_count)}
        if not self.cuda:
            names = [n for n, _ in zip(self.ema_named, self.params)]
            for i, (n, p) in enumerate(zip(names, self.params)):
                st = self.optimizer.state.get(p, {})
                e = {"name": n}
                if st:
                    e["exp_avg"] = st["exp_avg"].detach().cpu()
                    e["exp_avg_sq"] = st["exp_avg_sq"].detach().cpu()
                d[f"entry_{i:06d}"] = e
            d["entry_count"] = len(names)
            return d
        m, v = self._full("m").cpu(), self._full("v").cpu()
        for i, n in enumerate(self.flat.names):
            o, c = self.flat.offsets[i], self.flat.numels[i]
            d[f"entry_{i:06d}"] = {"name": n, "exp_avg": m[o:o + c].clone(), "exp_avg_sq": v[o:o + c].clone()}
        d["entry_count"] = len(self.flat.names)
        return d

    def load_optimizer_state(self, d: dict) -> None:
        if self.muon is not None:
            self.muon.load_state_dict(d)
            self.step_count = int(d["step"])
            return
        if d.get("kind") != "adamw":
            raise ValueError(f"resume: optimizer kind {d.get('kind')!r} does not match 'adamw'")
        entries = {d[f"entry_{i:06d}"]["name"]: d[f"entry_{i:06d}"] for i in range(int(d["entry_count"]))}
        self.step_count = int(d["step"])
        if not self.cuda:
            for n, p in zip(self.ema_named, self.params):
                e = entries.get(n)
                if e is None or "exp_avg" not in e:
                    continue
                self.optimizer.state[p] = {"step": torch.tensor(float(self.step_count)),
                                           "exp_avg": e["exp_avg"].to(p.device).view_as(p).clone(),
                                           "exp_avg_sq": e["exp_avg_sq"].to(p.device).view_as(p).clone()}
            return
        full_m = torch.zeros(self.flat.total, dtype=torch.float32)
        full_v = torch.zeros(self.flat.total, dtype=torch.float32)
        for i, n in enumerate(self.flat.names):
            e = entries.get(n)
            if e is None:
                raise ValueError(f"resume: optimizer state has no entry for {n}")
            o, c = self.flat.offsets[i], self.flat.numels[i]
            full_m[o:o + c] = e["exp_avg"].reshape(-1)
            full_v[o:o + c] = e["exp_avg_sq"].reshape(-1)
        sharded = getattr(self, "master_shard", None) is not None and self.master is None
        if sharded:
            self.m.copy_(self.grad_sync.shard_of(full_m))
            self.v.copy_(self.grad_sync.shard_of(full_v))
        else:
            self.m.copy_(full_m)
            self.v.copy_(full_v)

    def load_ema_state(self, state: Dict[str, torch.Tensor]) -> None:
        """EMA shadow from a name -> tensor dict keyed by parameter names."""
        if not self.cuda:
            if self.ema is None:
                return
            with torch.no_grad():
                for n, t in zip(self.ema_named, self.ema):
                    if n in state:
                        t.copy_(state[n].view_as(t))
            return
        if self.ema_buf is None:
            return
        full = torch.zeros(self.flat.total, dtype=torch.float32)
        for i, n in enumerate(self.flat.names):
            o, c = self.flat.offsets[i], self.flat.numels[i]
            if n in state:
                full[o:o + c] = state[n].reshape(-1).float()
        sharded = getattr(self, "master_shard", None) is not None and self.master is None
        if sharded:
            self.ema_buf.copy_(self.grad_sync.shard_of(full))
        else:
            self.ema_buf.copy_(full)
