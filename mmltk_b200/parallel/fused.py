"""Fused in-kernel data-parallel gradient step over NVSwitch peer memory.

Per step (two kernels, replayed from the engine's CUDA graph):

1. ``rs``: barrier on "gradients ready", then every rank reduces ITS shard of
   the flat bf16 gradient buffer by reading that shard from every peer's buffer
   over NVLink (16-byte P2P loads, fp32 accumulation in rank order) and
   publishes the shard's sum of squares to every rank;
2. ``update``: every rank combines the N sums of squares into the global norm
   of the averaged gradient (same value on every rank), clips, runs AdamW on
   its fp32 master shard (ZeRO-1: moments and master weights are sharded),
   updates its EMA shard and writes the new bf16 parameters straight into
   every peer's parameter buffer (P2P stores = all-gather), then waits until
   every peer has delivered its shard.

The reference instead all-reduces every fp32 gradient with NCCL after the
whole backward and runs a replicated optimizer on every rank
(`src/rfdetr/training/train.cpp:876-887,1389-1410`).

Peer buffers are plain ``cudaMalloc`` allocations exported with CUDA IPC and
mapped by every other rank (one process per GPU, one node).  ``torch.distributed``
is only used for the one-time handle exchange and the initial broadcast.
Every device-side wait is bounded (``spin_limit`` polls); a rank that never
arrives makes its peers' kernels return with a non-zero status that
``check()`` turns into an exception -- no GPU is left spinning.
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist

from ..ops._ext import kernels

__all__ = ["FusedGradSync", "shard_chunks"]

ERRORS = {1: "a peer never signalled 'gradients ready'", 2: "a peer never published its gradient norm",
          3: "a peer never delivered its parameter shard", 4: "a peer never joined the small all-reduce",
          5: "a peer never joined the byte all-gather"}


def shard_chunks(chunks: torch.Tensor, off: int, size: int) -> torch.Tensor:
    """Intersect the global (offset, length, group) table with [off, off+size); shard-local offsets."""
    rows = []
    for o, n, g in chunks.tolist():
        a, b = max(o, off), min(o + n, off + size)
        if a < b:
            rows.append((a - off, b - a, g))
    if not rows:
        rows.append((0, 0, 0))
    return torch.tensor(rows, dtype=torch.int64)


class FusedGradSync:
    def __init__(self, group=None, spin_limit: int = 1 << 26):
        self.group = group
        self.world_size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.pad_multiple = self.world_size * 64
        self.spin_limit = int(spin_limit)
        self.device = torch.device("cuda", torch.cuda.current_device())
        self._handles: List[bytes] = []
        self._keep = []
        self._opened: List[int] = []
        self.failed: Optional[str] = None

    # ---------------------------------------------------------------- buffers
    def alloc(self, numel: int, dtype) -> torch.Tensor:
        es = torch.tensor([], dtype=dtype).element_size()
        raw, handle = kernels().ipc_alloc(numel * es, self.device.index)
        self._keep.append(raw)
        self._handles.append(handle)
        return raw.view(dtype)[:numel]

    def setup(self, engine) -> None:
        k = kernels()
        dev = self.device
        flags, fh = k.ipc_alloc(k.ddp_flag_words() * 4, dev.index)
        small, sh = k.ipc_alloc(k.ddp_small_floats() * 4, dev.index)
        self._keep += [flags, small]
        mine = [self._handles[0], self._handles[1], fh, sh]  # param, grad, flags, small
        everyone = [None] * self.world_size
        dist.all_gather_object(everyone, mine, group=self.group)
        local = [engine.flat.param_buf.data_ptr(), engine.flat.grad_buf.data_ptr(), flags.data_ptr(), small.data_ptr()]
        ptrs = [[0] * self.world_size for _ in range(4)]
        for j, hs in enumerate(everyone):
            for b in range(4):
                if j == self.rank:
                    ptrs[b][j] = local[b]
                else:
                    p = k.ipc_open(hs[b], dev.index)
                    self._opened.append(p)
                    ptrs[b][j] = p
        self.ctrl = torch.zeros(8, dtype=torch.int32, device=dev)
        self.ctrl[0] = 1       # step epoch
        self.ctrl[1] = 1       # small all-reduce epoch
        self.ctrl[4] = 1       # byte all-gather epoch
        self.comm = k.DdpComm(ptrs[1], ptrs[0], ptrs[2], ptrs[3], self.rank, self.world_size,
                              flags.view(torch.int32), small.view(torch.float32), self.ctrl, self.spin_limit)
        # identical starting point on every rank
        dist.broadcast(engine.flat.param_buf, 0, group=self.group)
        dist.broadcast(engine.master, 0, group=self.group)
        P = engine.flat.total
        S = P // self.world_size
        self.off, self.size = self.rank * S, S
        engine.master_shard = engine.master[self.off:self.off + S].clone()
        engine.master = None  # the full fp32 copy is only kept as shards
        engine.m = torch.zeros(S, dtype=torch.float32, device=dev)
        engine.v = torch.zeros(S, dtype=torch.float32, device=dev)
        engine.ema_buf = engine.master_shard.clone() if engine.opts.use_ema else None
        self.gshard = torch.zeros(S, dtype=torch.float32, device=dev)
        self.partials = torch.zeros(k.ddp_rs_blocks(), dtype=torch.float32, device=dev)
        self.chunks = shard_chunks(engine.flat.chunk_table(), self.off, S).to(dev)
        self._stage = engine.flat.grad_buf.view(torch.uint8)   # byte all-gather staging (between steps)
        dist.barrier(group=self.group)

    # ---------------------------------------------------------------- step
    def all_reduce_small(self, t: torch.Tensor) -> torch.Tensor:
        t = t.float().contiguous()
        self.comm.small_allreduce(t)
        return t

    def step(self, engine) -> None:
        if self.failed is not None:
            raise RuntimeError(f"fused DDP gradient step is unusable after an earlier failure: {self.failed}")
        self.comm.rs(self.off, self.size, self.gshard, self.partials)
        self.comm.update(self.off, self.chunks, self.gshard, engine.master_shard, engine.m, engine.v, engine.ema_buf,
                         engine.group_hyper, engine.scalars, engine.flags)

    def after_step(self, engine) -> None:
        pass

    def status_tensor(self) -> torch.Tensor:
        return self.ctrl[3:4]

    def check(self, code: int) -> None:
        """Raise if the step's kernels reported a status.  A timed-out wait leaves the kernels'
        arrival counters part-way through a step, so the sync cannot be used again: every later
        ``step`` raises too (recover by restarting the ranks and resuming from a checkpoint)."""
        if code:
            self.failed = (f"fused DDP step failed on rank {self.rank}: {ERRORS.get(code, code)} "
                           f"within the wait limit")
            raise RuntimeError(self.failed)

    def all_gather_tensor(self, t: torch.Tensor) -> List[torch.Tensor]:
        """Every rank's ``t`` (same dtype and trailing shape on every rank, any first dimension),
        in rank order, as CPU tensors.  Collective; runs between steps only: each rank stages its
        bytes in its own gradient buffer and every rank reads every peer's bytes straight out of
        that buffer over NVLink (16-byte loads), between two device-side barriers.  The next step
        clears the gradient buffer before it accumulates into it."""
        if self.failed is not None:
            raise RuntimeError(f"fused DDP sync is unusable after an earlier failure: {self.failed}")
        dev = self.device
        tail = tuple(t.shape[1:])
        raw = t.detach().contiguous().reshape(-1).view(torch.uint8)
        # 16-byte header with the exact byte count, then the payload padded to 16 bytes
        n = raw.numel()
        n16 = 1 + (n + 15) // 16
        if n16 >= (1 << 24):
            raise ValueError(f"all_gather_tensor: {n} bytes is above the 256 MB limit of one gather")
        if n16 * 16 > self._stage.numel():
            raise ValueError(f"all_gather_tensor: {n} bytes do not fit the {self._stage.numel()}-byte staging buffer")
        counts = torch.zeros(self.world_size, dtype=torch.float32, device=dev)
        counts[self.rank] = float(n16)        # exact: below 2^24
        self.comm.small_allreduce(counts)
        head = torch.zeros(16, dtype=torch.uint8)
        head[:8] = torch.tensor([n], dtype=torch.int64).view(torch.uint8)
        self._stage[:16].copy_(head.to(dev, non_blocking=False))
        if n:
            self._stage[16:16 + n].copy_(raw.to(dev))
        sizes = [int(c) for c in counts.cpu().tolist()]
        offs = [sum(sizes[:j]) for j in range(self.world_size)]
        out = torch.empty(sum(sizes) * 16, dtype=torch.uint8, device=dev)
        self.comm.gather_bytes(out, offs, sizes)
        host = out.cpu()
        self.check(int(self.ctrl[3].item()))
        parts = []
        for j in range(self.world_size):
            b = host[offs[j] * 16:(offs[j] + sizes[j]) * 16]
            nb = int(b[:8].view(torch.int64).item())
            parts.append(b[16:16 + nb].clone().view(t.dtype).reshape(-1, *tail))
        return parts

    # ---------------------------------------------------------------- state
    def gather_full(self, shard: torch.Tensor) -> torch.Tensor:
        out = torch.empty(shard.numel() * self.world_size, dtype=shard.dtype, device=shard.device)
        dist.all_gather_into_tensor(out, shard.contiguous(), group=self.group)
        return out

    def gather_ema(self, engine) -> Optional[torch.Tensor]:
        return None if engine.ema_buf is None else self.gather_full(engine.ema_buf)

    def gather_master(self, engine) -> torch.Tensor:
        return self.gather_full(engine.master_shard)

    def cpu_average(self, params) -> None:
        raise RuntimeError("the fused NVSwitch gradient step needs CUDA tensors")

    def close(self) -> None:
        k = kernels()
        for p in self._opened:
            k.ipc_close(p)
        self._opened = []
