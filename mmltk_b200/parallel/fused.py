"""Fused in-kernel data-parallel gradient step over NVSwitch peer memory.

Per step (kernels replayed from the engine's CUDA graph):

1. ``rs`` per gradient bucket: the flat gradient buffer is laid out in backward-completion order
   (``FlatParams(stage=...)``), so each bucket is one contiguous range.  When the backward pass
   reaches a ViT layer's input (``GradMark``), the bucket it completed is reduce-scattered on a
   side stream while the pass goes on: a barrier on "bucket ready", then every rank sums ITS slice
   of the bucket over every peer's buffer over NVLink (16-byte P2P loads, all peers' loads in
   flight at once, fp32 accumulation in rank order) into its fp32 shard, plus the slice's sum of
   squares.  The last bucket (patch / position embeddings and whatever no mark covered) runs after
   the backward pass;
2. ``publish``: the shard's sum of squares to every rank;
3. ``update``: every rank combines the N sums of squares into the global norm of the averaged
   gradient (same value on every rank), clips, runs AdamW on its fp32 master shard (ZeRO-1:
   moments and master weights are sharded), updates its EMA shard and writes the new bf16
   parameters straight into every peer's parameter buffer (16-byte P2P stores = all-gather),
   then waits until every peer has delivered its shard.

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

import os
from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from ..ops._ext import kernels

__all__ = ["FusedGradSync", "shard_chunks", "plan_buckets", "rank_slices"]

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


def plan_buckets(total: int, mark_bounds: List[int], min_elems: int) -> List[Tuple[Optional[int], int, int]]:
    """Buckets of a flat buffer laid out in backward-completion order (complete from the end).

    ``mark_bounds[i]``: flat offset from which every gradient is complete when backward reaches
    mark i (non-increasing in firing order, marks fire as i = len - 1 .. 0).  Returns
    [(mark or None, start, end)] in firing order; consecutive marks are merged until a bucket
    holds ``min_elems``; the last bucket (mark None) runs after the backward pass."""
    out: List[Tuple[Optional[int], int, int]] = []
    end = total
    for i in range(len(mark_bounds) - 1, -1, -1):
        b = mark_bounds[i]
        if end - b >= min_elems and len(out) < 30:
            out.append((i, b, end))
            end = b
    out.append((None, 0, end))
    return [t for t in out if t[2] > t[1]] or [(None, 0, total)]


def rank_slices(buckets: Sequence[Tuple[Optional[int], int, int]], world: int, rank: int) -> List[Tuple[int, int]]:
    """This rank's [a, b) of every bucket: the bucket cut into ``world`` 64-element-aligned parts."""
    out = []
    for _, s0, s1 in buckets:
        units = (s1 - s0) // 64
        a = s0 + (units * rank // world) * 64
        b = s0 + (units * (rank + 1) // world) * 64 if rank + 1 < world else s1
        out.append((a, b))
    return out


class FusedGradSync:
    # the flat buffer is laid out by backward-completion stage (the engine asks the model for it)
    bucketed = True

    def __init__(self, group=None, spin_limit: int = 1 << 26, overlap: Optional[bool] = None,
                 min_bucket: int = 4 << 20):
        self.group = group
        self.world_size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.pad_multiple = self.world_size * 64
        self.spin_limit = int(spin_limit)
        self.device = torch.device("cuda", torch.cuda.current_device())
        # reduce-scatter overlapped with the backward pass: off unless asked for (MMLTK_DDP_OVERLAP=1);
        # on two B200s it measured slower than one reduce-scatter after the backward pass
        self.overlap = (os.environ.get("MMLTK_DDP_OVERLAP", "0") == "1") if overlap is None else bool(overlap)
        self.min_bucket = int(min_bucket)
        self._handles: List[bytes] = []
        self._keep = []
        self._opened: List[int] = []
        self.failed: Optional[str] = None
        self._armed = False
        self._next = 0

    # ---------------------------------------------------------------- buffers
    def alloc(self, numel: int, dtype) -> torch.Tensor:
        es = torch.tensor([], dtype=dtype).element_size()
        raw, handle = kernels().ipc_alloc(numel * es, self.device.index)
        self._keep.append(raw)
        self._handles.append(handle)
        return raw.view(dtype)[:numel]

    def setup(self, engine) -> None:
        """Sharded mode: peer mappings, buckets, and ZeRO-1 shards of the master weights, Adam
        moments and EMA (this rank's slice of every bucket)."""
        dev = self.device
        self._connect(engine)
        # identical starting point on every rank
        dist.broadcast(engine.flat.param_buf, 0, group=self.group)
        dist.broadcast(engine.master, 0, group=self.group)
        self._plan(engine)
        flat = engine.flat
        S = self.size
        master = engine.master
        engine.master_shard = torch.cat([master[a:b] for a, b in self.slices]).contiguous()
        engine.master = None  # the full fp32 copy is only kept as shards
        engine.m = torch.zeros(S, dtype=torch.float32, device=dev)
        engine.v = torch.zeros(S, dtype=torch.float32, device=dev)
        engine.ema_buf = engine.master_shard.clone() if engine.opts.use_ema else None
        table = flat.chunk_table()
        rows, deltas = [], []
        for (a, b), lo in zip(self.slices, self.local_off):
            part = shard_chunks(table, a, b - a)
            for o, n, g in part.tolist():
                if n:
                    rows.append((lo + o, n, g))
                    deltas.append(a - lo)
        if not rows:
            rows, deltas = [(0, 0, 0)], [0]
        self.chunks = torch.tensor(rows, dtype=torch.int64, device=dev)
        self.gdelta = torch.tensor(deltas, dtype=torch.int64, device=dev)
        dist.barrier(group=self.group)

    def _connect(self, engine) -> None:
        """Exchange CUDA-IPC handles of the parameter / gradient / flag / small buffers and build the
        kernels' peer tables."""
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

    def setup_replicated(self, engine) -> None:
        """Gradient all-reduce only (optimizers that keep every full matrix, e.g. Muon): the same
        peer mappings and bucket reduce-scatter, then each rank's reduced slices written back into
        every rank's gradient buffer (``all_reduce_grads``); master weights stay replicated."""
        self._connect(engine)
        dist.broadcast(engine.flat.param_buf, 0, group=self.group)
        dist.broadcast(engine.master, 0, group=self.group)
        self._plan(engine)
        dist.barrier(group=self.group)

    def all_reduce_grads(self, engine) -> None:
        """Sum of every rank's bf16 gradient buffer, left in every rank's buffer (fp32 accumulation in
        rank order, rounded to bf16 once)."""
        if self.failed is not None:
            raise RuntimeError(f"fused DDP sync is unusable after an earlier failure: {self.failed}")
        cur = torch.cuda.current_stream(self.device)
        for j in range(len(self.buckets)):
            self._launch(j, cur)
        self.comm.grad_allgather([a for a, _ in self.slices], [b - a for a, b in self.slices], self.local_off,
                                 self.gshard)

    def _plan(self, engine) -> None:
        """Buckets, this rank's slices of them, the fp32 shard and the reduction partials."""
        k = kernels()
        dev = self.device
        flat = engine.flat
        P = flat.total
        # buckets: the backward pass completes the flat buffer from its end (stage order); mark i
        # (ViT layer i's input) completes everything from the first parameter of layer i on
        model = engine.model
        marks = model.grad_mark_count() if (self.overlap and hasattr(model, "set_grad_marks")) else 0
        bounds = []
        for i in range(marks):
            starts = [o for o, n in zip(flat.offsets, flat.names) if model.grad_stage(n) >= i + 1]
            bounds.append(min(starts) if starts else P)
        self.buckets = plan_buckets(P, bounds, self.min_bucket)
        self.slices_of = [rank_slices(self.buckets, self.world_size, r) for r in range(self.world_size)]
        self.slices = self.slices_of[self.rank]
        self.local_off = []
        S = 0
        for a, b in self.slices:
            self.local_off.append(S)
            S += b - a
        self.size = S
        self.mark_bucket = {m: j for j, (m, _, _) in enumerate(self.buckets) if m is not None}
        self.gshard = torch.zeros(S, dtype=torch.float32, device=dev)
        # reduce-scatter CTAs per bucket: few for the ones that overlap the backward pass
        self.blocks = [k.ddp_rs_blocks(m is not None) for (m, _, _) in self.buckets]
        self.p_off = [sum(self.blocks[:j]) for j in range(len(self.buckets))]
        self.partials = torch.zeros(sum(self.blocks), dtype=torch.float32, device=dev)
        self._stage = flat.grad_buf.view(torch.uint8)   # byte all-gather staging (between steps)
        self.side = torch.cuda.Stream(dev)
        if marks:
            model.set_grad_marks(self._on_mark)

    # ---------------------------------------------------------------- step
    def all_reduce_small(self, t: torch.Tensor) -> torch.Tensor:
        t = t.float().contiguous()
        self.comm.small_allreduce(t)
        return t

    def arm(self) -> None:
        """The next backward pass is the optimizer step's last: its marks launch the buckets."""
        self._armed = True
        self._next = 0

    def _launch(self, j: int, stream) -> None:
        a, b = self.slices[j]
        with torch.cuda.stream(stream):
            self.comm.rs(a, b - a, self.gshard, self.local_off[j], self.partials, self.p_off[j], j, self.blocks[j])

    def _on_mark(self, i: int) -> None:
        """Backward reached ViT layer i's input: reduce the bucket it completed on the side stream
        (ordered after everything the main stream has issued so far)."""
        j = self.mark_bucket.get(i)
        if not self._armed or j is None or j != self._next:
            return
        cur = torch.cuda.current_stream(self.device)
        self.side.wait_stream(cur)
        self._launch(j, self.side)
        self._next = j + 1

    def step(self, engine) -> None:
        if self.failed is not None:
            raise RuntimeError(f"fused DDP gradient step is unusable after an earlier failure: {self.failed}")
        cur = torch.cuda.current_stream(self.device)
        launched = self._next if self._armed else 0
        for j in range(launched, len(self.buckets)):      # the rest (at least the last bucket)
            self._launch(j, cur)
        if launched:
            cur.wait_stream(self.side)
        self._armed = False
        self._next = 0
        self.comm.publish(self.partials, self.partials.numel())
        self.comm.update(self.chunks, self.gdelta, self.gshard, engine.master_shard, engine.m, engine.v,
                         engine.ema_buf, engine.group_hyper, engine.scalars, engine.flags)

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
    def shard_of(self, full: torch.Tensor) -> torch.Tensor:
        """This rank's shard (its slice of every bucket, in bucket order) of a full flat vector."""
        return torch.cat([full[a:b] for a, b in self.slices])

    def gather_full(self, shard: torch.Tensor) -> torch.Tensor:
        """The full flat vector from every rank's shard (each rank holds its slice of every bucket)."""
        sizes = [sum(b - a for a, b in sl) for sl in self.slices_of]
        cap = max(sizes)
        mine = torch.zeros(cap, dtype=shard.dtype, device=shard.device)
        mine[:shard.numel()].copy_(shard)
        allp = torch.empty(cap * self.world_size, dtype=shard.dtype, device=shard.device)
        dist.all_gather_into_tensor(allp, mine, group=self.group)
        total = max(b for sl in self.slices_of for _, b in sl)
        out = torch.zeros(total, dtype=shard.dtype, device=shard.device)
        for r, sl in enumerate(self.slices_of):
            lo = r * cap
            for a, b in sl:
                out[a:b].copy_(allp[lo:lo + (b - a)])
                lo += b - a
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
