"""Process-per-GPU launch and the distributed context.

Reference (`src/rfdetr/training/train.cpp:839-868`, CLI fork in
`src/rfdetr/cli/cli.cpp`): the parent process forks one child per
``--device-ids`` entry with its arguments rewritten (``--device-id``,
``--dist-worker``, ``--dist-rank``, ``--dist-world-size``,
``--dist-store-file``, a share of ``--workers``), forwards SIGTERM/SIGINT to
every child, and fails as soon as one child fails.  Children rendezvous
through a ``FileStore`` at ``--dist-store-file``.

Here the same flags are honoured; a ``torchrun`` environment (RANK /
WORLD_SIZE / LOCAL_RANK / MASTER_ADDR) is accepted as well.  The process group
is NCCL on CUDA (the fused NVSwitch gradient step uses it only for setup) and
gloo on CPU, with a bounded timeout so that a lost rank ends the others with
an error instead of a hang.
"""
from __future__ import annotations

import dataclasses
import datetime
import os
import signal
import subprocess
import sys
import tempfile
import time
from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

__all__ = ["DistContext", "init_distributed", "launch_workers", "rank_plan", "rewrite_worker_argv"]


@dataclasses.dataclass
class DistContext:
    enabled: bool = False
    rank: int = 0
    world_size: int = 1
    local_rank: int = 0
    device: torch.device = dataclasses.field(default_factory=lambda: torch.device("cpu"))
    owns_group: bool = False

    @property
    def main(self) -> bool:
        return self.rank == 0

    def barrier(self) -> None:
        if self.enabled:
            dist.barrier()

    def close(self) -> None:
        if self.enabled and self.owns_group and dist.is_initialized():
            dist.destroy_process_group()


def init_distributed(rank: Optional[int] = None, world_size: Optional[int] = None, device_id: Optional[int] = None,
                     store_file: str = "", timeout_s: float = 600.0, backend: Optional[str] = None) -> DistContext:
    env_world = int(os.environ.get("WORLD_SIZE", "1"))
    world = world_size if (world_size is not None and world_size > 1) else env_world
    cuda = torch.cuda.is_available()
    if world <= 1:
        dev = torch.device("cuda", device_id or 0) if cuda else torch.device("cpu")
        if cuda:
            torch.cuda.set_device(dev)
        return DistContext(False, 0, 1, 0, dev)
    r = rank if (rank is not None and world_size is not None and world_size > 1) else int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(r)))
    dev_index = device_id if device_id is not None and world_size is not None and world_size > 1 else local
    dev = torch.device("cuda", dev_index) if cuda else torch.device("cpu")
    if cuda:
        torch.cuda.set_device(dev)
    be = backend or ("nccl" if cuda else "gloo")
    owns = False
    if not dist.is_initialized():
        kw = dict(backend=be, rank=r, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
        if cuda and be == "nccl":
            kw["device_id"] = dev
        if store_file:
            kw["store"] = dist.FileStore(store_file, world)
        else:
            kw["init_method"] = "env://"
        dist.init_process_group(**kw)
        owns = True
    return DistContext(True, dist.get_rank(), dist.get_world_size(), local, dev, owns)


_DIST_FLAGS_WITH_VALUE = ("--device-id", "--device-ids", "--dist-rank", "--dist-world-size", "--dist-store-file",
                          "--workers", "--cpu-affinity")


def rewrite_worker_argv(argv: Sequence[str], rank: int, world: int, device: int, store: str,
                        workers: Optional[int] = None, cpu_affinity: Optional[str] = None) -> List[str]:
    """Child argument list: the parent's minus the multi-device / rendezvous flags, plus this rank's."""
    out, skip = [], False
    for a in argv:
        if skip:
            skip = False
            continue
        if a in _DIST_FLAGS_WITH_VALUE:
            skip = True
            continue
        if any(a.startswith(f + "=") for f in _DIST_FLAGS_WITH_VALUE) or a == "--dist-worker":
            continue
        out.append(a)
    out += ["--device-id", str(device), "--dist-worker", "--dist-rank", str(rank), "--dist-world-size", str(world),
            "--dist-store-file", store]
    if workers is not None:
        out += ["--workers", str(workers)]
    if cpu_affinity:
        out += ["--cpu-affinity", cpu_affinity]
    return out


def rank_plan(world: int, workers: int = 0, cpu_affinity: str = "") -> List[Tuple[Optional[int], str]]:
    """(worker budget, CPU list) per rank: contiguous CPU shards of ``cpu_affinity`` (or of
    the allowed set), the worker budget split evenly and clamped to the shard (>= 3)."""
    from ..ops._ext import native
    from ..utils.runtime import rank_cpu_shards
    n = native()
    shards = rank_cpu_shards(world, cpu_affinity)
    out = []
    for r in range(world):
        per = max(1, workers // world + (1 if r < workers % world else 0)) if workers else None
        shard = shards[r]
        if len(shard) >= 3:
            per = n.clamp_workers(per or 0, len(shard), 0, 3)
        out.append((per, n.format_cpuset(shard) if shard else ""))
    return out


def launch_workers(argv: Sequence[str], device_ids: Sequence[int], workers: int = 0, python: Optional[str] = None,
                   entry: Optional[Sequence[str]] = None, poll_s: float = 0.2, cpu_affinity: str = "") -> int:
    """Run one child per device and wait.  Returns 0, or the first failing child's exit code
    (the others are terminated).  SIGINT / SIGTERM received by the parent go to every child.
    Each child gets a contiguous shard of the CPUs and its share of ``--workers``
    (``rank_plan``)."""
    world = len(device_ids)
    store = os.path.join(tempfile.gettempdir(), f"mmltk_rfdetr_train_{os.getpid()}.store")
    if os.path.exists(store):
        os.remove(store)
    base = list(entry) if entry is not None else [python or sys.executable, "-m", "mmltk_b200.cli"]
    plan = rank_plan(world, workers, cpu_affinity)
    children: List[subprocess.Popen] = []
    for r, d in enumerate(device_ids):
        per, cpus = plan[r]
        cmd = base + rewrite_worker_argv(argv, r, world, int(d), store, per, cpus or None)
        children.append(subprocess.Popen(cmd))

    def forward(sig, _frame):
        for c in children:
            if c.poll() is None:
                c.send_signal(sig)

    old = {s: signal.signal(s, forward) for s in (signal.SIGINT, signal.SIGTERM)}
    code = 0
    try:
        while True:
            states = [c.poll() for c in children]
            failed = [s for s in states if s not in (None, 0)]
            if failed:
                code = failed[0]
                for c in children:
                    if c.poll() is None:
                        c.terminate()
                deadline = time.time() + 30
                for c in children:
                    try:
                        c.wait(max(0.1, deadline - time.time()))
                    except subprocess.TimeoutExpired:
                        c.kill()
                break
            if all(s == 0 for s in states):
                break
            time.sleep(poll_s)
    finally:
        for s, h in old.items():
            signal.signal(s, h)
        if os.path.exists(store):
            try:
                os.remove(store)
            except OSError:
                pass
    return int(code)
