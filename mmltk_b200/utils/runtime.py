"""Per-process host runtime: which CPUs the loader, the GPU-feeding thread and the CPU
pool run on, how many threads each gets, and (optionally) raised scheduling priority.

Behaviour of the reference's runtime split and execution policy
(``src/rfdetr/core/runtime.cpp:47-140``, ``src/rfdetr/runtime.h:11-64``,
``src/execution_policy.cpp``; per-rank CPU shards in
``src/rfdetr/cli/distributed_train_launcher.cpp:118-146``), on the native
``exec_policy`` module:

* the rank's CPU set is ``--cpu-affinity`` (a subset of the allowed set) or the
  allowed set; under the multi-GPU launcher each rank gets a contiguous shard;
* ``--workers`` (0: one per CPU) is clamped to the set (at least 3) and split into
  loader (prefetch + 1), gather, lane and CPU-pool threads;
* the loader's producer thread is pinned to the first CPUs of the set, the global
  worker pool (batch gather, LSAP, evaluator) to the rest of the loader's CPUs and the
  CPU-pool slice, and the lane (the Python thread that launches GPU work) to the lane
  and CPU-pool slices -- off the loader's first CPU.
"""
from __future__ import annotations

import dataclasses
import logging
import os
from typing import Dict, List

from ..ops._ext import native

log = logging.getLogger("mmltk.runtime")

__all__ = ["HostRuntime", "setup_host_runtime", "rank_cpu_shards", "gpu_local_cpus"]


@dataclasses.dataclass
class HostRuntime:
    cpus: List[int]
    workers: int
    split: Dict[str, int]
    loader_cpus: List[int]
    lane_cpus: List[int]
    pool_cpus: List[int]
    pool_threads: int
    main_cpus: List[int]          # where the calling (lane) thread runs
    policy: Dict[str, object]

    def describe(self) -> str:
        f = native().format_cpuset
        return (f"cpus={f(self.cpus)} workers={self.workers} loader={self.split['loader']}@{f(self.loader_cpus)} "
                f"lane={self.split['lane']}@{f(self.main_cpus)} pool={self.pool_threads}@{f(self.pool_cpus)} "
                f"nice={self.policy.get('nice')}")


def setup_host_runtime(workers: int = 0, lanes: int = 1, prefetch: int = 2, cpu_affinity: str = "",
                       pin: bool = True, high_priority: bool = False) -> HostRuntime:
    """Resolve the CPU set and thread split; with ``pin``, place the global worker pool and
    the calling thread (the lane).  The loader's producer thread is placed by passing
    ``loader_cpus`` to ``BatchLoader(cpus=...)``."""
    n = native()
    cpus = [int(c) for c in n.resolve_cpu_affinity(cpu_affinity or "")]
    if len(cpus) >= 3:
        total = n.clamp_workers(int(workers), len(cpus), 0, 3)
        if workers and total != workers:
            log.warning("runtime: --workers %d clamped to %d for cpuset %s", workers, total, n.format_cpuset(cpus))
    else:
        total = max(3, int(workers) if workers and workers > 0 else 3)
        log.warning("runtime: cpuset %s has fewer than 3 CPUs; helper threads will share them", n.format_cpuset(cpus))
    split = dict(n.split_runtime(total, max(1, int(lanes or 1)), max(0, int(prefetch))))
    off = 0
    loader = list(n.cpu_slice(cpus, off, split["loader"])) or cpus
    off += split["loader"]
    lane = list(n.cpu_slice(cpus, off, split["lane"])) or cpus
    off += split["lane"]
    pool = list(n.cpu_slice(cpus, off, split["cpu"])) or cpus
    # gather work runs on the global pool too: it spans the loader's and the pool's CPUs
    pool_cpus = sorted(set(pool) | set(loader[1:] if len(loader) > 1 else loader))
    pool_threads = max(1, split["gather"] + split["cpu"])
    main_cpus = sorted(os.sched_getaffinity(0))
    if pin:
        pool_threads = n.configure_worker_pool(pool_threads, pool_cpus)
        want = sorted(set(lane) | set(pool))
        try:
            os.sched_setaffinity(0, want)
            main_cpus = want
        except OSError as e:   # a container may refuse; placement is an optimisation only
            log.warning("runtime: could not pin the lane thread to %s: %s", want, e)
    policy = dict(n.apply_thread_policy(-20, False, True) if high_priority else n.capture_policy())
    return HostRuntime(cpus, total, split, loader, lane, pool_cpus, pool_threads, main_cpus, policy)


def rank_cpu_shards(world: int, cpu_affinity: str = "") -> List[List[int]]:
    """Contiguous CPU shard per rank (empty lists when there are fewer CPUs than ranks)."""
    n = native()
    cpus = [int(c) for c in n.resolve_cpu_affinity(cpu_affinity or "")]
    return [list(n.shard_cpus(cpus, r, world)) for r in range(world)]


def gpu_local_cpus(device) -> List[int]:
    """CPUs of the GPU's own NUMA node (NVML's CPU affinity of the device, found by PCI bus id)
    that this process may run on; empty when NVML or the bus id is unavailable."""
    import torch
    try:
        import pynvml
        props = torch.cuda.get_device_properties(device)
        bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        pynvml.nvmlInit()
        try:
            h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            words = (os.cpu_count() + 63) // 64
            mask = pynvml.nvmlDeviceGetCpuAffinity(h, words)
        finally:
            pynvml.nvmlShutdown()
    except Exception as e:   # no NVML, no such attribute, not a physical GPU
        log.debug("gpu_local_cpus: %s", e)
        return []
    local = {64 * w + b for w, m in enumerate(mask) for b in range(64) if (int(m) >> b) & 1}
    return sorted(local & set(os.sched_getaffinity(0)))
