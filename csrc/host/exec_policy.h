// Host execution policy: CPU sets, per-rank CPU shards, worker budgets, the split of a
// rank's worker budget into loader / gather / lane / CPU-pool threads, and best-effort
// scheduling priority.
//
// Counterpart of the reference's `include/execution_policy.h:9-36`,
// `src/execution_policy.cpp` (process/worker policy, worker-budget clamp) and
// `src/rfdetr/runtime.h:11-64`, `src/rfdetr/core/runtime.cpp:74-140` (runtime split).
// Priority changes never fail the caller: a request the kernel refuses (no
// CAP_SYS_NICE, no realtime budget) leaves that setting as it was, and the snapshot
// reports what is in force.
#pragma once

#include <string>
#include <vector>

namespace mmltk {

struct PolicySnapshot {
    std::vector<int> affinity;   // CPUs the calling thread may run on
    int online_cpus = 0;
    int nice = 0;
    int sched_policy = 0;        // SCHED_OTHER / SCHED_FIFO / SCHED_RR / ...
    int sched_priority = 0;
    int io_class = 0;            // IOPRIO_CLASS_{NONE,RT,BE,IDLE}
    int io_data = 0;
};

struct RuntimeSplit {
    int loader = 0;   // batch producer threads (prefetch depth + 1, at least one when prefetching)
    int gather = 0;   // threads that gather images of one batch
    int lane = 1;     // GPU-feeding (training / inference lane) threads
    int cpu = 1;      // general CPU pool (matcher LSAP, evaluator)
};

std::vector<int> allowed_cpus();                                // sched_getaffinity of this thread
// "" -> allowed_cpus(); else the parsed list, which must be a subset of the allowed set
std::vector<int> resolve_cpu_affinity(const std::string& spec);
// contiguous block `rank` of `world` blocks (sizes differ by at most one); empty if world > cpus
std::vector<int> shard_cpus(const std::vector<int>& cpus, int rank, int world);
// requested (<= 0: one per CPU) limited to the CPUs left after `reserved`, never below `minimum`
int clamp_workers(int requested, int cpus, int reserved = 0, int minimum = 1);
RuntimeSplit split_runtime(int workers, int lanes, int prefetch);
// `count` CPUs starting at `offset` (wrapping), sorted and unique
std::vector<int> cpu_slice(const std::vector<int>& cpus, int offset, int count);

bool set_thread_affinity(const std::vector<int>& cpus);
// lowest nice value the kernel allows (down to `target_nice`), optionally SCHED_RR at the
// highest permitted priority and realtime I/O priority (falling back to best-effort 0)
PolicySnapshot apply_thread_policy(int target_nice, bool realtime_sched, bool realtime_io);
PolicySnapshot capture_policy();

}  // namespace mmltk
