#ifndef _GNU_SOURCE
#define _GNU_SOURCE
#endif
#include "exec_policy.h"

#include <pthread.h>
#include <sched.h>
#include <sys/resource.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <set>
#include <stdexcept>

#include "worker_pool.h"

namespace mmltk {

namespace {

// ioprio encoding of the Linux ABI (include/uapi/linux/ioprio.h): class in the top bits
constexpr int kIoprioClassShift = 13;
constexpr int kIoprioWhoProcess = 1;
constexpr int kIoprioClassRt = 1;
constexpr int kIoprioClassBe = 2;

int ioprio_value(int cls, int data) { return (cls << kIoprioClassShift) | data; }

bool set_ioprio(int cls, int data) {
#ifdef SYS_ioprio_set
    return ::syscall(SYS_ioprio_set, kIoprioWhoProcess, 0, ioprio_value(cls, data)) == 0;
#else
    (void)cls;
    (void)data;
    return false;
#endif
}

}  // namespace

std::vector<int> allowed_cpus() {
    cpu_set_t set;
    CPU_ZERO(&set);
    std::vector<int> out;
    if (pthread_getaffinity_np(pthread_self(), sizeof(set), &set) == 0) {
        for (int c = 0; c < CPU_SETSIZE; ++c)
            if (CPU_ISSET(c, &set)) out.push_back(c);
    }
    if (out.empty()) {
        const long n = ::sysconf(_SC_NPROCESSORS_ONLN);
        for (int c = 0; c < std::max(1L, n); ++c) out.push_back(c);
    }
    return out;
}

std::vector<int> resolve_cpu_affinity(const std::string& spec) {
    const std::vector<int> allowed = allowed_cpus();
    if (spec.empty()) return allowed;
    std::vector<int> want = parse_cpuset(spec);
    if (want.empty()) throw std::invalid_argument("cpu affinity '" + spec + "' names no CPU");
    const std::set<int> ok(allowed.begin(), allowed.end());
    for (int c : want)
        if (!ok.count(c))
            throw std::invalid_argument("cpu affinity '" + spec + "': CPU " + std::to_string(c) +
                                        " is not in this process's allowed set " + format_cpuset(allowed));
    return want;
}

std::vector<int> shard_cpus(const std::vector<int>& cpus, int rank, int world) {
    if (world <= 0 || rank < 0 || rank >= world) throw std::invalid_argument("shard_cpus: bad rank / world");
    const int n = static_cast<int>(cpus.size());
    if (n < world) return {};
    const int base = n / world, extra = n % world;
    const int begin = rank * base + std::min(rank, extra);
    const int len = base + (rank < extra ? 1 : 0);
    return std::vector<int>(cpus.begin() + begin, cpus.begin() + begin + len);
}

int clamp_workers(int requested, int cpus, int reserved, int minimum) {
    const int avail = std::max(0, cpus - std::max(0, reserved));
    const int want = requested > 0 ? requested : avail;
    return std::max(std::max(1, minimum), std::min(want, std::max(avail, 1)));
}

RuntimeSplit split_runtime(int workers, int lanes, int prefetch) {
    RuntimeSplit s;
    const int total = std::max(1, workers);
    const int want_loader = prefetch > 0 ? prefetch + 1 : 0;
    const int want_lanes = std::max(1, lanes);
    if (total < 3) {
        // too few threads to split: one of each, overlapping
        s.loader = want_loader > 0 ? 1 : 0;
        s.gather = s.loader;
        s.lane = 1;
        s.cpu = 1;
        return s;
    }
    // lanes first (they feed the GPU), then the loader, the rest is the CPU pool (>= 1)
    s.lane = std::min(want_lanes, total - (want_loader > 0 ? 1 : 0) - 1);
    s.loader = std::min(want_loader, total - s.lane - 1);
    s.gather = s.loader > 0 ? std::max(1, s.loader - 1) : 0;
    s.cpu = total - s.loader - s.lane;
    return s;
}

std::vector<int> cpu_slice(const std::vector<int>& cpus, int offset, int count) {
    std::vector<int> out;
    if (cpus.empty() || count <= 0) return out;
    for (int i = 0; i < count; ++i) out.push_back(cpus[static_cast<size_t>(offset + i) % cpus.size()]);
    std::sort(out.begin(), out.end());
    out.erase(std::unique(out.begin(), out.end()), out.end());
    return out;
}

bool set_thread_affinity(const std::vector<int>& cpus) {
    if (cpus.empty()) return false;
    cpu_set_t set;
    CPU_ZERO(&set);
    for (int c : cpus)
        if (c >= 0 && c < CPU_SETSIZE) CPU_SET(c, &set);
    return pthread_setaffinity_np(pthread_self(), sizeof(set), &set) == 0;
}

PolicySnapshot capture_policy() {
    PolicySnapshot s;
    s.affinity = allowed_cpus();
    s.online_cpus = static_cast<int>(std::max(0L, ::sysconf(_SC_NPROCESSORS_ONLN)));
    errno = 0;
    const int nv = ::getpriority(PRIO_PROCESS, 0);
    s.nice = (nv == -1 && errno != 0) ? 0 : nv;
    sched_param sp{};
    int pol = 0;
    if (pthread_getschedparam(pthread_self(), &pol, &sp) == 0) {
        s.sched_policy = pol;
        s.sched_priority = sp.sched_priority;
    }
#ifdef SYS_ioprio_get
    const long io = ::syscall(SYS_ioprio_get, kIoprioWhoProcess, 0);
    if (io >= 0) {
        s.io_class = static_cast<int>(io >> kIoprioClassShift);
        s.io_data = static_cast<int>(io & ((1 << kIoprioClassShift) - 1));
    }
#endif
    return s;
}

PolicySnapshot apply_thread_policy(int target_nice, bool realtime_sched, bool realtime_io) {
    // nice: walk down from the current value; stop at the first value the kernel refuses
    errno = 0;
    int cur = ::getpriority(PRIO_PROCESS, 0);
    if (!(cur == -1 && errno != 0)) {
        for (int v = cur - 1; v >= std::max(-20, target_nice); --v) {
            if (::setpriority(PRIO_PROCESS, 0, v) != 0) break;
        }
    }
    if (realtime_sched) {
        const int hi = sched_get_priority_max(SCHED_RR);
        for (int p = hi; p >= 1; --p) {
            sched_param sp{};
            sp.sched_priority = p;
            if (pthread_setschedparam(pthread_self(), SCHED_RR, &sp) == 0) break;
        }
    }
    if (!(realtime_io && set_ioprio(kIoprioClassRt, 0))) {
        for (int d = 0; d <= 7; ++d)
            if (set_ioprio(kIoprioClassBe, d)) break;
    }
    return capture_policy();
}

}  // namespace mmltk
