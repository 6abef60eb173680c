// Python bindings of the execution policy (exec_policy.h) and of the global worker pool's
// size / CPU placement.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "exec_policy.h"
#include "worker_pool.h"

namespace py = pybind11;

namespace mmltk {

namespace {

py::dict snapshot_dict(const PolicySnapshot& s) {
    py::dict d;
    d["affinity"] = s.affinity;
    d["online_cpus"] = s.online_cpus;
    d["nice"] = s.nice;
    d["sched_policy"] = s.sched_policy;
    d["sched_priority"] = s.sched_priority;
    d["io_class"] = s.io_class;
    d["io_data"] = s.io_data;
    return d;
}

}  // namespace

void register_exec_api(py::module& m) {
    m.def("allowed_cpus", &allowed_cpus);
    m.def("resolve_cpu_affinity", &resolve_cpu_affinity, py::arg("spec"));
    m.def("shard_cpus", &shard_cpus, py::arg("cpus"), py::arg("rank"), py::arg("world"));
    m.def("clamp_workers", &clamp_workers, py::arg("requested"), py::arg("cpus"), py::arg("reserved") = 0,
          py::arg("minimum") = 1);
    m.def("cpu_slice", &cpu_slice, py::arg("cpus"), py::arg("offset"), py::arg("count"));
    m.def("split_runtime", [](int workers, int lanes, int prefetch) {
        const RuntimeSplit s = split_runtime(workers, lanes, prefetch);
        py::dict d;
        d["loader"] = s.loader;
        d["gather"] = s.gather;
        d["lane"] = s.lane;
        d["cpu"] = s.cpu;
        return d;
    }, py::arg("workers"), py::arg("lanes"), py::arg("prefetch"));
    m.def("set_thread_affinity", &set_thread_affinity, py::arg("cpus"));
    m.def("apply_thread_policy", [](int target_nice, bool realtime_sched, bool realtime_io) {
        return snapshot_dict(apply_thread_policy(target_nice, realtime_sched, realtime_io));
    }, py::arg("target_nice") = -20, py::arg("realtime_sched") = false, py::arg("realtime_io") = true);
    m.def("capture_policy", [] { return snapshot_dict(capture_policy()); });
    m.def("configure_worker_pool", [](int threads, std::vector<int> cpus) {
        return WorkerPool::configure_global(threads, std::move(cpus));
    }, py::arg("threads"), py::arg("cpus"));
}

}  // namespace mmltk
