// Registry of the per-kernel-file debug status words (see MMLTK_DEBUG_CHECK in common.cuh) and the
// torch-facing accessors.  In a release build nothing registers, debug_status() returns 0 and
// debug_build() is false.
#include <mutex>
#include <vector>

#include "torch_ops.h"

namespace mmltk {

namespace {
std::mutex& reg_mutex() {
    static std::mutex m;
    return m;
}
std::vector<DebugReader>& readers() {
    static std::vector<DebugReader> r;
    return r;
}
}  // namespace

bool register_debug_reader(DebugReader reader) {
    std::lock_guard<std::mutex> lk(reg_mutex());
    readers().push_back(reader);
    return true;
}

namespace {

// first non-zero code among the registered words (all are read and cleared); synchronises the device
int64_t debug_status() {
    std::lock_guard<std::mutex> lk(reg_mutex());
    unsigned first = 0;
    for (auto r : readers()) {
        const unsigned v = r();
        if (v && !first) first = v;
    }
    return first;
}

bool debug_build() {
#if defined(MMLTK_DEBUG_BOUNDS) && MMLTK_DEBUG_BOUNDS
    return true;
#else
    return false;
#endif
}

}  // namespace

void register_debug_ops(pybind11::module& m) {
    m.def("debug_status", &debug_status);
    m.def("debug_build", &debug_build);
}

}  // namespace mmltk
