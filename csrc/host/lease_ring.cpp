#include "lease_ring.h"

#include <chrono>
#include <stdexcept>

#include <torch/extension.h>

#include "native_api.h"

namespace mmltk::live {

LeaseRing::LeaseRing(int slots) : state_(size_t(slots), kFree), seq_(size_t(slots), 0) {
    if (slots < 2) throw std::invalid_argument("lease ring: at least two slots");
}

int LeaseRing::acquire_write() {
    std::lock_guard<std::mutex> lk(mu_);
    for (size_t i = 0; i < state_.size(); ++i)
        if (state_[i] == kFree) {
            state_[i] = kWriting;
            return int(i);
        }
    // recycle the oldest frame the consumer never took
    int oldest = -1;
    for (size_t i = 0; i < state_.size(); ++i)
        if (state_[i] == kPublished && (oldest < 0 || seq_[i] < seq_[size_t(oldest)])) oldest = int(i);
    if (oldest >= 0) {
        state_[size_t(oldest)] = kWriting;
        ++dropped_;
    }
    return oldest;
}

void LeaseRing::publish(int slot, uint64_t seq) {
    {
        std::lock_guard<std::mutex> lk(mu_);
        if (slot < 0 || size_t(slot) >= state_.size() || state_[size_t(slot)] != kWriting)
            throw std::logic_error("lease ring: publish of a slot that is not being written");
        state_[size_t(slot)] = kPublished;
        seq_[size_t(slot)] = seq;
        ++published_;
    }
    cv_.notify_all();
}

int LeaseRing::acquire_latest(double timeout_s, uint64_t* seq) {
    std::unique_lock<std::mutex> lk(mu_);
    auto ready = [this] {
        if (closed_) return true;
        for (auto s : state_)
            if (s == kPublished) return true;
        return false;
    };
    if (!cv_.wait_for(lk, std::chrono::duration<double>(timeout_s), ready)) return -1;
    int best = -1;
    for (size_t i = 0; i < state_.size(); ++i)
        if (state_[i] == kPublished && (best < 0 || seq_[i] > seq_[size_t(best)])) best = int(i);
    if (best < 0) return -1;   // closed with nothing pending
    // older published frames are skipped: free them
    for (size_t i = 0; i < state_.size(); ++i)
        if (state_[i] == kPublished && int(i) != best) {
            state_[i] = kFree;
            ++dropped_;
        }
    state_[size_t(best)] = kLeased;
    if (seq) *seq = seq_[size_t(best)];
    return best;
}

void LeaseRing::release(int slot) {
    {
        std::lock_guard<std::mutex> lk(mu_);
        if (slot < 0 || size_t(slot) >= state_.size() || state_[size_t(slot)] != kLeased)
            throw std::logic_error("lease ring: release of a slot that is not leased");
        state_[size_t(slot)] = kFree;
    }
    cv_.notify_all();
}

void LeaseRing::close() {
    {
        std::lock_guard<std::mutex> lk(mu_);
        closed_ = true;
    }
    cv_.notify_all();
}

uint64_t LeaseRing::dropped() const {
    std::lock_guard<std::mutex> lk(mu_);
    return dropped_;
}

uint64_t LeaseRing::published() const {
    std::lock_guard<std::mutex> lk(mu_);
    return published_;
}

}  // namespace mmltk::live

namespace mmltk {

void register_live_api(pybind11::module& m) {
    using live::LeaseRing;
    py::class_<LeaseRing>(m, "LeaseRing")
        .def(py::init<int>())
        .def("acquire_write", &LeaseRing::acquire_write)
        .def("publish", &LeaseRing::publish)
        .def("acquire_latest",
             [](LeaseRing& r, double timeout) -> py::object {
                 uint64_t seq = 0;
                 int s;
                 {
                     py::gil_scoped_release nogil;
                     s = r.acquire_latest(timeout, &seq);
                 }
                 if (s < 0) return py::none();
                 return py::make_tuple(s, seq);
             },
             py::arg("timeout") = 1.0)
        .def("release", &LeaseRing::release)
        .def("close", &LeaseRing::close)
        .def("dropped", &LeaseRing::dropped)
        .def("published", &LeaseRing::published)
        .def("slots", &LeaseRing::slots);
}

}  // namespace mmltk
