// Python bindings of the host-side native library (`mmltk_b200._native`).
#include <torch/extension.h>

#include <cmath>
#include <cstring>
#include <limits>
#include <vector>

#include "lsap.h"
#include "native_api.h"
#include "worker_pool.h"

namespace mmltk {

namespace {

// scipy-compatible single problem: returns (rows, cols) int64.
std::vector<torch::Tensor> lsap_py(torch::Tensor cost, bool maximize) {
    TORCH_CHECK(cost.dim() == 2, "cost must be 2-D");
    auto c = cost.to(torch::kFloat64).contiguous();
    const int64_t nr = c.size(0), nc = c.size(1);
    const int64_t n = std::min(nr, nc);
    auto rows = torch::empty({n}, torch::kInt64);
    auto cols = torch::empty({n}, torch::kInt64);
    LsapWorkspace ws;
    const auto st = lsap_solve(nr, nc, c.data_ptr<double>(), maximize, rows.data_ptr<int64_t>(),
                               cols.data_ptr<int64_t>(), ws);
    TORCH_CHECK(st != LsapStatus::kInvalid, "cost matrix contains invalid numeric entries");
    TORCH_CHECK(st != LsapStatus::kInfeasible, "cost matrix is infeasible");
    return {rows, cols};
}

// Batched Hungarian matching for Group-DETR.
//   cost   [NL, B, Q, T] float32 (CPU), Q = groups * Qg, T >= max(counts)
//   counts [B] int64
// returns match [NL, B, groups, T] int32: for target slot t of image b the
// matched query index (in [0, Q)) of each group, -1 when unmatched / padded.
torch::Tensor match_batched(torch::Tensor cost, torch::Tensor counts, int64_t groups) {
    TORCH_CHECK(cost.dim() == 4 && cost.device().is_cpu(), "cost must be a CPU [NL,B,Q,T] tensor");
    auto c = cost.to(torch::kFloat32).contiguous();
    auto cnt = counts.to(torch::kInt64).contiguous();
    const int64_t NL = c.size(0), B = c.size(1), Q = c.size(2), T = c.size(3);
    TORCH_CHECK(groups >= 1 && Q % groups == 0, "query count must be divisible by groups");
    TORCH_CHECK(cnt.numel() == B, "counts must have one entry per image");
    const int64_t Qg = Q / groups;
    auto out = torch::full({NL, B, groups, T}, -1, torch::kInt32);
    const float* cp = c.data_ptr<float>();
    const int64_t* np = cnt.data_ptr<int64_t>();
    int32_t* op = out.data_ptr<int32_t>();
    const int64_t tasks = NL * B * groups;
    WorkerPool::global().parallel_for(tasks, [&](int64_t task) {
        thread_local LsapWorkspace ws;
        thread_local std::vector<double> m;
        thread_local std::vector<int64_t> rr, cc;
        const int64_t g = task % groups;
        const int64_t b = (task / groups) % B;
        const int64_t l = task / (groups * B);
        const int64_t nt = std::min<int64_t>(np[b], T);
        if (nt <= 0) return;
        m.resize(static_cast<size_t>(Qg * nt));
        const float* base = cp + ((l * B + b) * Q + g * Qg) * T;
        for (int64_t q = 0; q < Qg; ++q)
            for (int64_t t = 0; t < nt; ++t) m[q * nt + t] = static_cast<double>(base[q * T + t]);
        lsap_sanitize(m.data(), Qg * nt);
        const int64_t k = std::min(Qg, nt);
        rr.resize(k);
        cc.resize(k);
        const auto st = lsap_solve(Qg, nt, m.data(), false, rr.data(), cc.data(), ws);
        if (st != LsapStatus::kOk) return;  // sanitized costs are always feasible
        int32_t* o = op + ((l * B + b) * groups + g) * T;
        for (int64_t i = 0; i < k; ++i) o[cc[i]] = static_cast<int32_t>(g * Qg + rr[i]);
    });
    return out;
}

std::vector<int64_t> parse_cpuset_py(const std::string& s) {
    auto v = parse_cpuset(s);
    return std::vector<int64_t>(v.begin(), v.end());
}

std::string format_cpuset_py(const std::vector<int64_t>& v) {
    return format_cpuset(std::vector<int>(v.begin(), v.end()));
}

}  // namespace

}  // namespace mmltk

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.doc() = "mmltk_b200 host-side native library";
    m.def("lsap", &mmltk::lsap_py, "rectangular linear sum assignment (scipy-compatible)", py::arg("cost"),
          py::arg("maximize") = false);
    m.def("match_batched", &mmltk::match_batched, "batched Group-DETR Hungarian matching");
    m.def("parse_cpuset", &mmltk::parse_cpuset_py);
    m.def("format_cpuset", &mmltk::format_cpuset_py);
    mmltk::register_native_api(m);
}
