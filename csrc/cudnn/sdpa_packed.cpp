// Scaled-dot-product attention backward through the cuDNN graph API with caller-given strides for
// every operand, so that dQ / dK / dV are written straight into their slices of the packed
// [N, L, 3, H, D] gradient of the fused QKV projection.
//
// PyTorch's cuDNN attention backward (`aten::_scaled_dot_product_cudnn_attention_backward`, the
// path `F.scaled_dot_product_attention` takes for these shapes) allocates dQ, dK and dV as three
// dense tensors; the packed projection gradient then costs one more read and write of 3 x N x L x C
// elements per layer.  Here the same cuDNN SDPA backward node writes into strided views instead.
// The forward stays PyTorch's cuDNN forward; its output O and its softmax statistics (natural-log
// log-sum-exp of the scaled scores, fp32) are the inputs this backward needs.
//
// Counterpart in the reference: the backward that autograd runs for its backbone attention call
// (`at::scaled_dot_product_attention`, src/rfdetr/layers/model.cpp:498), whose q / k / v gradients
// libtorch then gathers into the projection's gradient.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cudnn_frontend.h>

#include <csignal>
#include <cstdio>
#include <execinfo.h>
#include <unistd.h>
#include <cstdlib>
#include <map>
#include <memory>
#include <mutex>
#include <sstream>
#include <string>
#include <unordered_map>
#include <vector>

namespace fe = cudnn_frontend;

namespace {

constexpr int64_t kQ = 1, kK = 2, kV = 3, kO = 4, kDO = 5, kStats = 6, kDQ = 7, kDK = 8, kDV = 9;

struct Plan {
    std::shared_ptr<fe::graph::Graph> graph;
    int64_t workspace = 0;
};

std::mutex g_mu;
std::map<int, cudnnHandle_t> g_handles;
std::map<std::string, std::shared_ptr<Plan>> g_plans;

cudnnHandle_t handle_for(int dev) {
    auto it = g_handles.find(dev);
    if (it != g_handles.end()) return it->second;
    cudnnHandle_t h = nullptr;
    TORCH_CHECK(cudnnCreate(&h) == CUDNN_STATUS_SUCCESS, "sdpa_packed: cudnnCreate failed");
    g_handles[dev] = h;
    return h;
}

// MMLTK_SDPA_TRACE=1: one stderr line per set-up / launch stage (locates a failing stage)
bool tracing() {
    static const bool on = [] {
        const char* e = std::getenv("MMLTK_SDPA_TRACE");
        return e != nullptr && e[0] == '1';
    }();
    return on;
}

void trace(const char* what) {
    if (tracing()) {
        std::fprintf(stderr, "[sdpa_packed] %s\n", what);
        std::fflush(stderr);
    }
}

// with tracing on, a SIGSEGV prints the native frames (library + offset) before the process ends
void on_segv(int sig) {
    void* frames[64];
    const int n = backtrace(frames, 64);
    backtrace_symbols_fd(frames, n, 2);
    std::signal(sig, SIG_DFL);
    std::raise(sig);
}

void install_trace_handler() {
    if (tracing()) std::signal(SIGSEGV, on_segv);
}

void check(fe::error_object e, const char* what) {
    trace(what);
    TORCH_CHECK(e.is_good(), "sdpa_packed: ", what, ": ", e.get_message());
}

std::vector<int64_t> dims_of(const torch::Tensor& t) { return t.sizes().vec(); }
std::vector<int64_t> strides_of(const torch::Tensor& t) { return t.strides().vec(); }

std::string key_of(int dev, double scale, const std::vector<torch::Tensor>& ts) {
    std::ostringstream os;
    os.precision(17);
    os << dev << '|' << scale << '|' << static_cast<int>(ts[0].scalar_type());
    for (const auto& t : ts) {
        os << '|';
        for (auto d : t.sizes()) os << d << ',';
        os << ';';
        for (auto s : t.strides()) os << s << ',';
    }
    return os.str();
}

std::shared_ptr<Plan> build_plan(cudnnHandle_t h, double scale, fe::DataType_t io, const torch::Tensor& q,
                                 const torch::Tensor& k, const torch::Tensor& v, const torch::Tensor& o,
                                 const torch::Tensor& dout, const torch::Tensor& stats, const torch::Tensor& dq,
                                 const torch::Tensor& dk, const torch::Tensor& dv) {
    trace("build: graph");
    auto g = std::make_shared<fe::graph::Graph>();
    g->set_io_data_type(io).set_intermediate_data_type(fe::DataType_t::FLOAT).set_compute_data_type(
        fe::DataType_t::FLOAT);
    auto in = [&](const char* name, int64_t uid, const torch::Tensor& t) {
        return g->tensor(fe::graph::Tensor_attributes().set_name(name).set_uid(uid).set_dim(dims_of(t)).set_stride(
            strides_of(t)));
    };
    auto Q = in("Q", kQ, q), K = in("K", kK, k), V = in("V", kV, v), O = in("O", kO, o), dO = in("dO", kDO, dout);
    // statistics [N, H, L] (or [N, H, L, 1]) -> [N, H, L, 1]
    const int64_t N = stats.size(0), H = stats.size(1), L = stats.size(2);
    auto S = g->tensor(fe::graph::Tensor_attributes()
                           .set_name("Stats")
                           .set_uid(kStats)
                           .set_dim({N, H, L, 1})
                           .set_stride({stats.stride(0), stats.stride(1), stats.stride(2), 1})
                           .set_data_type(fe::DataType_t::FLOAT));
    auto attrs = fe::graph::SDPA_backward_attributes().set_name("sdpa_bwd").set_attn_scale(static_cast<float>(scale));
    trace("build: sdpa_backward node");
    auto outs = g->sdpa_backward(Q, K, V, O, dO, S, attrs);
    outs[0]->set_output(true).set_uid(kDQ).set_dim(dims_of(dq)).set_stride(strides_of(dq));
    outs[1]->set_output(true).set_uid(kDK).set_dim(dims_of(dk)).set_stride(strides_of(dk));
    outs[2]->set_output(true).set_uid(kDV).set_dim(dims_of(dv)).set_stride(strides_of(dv));
    check(g->validate(), "validate");
    check(g->build_operation_graph(h), "build_operation_graph");
    check(g->create_execution_plans({fe::HeurMode_t::A}), "create_execution_plans");
    check(g->check_support(h), "check_support");
    check(g->build_plans(h), "build_plans");
    auto p = std::make_shared<Plan>();
    check(g->get_workspace_size(p->workspace), "get_workspace_size");
    p->graph = g;
    return p;
}

void check_operand(const torch::Tensor& t, const torch::Tensor& like) {
    TORCH_CHECK(t.is_cuda() && t.dim() == 4 && t.scalar_type() == like.scalar_type() && t.device() == like.device(),
                "sdpa_packed: operands must be 4-D CUDA tensors of the query's dtype and device");
    TORCH_CHECK(t.stride(3) == 1, "sdpa_packed: operands need a unit stride in the head dimension");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, "sdpa_packed: operands must be 16-byte aligned");
}

void check_stats(const torch::Tensor& stats, const torch::Tensor& q) {
    TORCH_CHECK(stats.is_cuda() && stats.scalar_type() == torch::kFloat &&
                    (stats.dim() == 3 || (stats.dim() == 4 && stats.size(3) == 1)) && stats.size(0) == q.size(0) &&
                    stats.size(1) == q.size(1) && stats.size(2) == q.size(2),
                "sdpa_packed: stats must be [N, H, L] or [N, H, L, 1] fp32");
}

// q / k / v / o / dout / dq / dk / dv: [N, H, L, D] views with any strides (unit stride in D);
// stats: the fp32 log-sum-exp PyTorch's cuDNN forward returns ([N, H, L] or [N, H, L, 1]).
void sdpa_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor dout,
              torch::Tensor stats, torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, double scale) {
    trace("enter");
    TORCH_CHECK(q.scalar_type() == torch::kBFloat16 || q.scalar_type() == torch::kHalf,
                "sdpa_packed: bf16 or fp16 operands expected");
    for (auto* p : {&q, &k, &v, &o, &dout, &dq, &dk, &dv}) check_operand(*p, q);
    TORCH_CHECK(q.sizes() == k.sizes() && q.sizes() == v.sizes() && q.sizes() == o.sizes() &&
                    q.sizes() == dout.sizes() && q.sizes() == dq.sizes() && q.sizes() == dk.sizes() &&
                    q.sizes() == dv.sizes(),
                "sdpa_packed: self-attention operands of one shape expected");
    check_stats(stats, q);
    trace("operands checked");
    const int dev = q.get_device();
    c10::cuda::CUDAGuard guard(q.device());
    const auto key = key_of(dev, scale, {q, k, v, o, dout, stats, dq, dk, dv});
    trace("key");
    // one handle per device, shared by the threads that drive it: plan lookup, stream binding and
    // the enqueue happen under one lock
    std::lock_guard<std::mutex> lk(g_mu);
    trace("handle");
    cudnnHandle_t h = handle_for(dev);
    std::shared_ptr<Plan> plan;
    auto it = g_plans.find(key);
    if (it == g_plans.end()) {
        const auto io = q.scalar_type() == torch::kBFloat16 ? fe::DataType_t::BFLOAT16 : fe::DataType_t::HALF;
        plan = build_plan(h, scale, io, q, k, v, o, dout, stats, dq, dk, dv);
        g_plans[key] = plan;
    } else {
        plan = it->second;
    }
    auto stream = at::cuda::getCurrentCUDAStream();
    TORCH_CHECK(cudnnSetStream(h, stream.stream()) == CUDNN_STATUS_SUCCESS, "sdpa_packed: cudnnSetStream failed");
    torch::Tensor ws;
    if (plan->workspace > 0) ws = torch::empty({plan->workspace}, q.options().dtype(torch::kUInt8));
    std::unordered_map<int64_t, void*> pack{{kQ, q.data_ptr()},   {kK, k.data_ptr()},       {kV, v.data_ptr()},
                                           {kO, o.data_ptr()},   {kDO, dout.data_ptr()},   {kStats, stats.data_ptr()},
                                           {kDQ, dq.data_ptr()}, {kDK, dk.data_ptr()},     {kDV, dv.data_ptr()}};
    trace("execute: begin");
    check(plan->graph->execute(h, pack, plan->workspace > 0 ? ws.data_ptr() : nullptr), "execute");
}

// True when sdpa_bwd has already built the cuDNN plan for these operands' shapes and strides.
bool has_plan(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor dout,
              torch::Tensor stats, torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, double scale) {
    std::lock_guard<std::mutex> lk(g_mu);
    return g_plans.count(key_of(q.get_device(), scale, {q, k, v, o, dout, stats, dq, dk, dv})) > 0;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.doc() = "cuDNN SDPA backward into caller-strided (packed) gradient views";
    install_trace_handler();
    m.def("sdpa_bwd", &sdpa_bwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("dout"),
          py::arg("stats"), py::arg("dq"), py::arg("dk"), py::arg("dv"), py::arg("scale"));
    m.def("has_plan", &has_plan, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("dout"),
          py::arg("stats"), py::arg("dq"), py::arg("dk"), py::arg("dv"), py::arg("scale"));
    m.def("cudnn_version", [] { return static_cast<int64_t>(cudnnGetVersion()); });
}
