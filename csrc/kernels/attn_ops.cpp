// Torch wrapper of the tcgen05 attention forward (attn_tc.cu).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <mutex>
#include <vector>

#include "torch_ops.h"

namespace mmltk {

namespace {

torch::Tensor& attn_status_word(const torch::Device& dev) {
    static std::mutex mu;
    static std::vector<torch::Tensor> words(64);
    std::lock_guard<std::mutex> lk(mu);
    auto& t = words.at(dev.index());
    if (!t.defined()) t = torch::zeros({1}, torch::TensorOptions().dtype(torch::kInt32).device(dev));
    return t;
}

// qkv [N, L, 3 * H * 64] bf16 (last dim contiguous, rows evenly spaced) -> (o [N, L, H * 64], lse [N, H, L]
// or an empty tensor).
std::vector<torch::Tensor> attn_fwd_tc(torch::Tensor qkv, int64_t heads, bool want_lse) {
    TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == torch::kBFloat16 && qkv.dim() == 3,
                "attn_fwd_tc: CUDA bf16 [N, L, 3C] expected");
    const int64_t N = qkv.size(0), L = qkv.size(1), C = heads * 64;
    TORCH_CHECK(qkv.size(2) == 3 * C, "attn_fwd_tc: head dim must be 64 (got last dim ", qkv.size(2), " for ", heads,
                " heads)");
    at::cuda::CUDAGuard guard(qkv.device());
    auto x = qkv;
    if (x.stride(2) != 1 || x.stride(1) % 8 != 0 || (N > 1 && x.stride(0) != L * x.stride(1)) ||
        reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 != 0)
        x = x.contiguous();
    auto o = torch::empty({N, L, C}, x.options());
    torch::Tensor lse;
    if (want_lse) lse = torch::empty({N, heads, L}, x.options().dtype(torch::kFloat32));
    check_cuda(launch_attn_fwd_tc(x.data_ptr(), x.stride(1), static_cast<int>(N), static_cast<int>(L),
                                  static_cast<int>(heads), o.data_ptr(), C, want_lse ? lse.data_ptr<float>() : nullptr,
                                  0.125f, attn_status_word(x.device()).data_ptr<int>(), cur_stream()),
               "attn_fwd_tc");
    return {o, want_lse ? lse : torch::empty({0}, x.options().dtype(torch::kFloat32))};
}

int64_t attn_tc_status(int64_t device) {
    auto& t = attn_status_word(torch::Device(torch::kCUDA, static_cast<c10::DeviceIndex>(device)));
    const int64_t v = t.item<int>();
    if (v) t.zero_();
    return v;
}

}  // namespace

void register_attn_ops(pybind11::module& m) {
    m.def("attn_fwd_tc", &attn_fwd_tc, py::arg("qkv"), py::arg("heads"), py::arg("want_lse") = false);
    m.def("attn_tc_status", &attn_tc_status, py::arg("device") = 0);
    m.def("attn_tc_blocks_per_sm", &attn_fwd_tc_blocks_per_sm);
    m.def("attn_tc_set_variant", &attn_fwd_tc_set_variant, py::arg("min_blocks"));
}

}  // namespace mmltk
