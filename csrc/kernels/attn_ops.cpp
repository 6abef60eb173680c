// Torch wrapper of the tcgen05 attention forward (attn_tc.cu).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cmath>
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

AttnOperand operand(const torch::Tensor& src, int64_t col) {
    TORCH_CHECK(src.is_cuda() && src.scalar_type() == torch::kBFloat16 && src.dim() == 2 && src.stride(1) == 1,
                "attn_short: operands are CUDA bf16 [rows, cols] matrices with unit column stride");
    return AttnOperand{src.data_ptr(), src.stride(0), src.size(1), static_cast<int>(col)};
}

// Short-sequence attention forward: q / k / v are columns of 2-D source matrices (head h of each at
// column col + h * D, rows n * L + i).  Returns o [nseq * L, H * D] and lse [nseq, H, L].
std::vector<torch::Tensor> attn_short_fwd(torch::Tensor qs, int64_t qcol, torch::Tensor ks, int64_t kcol,
                                          torch::Tensor vs, int64_t vcol, int64_t nseq, int64_t L, int64_t heads,
                                          int64_t D) {
    TORCH_CHECK(attn_short_supported(static_cast<int>(L), static_cast<int>(D)), "attn_short: L <= 384, D in {32, 64}");
    for (const auto* t : {&qs, &ks, &vs})
        TORCH_CHECK(t->size(0) == nseq * L, "attn_short: every source has nseq * L rows");
    at::cuda::CUDAGuard guard(qs.device());
    auto o = torch::empty({nseq * L, heads * D}, qs.options());
    auto lse = torch::empty({nseq, heads, L}, qs.options().dtype(torch::kFloat32));
    check_cuda(launch_attn_short_fwd(operand(qs, qcol), operand(ks, kcol), operand(vs, vcol), static_cast<int>(nseq),
                                     static_cast<int>(L), static_cast<int>(heads), static_cast<int>(D), o.data_ptr(),
                                     o.stride(0), 0, lse.data_ptr<float>(), 1.f / std::sqrt(static_cast<float>(D)),
                                     attn_status_word(qs.device()).data_ptr<int>(), cur_stream()),
               "attn_short_fwd");
    return {o, lse};
}

// Backward: writes dq / dk / dv into columns of the given destination matrices (head h at col + h * D).
void attn_short_bwd(torch::Tensor qs, int64_t qcol, torch::Tensor ks, int64_t kcol, torch::Tensor vs, int64_t vcol,
                    torch::Tensor o, torch::Tensor dout, torch::Tensor lse, int64_t nseq, int64_t L, int64_t heads,
                    int64_t D, torch::Tensor dq, int64_t dqcol, torch::Tensor dk, int64_t dkcol, torch::Tensor dv,
                    int64_t dvcol) {
    TORCH_CHECK(attn_short_supported(static_cast<int>(L), static_cast<int>(D)), "attn_short: L <= 384, D in {32, 64}");
    TORCH_CHECK(lse.is_cuda() && lse.scalar_type() == torch::kFloat32 && lse.is_contiguous() &&
                    lse.numel() == nseq * heads * L,
                "attn_short_bwd: lse [nseq, H, L] fp32");
    for (const auto* t : {&o, &dout, &dq, &dk, &dv})
        TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kBFloat16 && t->dim() == 2 && t->stride(1) == 1 &&
                        t->size(0) == nseq * L,
                    "attn_short_bwd: o / dout / gradients are bf16 [nseq * L, cols]");
    at::cuda::CUDAGuard guard(qs.device());
    auto delta = torch::empty({nseq, heads, L}, lse.options());
    torch::Tensor acc;
    if (D == 64) acc = torch::empty({nseq * heads, L, 64}, lse.options());
    check_cuda(launch_attn_short_bwd(operand(qs, qcol), operand(ks, kcol), operand(vs, vcol), operand(dout, 0),
                                     o.data_ptr(), o.stride(0), 0, lse.data_ptr<float>(), delta.data_ptr<float>(),
                                     D == 64 ? acc.data_ptr<float>() : nullptr, static_cast<int>(nseq),
                                     static_cast<int>(L), static_cast<int>(heads), static_cast<int>(D), dq.data_ptr(),
                                     dq.stride(0), static_cast<int>(dqcol), dk.data_ptr(), dk.stride(0),
                                     static_cast<int>(dkcol), dv.data_ptr(), dv.stride(0), static_cast<int>(dvcol),
                                     1.f / std::sqrt(static_cast<float>(D)),
                                     attn_status_word(qs.device()).data_ptr<int>(), cur_stream()),
               "attn_short_bwd");
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
    m.def("attn_short_fwd", &attn_short_fwd);
    m.def("attn_short_bwd", &attn_short_bwd);
    m.def("attn_short_smem_bytes", &attn_short_smem_bytes);
    m.def("attn_short_set_fwd_variant", &attn_short_set_fwd_variant, py::arg("variant"));
    m.def("attn_short_fwd_variant", &attn_short_fwd_variant);
    m.def("attn_short_set_bwd_variant", &attn_short_set_bwd_variant, py::arg("variant"));
    m.def("attn_short_bwd_variant", &attn_short_bwd_variant);
    m.def("attn_tc_blocks_per_sm", &attn_fwd_tc_blocks_per_sm);
    m.def("attn_tc_set_variant", &attn_fwd_tc_set_variant, py::arg("min_blocks"));
}

}  // namespace mmltk
