// Torch wrappers of the op families that have their own kernel files.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "torch_ops.h"

namespace mmltk {

namespace {

torch::Tensor aligned16(const torch::Tensor& t) {
    auto c = t.contiguous();
    if (reinterpret_cast<uintptr_t>(c.data_ptr()) % 16 != 0) c = c.clone();
    return c;
}

torch::Tensor dense_focal_neg_fwd(torch::Tensor x, double coef) {
    TORCH_CHECK(x.is_cuda(), "dense_focal_neg_fwd: CUDA tensor expected");
    at::cuda::CUDAGuard guard(x.device());
    auto xc = aligned16(x);
    const int64_t n = xc.numel();
    auto opts = xc.options().dtype(torch::kFloat32);
    auto partials = torch::empty({dense_neg_blocks(n)}, opts);
    auto counter = torch::zeros({1}, xc.options().dtype(torch::kInt32));
    auto out = torch::empty({}, opts);
    check_cuda(launch_dense_neg_fwd(dtype_of(xc), xc.data_ptr(), n, static_cast<float>(coef),
                                    partials.data_ptr<float>(), reinterpret_cast<unsigned int*>(counter.data_ptr()),
                                    out.data_ptr<float>(), cur_stream()),
               "dense_focal_neg_fwd");
    return out;
}

torch::Tensor dense_focal_neg_bwd(torch::Tensor x, torch::Tensor g, double coef) {
    at::cuda::CUDAGuard guard(x.device());
    auto xc = aligned16(x);
    auto gf = g.to(torch::kFloat32).contiguous();
    auto dx = torch::empty_like(xc);
    check_cuda(launch_dense_neg_bwd(dtype_of(xc), xc.data_ptr(), gf.data_ptr<float>(), xc.numel(),
                                    static_cast<float>(coef), dx.data_ptr(), cur_stream()),
               "dense_focal_neg_bwd");
    return dx.view(x.sizes());
}

// sum over rows of a [M, N] tensor -> [N] in out_dtype
torch::Tensor colsum(torch::Tensor x, c10::optional<at::ScalarType> out_dtype) {
    TORCH_CHECK(x.is_cuda() && x.dim() == 2, "colsum: CUDA [M,N] expected");
    at::cuda::CUDAGuard guard(x.device());
    auto xc = aligned16(x);
    const int64_t M = xc.size(0);
    const int N = static_cast<int>(xc.size(1));
    auto ot = out_dtype.has_value() ? *out_dtype : xc.scalar_type();
    auto out = torch::empty({N}, xc.options().dtype(ot));
    auto part = torch::empty({colsum_parts(M, N), N}, xc.options().dtype(torch::kFloat32));
    check_cuda(launch_colsum(dtype_of(xc), dtype_of(out), 0, xc.data_ptr(), nullptr, nullptr, nullptr, M, N,
                             part.data_ptr<float>(), out.data_ptr(), cur_stream()),
               "colsum");
    return out;
}

// LayerScale backward: g_pre = gy * gamma, g_gamma = colsum(gy * pre)
std::vector<torch::Tensor> scale_bwd(torch::Tensor gy, torch::Tensor pre, torch::Tensor gamma) {
    TORCH_CHECK(gy.sizes() == pre.sizes() && gy.dim() == 2, "scale_bwd: shape mismatch");
    TORCH_CHECK(gamma.scalar_type() == gy.scalar_type(), "scale_bwd: gamma dtype must match");
    at::cuda::CUDAGuard guard(gy.device());
    auto g = aligned16(gy), p = aligned16(pre), gm = aligned16(gamma);
    const int64_t M = g.size(0);
    const int N = static_cast<int>(g.size(1));
    auto gpre = torch::empty_like(g);
    auto ggamma = torch::empty({N}, gamma.options());
    auto part = torch::empty({colsum_parts(M, N), N}, g.options().dtype(torch::kFloat32));
    check_cuda(launch_colsum(dtype_of(g), dtype_of(gamma), 1, g.data_ptr(), p.data_ptr(), gm.data_ptr(),
                             gpre.data_ptr(), M, N, part.data_ptr<float>(), ggamma.data_ptr(), cur_stream()),
               "scale_bwd");
    return {gpre, ggamma};
}

torch::Tensor act_bwd(torch::Tensor gy, torch::Tensor pre, int64_t act) {
    TORCH_CHECK(gy.sizes() == pre.sizes() && gy.scalar_type() == pre.scalar_type(), "act_bwd: mismatch");
    at::cuda::CUDAGuard guard(gy.device());
    auto g = aligned16(gy), p = aligned16(pre);
    auto out = torch::empty_like(g);
    check_cuda(launch_act_bwd(dtype_of(g), g.data_ptr(), p.data_ptr(), out.data_ptr(), g.numel(),
                              static_cast<int>(act), cur_stream()),
               "act_bwd");
    return out;
}

}  // namespace

void register_more_ops(pybind11::module& m) {
    m.def("dense_focal_neg_fwd", &dense_focal_neg_fwd);
    m.def("dense_focal_neg_bwd", &dense_focal_neg_bwd);
    m.def("colsum", &colsum, py::arg("x"), py::arg("out_dtype") = py::none());
    m.def("scale_bwd", &scale_bwd);
    m.def("act_bwd", &act_bwd);
    register_ddp_ops(m);
    register_gemm_ops(m);
    register_aug_ops(m);
}

}  // namespace mmltk
