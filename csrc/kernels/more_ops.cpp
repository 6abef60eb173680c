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

}  // namespace

void register_more_ops(pybind11::module& m) {
    m.def("dense_focal_neg_fwd", &dense_focal_neg_fwd);
    m.def("dense_focal_neg_bwd", &dense_focal_neg_bwd);
}

}  // namespace mmltk
