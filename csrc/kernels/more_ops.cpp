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

// Destination of a column reduction: `acc` (accumulated into, e.g. a parameter's .grad view) or a new tensor.
torch::Tensor reduce_target(const c10::optional<torch::Tensor>& acc, int64_t N, const torch::TensorOptions& o) {
    if (acc && acc->defined()) {
        TORCH_CHECK(acc->is_cuda() && acc->is_contiguous() && acc->numel() == N, "reduction target: [N] contiguous");
        return *acc;
    }
    return torch::empty({N}, o);
}

// sum over rows of a [M, N] tensor -> [N] in out_dtype, or added into `out`
// [R, C] bf16 with row rows[i] += src[i] (rows may repeat): the backward of src = table.index_select(0, rows)
torch::Tensor index_add_rows(torch::Tensor src, torch::Tensor rows, int64_t R) {
    TORCH_CHECK(src.is_cuda() && src.dim() == 2 && src.is_contiguous() && src.scalar_type() == torch::kBFloat16,
                "index_add_rows: src must be a contiguous bf16 [n, C] CUDA tensor");
    TORCH_CHECK(rows.is_cuda() && rows.scalar_type() == torch::kInt64 && rows.is_contiguous() &&
                    rows.numel() == src.size(0),
                "index_add_rows: rows must be a contiguous int64 [n] CUDA tensor");
    TORCH_CHECK(src.size(1) % 8 == 0, "index_add_rows: C % 8 == 0 required");
    at::cuda::CUDAGuard guard(src.device());
    auto out = torch::zeros({R, src.size(1)}, src.options());
    check_cuda(launch_index_add_rows(src.data_ptr(), rows.data_ptr<int64_t>(), out.data_ptr(), src.size(0),
                                     static_cast<int>(src.size(1)), cur_stream()),
               "index_add_rows");
    return out;
}

// [B, Cin, H, W] -> [B * (H/p) * (W/p), Cin * p * p]: non-overlapping patches as GEMM rows
torch::Tensor patch_unfold(torch::Tensor img, int64_t p) {
    TORCH_CHECK(img.is_cuda() && img.dim() == 4 && img.is_contiguous(), "patch_unfold: contiguous CUDA [B, C, H, W]");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(img.data_ptr()) % 16 == 0, "patch_unfold: 16-byte aligned image");
    const int64_t B = img.size(0), C = img.size(1), H = img.size(2), W = img.size(3);
    TORCH_CHECK(p % 8 == 0 && H % p == 0 && W % p == 0, "patch_unfold: p % 8 == 0 and p dividing H, W");
    at::cuda::CUDAGuard guard(img.device());
    auto out = torch::empty({B * (H / p) * (W / p), C * p * p}, img.options());
    check_cuda(launch_patch_unfold(dtype_of(img), img.data_ptr(), out.data_ptr(), static_cast<int>(B),
                                   static_cast<int>(C), static_cast<int>(H), static_cast<int>(W), static_cast<int>(p),
                                   cur_stream()),
               "patch_unfold");
    return out;
}

// indices of the k largest entries of every row of x [..., N] (sorted, value descending)
torch::Tensor row_topk(torch::Tensor x, int64_t k) {
    TORCH_CHECK(x.is_cuda() && x.dim() >= 1 && x.is_contiguous() &&
                    (x.scalar_type() == torch::kFloat32 || x.scalar_type() == torch::kBFloat16),
                "row_topk: contiguous fp32 / bf16 CUDA tensor expected");
    const int64_t N = x.size(-1);
    TORCH_CHECK(k >= 1 && k <= N && k <= 1024, "row_topk: 1 <= k <= min(N, 1024)");
    at::cuda::CUDAGuard guard(x.device());
    auto sizes = x.sizes().vec();
    sizes.back() = k;
    auto idx = torch::empty(sizes, x.options().dtype(torch::kInt64));
    check_cuda(launch_row_topk(dtype_of(x), x.data_ptr(), x.numel() / N, N, static_cast<int>(k), idx.data_ptr<int64_t>(),
                               cur_stream()),
               "row_topk");
    return idx;
}

// x [G, M, N] -> [G, N] column sums per group (fp32 accumulation), one launch
torch::Tensor colsum_grouped(torch::Tensor x, c10::optional<at::ScalarType> out_dtype) {
    TORCH_CHECK(x.is_cuda() && x.dim() == 3 && x.is_contiguous(), "colsum_grouped: contiguous CUDA [G, M, N] expected");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 && x.size(2) % 8 == 0,
                "colsum_grouped: 16-byte aligned rows, N % 8 == 0");
    at::cuda::CUDAGuard guard(x.device());
    auto ot = out_dtype.has_value() ? *out_dtype : x.scalar_type();
    auto o = torch::empty({x.size(0), x.size(2)}, x.options().dtype(ot));
    check_cuda(launch_colsum(dtype_of(x), dtype_of(o), 0, x.data_ptr(), nullptr, nullptr, nullptr, x.size(1),
                             static_cast<int>(x.size(2)), o.data_ptr(), cur_stream(), false, static_cast<int>(x.size(0))),
               "colsum_grouped");
    return o;
}

torch::Tensor colsum(torch::Tensor x, c10::optional<at::ScalarType> out_dtype, c10::optional<torch::Tensor> out) {
    TORCH_CHECK(x.is_cuda() && x.dim() == 2, "colsum: CUDA [M,N] expected");
    at::cuda::CUDAGuard guard(x.device());
    auto xc = aligned16(x);
    const int64_t M = xc.size(0);
    const int N = static_cast<int>(xc.size(1));
    auto ot = out_dtype.has_value() ? *out_dtype : xc.scalar_type();
    const bool acc = out && out->defined();
    auto o = reduce_target(out, N, xc.options().dtype(ot));
    check_cuda(launch_colsum(dtype_of(xc), dtype_of(o), 0, xc.data_ptr(), nullptr, nullptr, nullptr, M, N,
                             o.data_ptr(), cur_stream(), acc),
               "colsum");
    return o;
}

// LayerScale + bias backward in one pass: g_pre = gy * gamma, g_gamma (+)= colsum(gy * pre),
// g_bias (+)= colsum(g_pre) (bias_grad: accumulation target; bias_dtype: output dtype otherwise)
std::vector<torch::Tensor> scale_bias_bwd(torch::Tensor gy, torch::Tensor pre, torch::Tensor gamma,
                                          c10::optional<torch::Tensor> gamma_grad, c10::optional<torch::Tensor> bias_grad,
                                          c10::optional<at::ScalarType> bias_dtype) {
    TORCH_CHECK(gy.sizes() == pre.sizes() && gy.dim() == 2, "scale_bias_bwd: shape mismatch");
    TORCH_CHECK(gamma.scalar_type() == gy.scalar_type(), "scale_bias_bwd: gamma dtype must match");
    at::cuda::CUDAGuard guard(gy.device());
    auto g = aligned16(gy), p = aligned16(pre), gm = aligned16(gamma);
    const int64_t M = g.size(0);
    const int N = static_cast<int>(g.size(1));
    auto gpre = torch::empty_like(g);
    const bool acc_g = gamma_grad && gamma_grad->defined();
    const bool acc_b = bias_grad && bias_grad->defined();
    auto ggamma = reduce_target(gamma_grad, N, gamma.options());
    auto gbias = reduce_target(bias_grad, N, g.options().dtype(bias_dtype.has_value() ? *bias_dtype : g.scalar_type()));
    TORCH_CHECK(ggamma.scalar_type() == gbias.scalar_type(), "scale_bias_bwd: gamma / bias gradients share a dtype");
    check_cuda(launch_scale_bias_bwd(dtype_of(g), dtype_of(ggamma), g.data_ptr(), p.data_ptr(), gm.data_ptr(),
                                     gpre.data_ptr(), M, N, ggamma.data_ptr(), acc_g, gbias.data_ptr(), acc_b,
                                     cur_stream()),
               "scale_bias_bwd");
    return {gpre, ggamma, gbias};
}

// LayerScale backward: g_pre = gy * gamma, g_gamma (+)= colsum(gy * pre)
std::vector<torch::Tensor> scale_bwd(torch::Tensor gy, torch::Tensor pre, torch::Tensor gamma,
                                     c10::optional<torch::Tensor> gamma_grad) {
    TORCH_CHECK(gy.sizes() == pre.sizes() && gy.dim() == 2, "scale_bwd: shape mismatch");
    TORCH_CHECK(gamma.scalar_type() == gy.scalar_type(), "scale_bwd: gamma dtype must match");
    at::cuda::CUDAGuard guard(gy.device());
    auto g = aligned16(gy), p = aligned16(pre), gm = aligned16(gamma);
    const int64_t M = g.size(0);
    const int N = static_cast<int>(g.size(1));
    auto gpre = torch::empty_like(g);
    const bool acc = gamma_grad && gamma_grad->defined();
    auto ggamma = reduce_target(gamma_grad, N, gamma.options());
    check_cuda(launch_colsum(dtype_of(g), dtype_of(ggamma), 1, g.data_ptr(), p.data_ptr(), gm.data_ptr(),
                             gpre.data_ptr(), M, N, ggamma.data_ptr(), cur_stream(), acc),
               "scale_bwd");
    return {gpre, ggamma};
}

// g_pre = gy * act'(pre) and the bias gradient colsum(g_pre) in one pass (added into bias_grad if given)
std::vector<torch::Tensor> act_bwd_bias(torch::Tensor gy, torch::Tensor pre, int64_t act,
                                        c10::optional<torch::Tensor> bias_grad, c10::optional<at::ScalarType> dt) {
    TORCH_CHECK(gy.sizes() == pre.sizes() && gy.scalar_type() == pre.scalar_type() && gy.dim() == 2,
                "act_bwd_bias: mismatch");
    at::cuda::CUDAGuard guard(gy.device());
    auto g = aligned16(gy), p = aligned16(pre);
    const int64_t M = g.size(0);
    const int N = static_cast<int>(g.size(1));
    auto gpre = torch::empty_like(g);
    const bool acc = bias_grad && bias_grad->defined();
    auto gb = reduce_target(bias_grad, N, g.options().dtype(dt.has_value() ? *dt : g.scalar_type()));
    check_cuda(launch_act_bwd_bias(dtype_of(g), dtype_of(gb), g.data_ptr(), p.data_ptr(), gpre.data_ptr(), M, N,
                                   static_cast<int>(act), gb.data_ptr(), acc, cur_stream()),
               "act_bwd_bias");
    return {gpre, gb};
}

torch::Tensor gelu_fwd(torch::Tensor x) {
    TORCH_CHECK(x.is_cuda(), "gelu_fwd: CUDA tensor expected");
    at::cuda::CUDAGuard guard(x.device());
    auto xc = aligned16(x);
    auto y = torch::empty_like(xc);
    check_cuda(launch_gelu_fwd(dtype_of(xc), xc.data_ptr(), y.data_ptr(), xc.numel(), cur_stream()), "gelu_fwd");
    return y;
}

// (GELU(x), GELU'(x)) in one pass
std::vector<torch::Tensor> gelu_fwd_deriv(torch::Tensor x) {
    TORCH_CHECK(x.is_cuda(), "gelu_fwd_deriv: CUDA tensor expected");
    at::cuda::CUDAGuard guard(x.device());
    auto xc = aligned16(x);
    auto y = torch::empty_like(xc);
    auto d = torch::empty_like(xc);
    check_cuda(launch_gelu_fwd(dtype_of(xc), xc.data_ptr(), y.data_ptr(), xc.numel(), cur_stream(), d.data_ptr()),
               "gelu_fwd_deriv");
    return {y, d};
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

torch::Tensor sine_embed_fwd(torch::Tensor pos, int64_t dim, torch::Tensor freq) {
    TORCH_CHECK(pos.is_cuda() && pos.scalar_type() == torch::kFloat32 && freq.scalar_type() == torch::kFloat32,
                "sine_embed_fwd: CUDA fp32 pos / freq expected");
    at::cuda::CUDAGuard guard(pos.device());
    auto p = pos.contiguous();
    const int n = static_cast<int>(p.size(-1));
    const int64_t rows = p.numel() / n;
    auto sizes = p.sizes().vec();
    sizes.back() = n * dim;
    auto out = torch::empty(sizes, p.options().dtype(torch::kBFloat16));
    check_cuda(launch_sine_embed_fwd(p.data_ptr<float>(), rows, n, static_cast<int>(dim),
                                     freq.contiguous().data_ptr<float>(), out.data_ptr(), cur_stream()),
               "sine_embed_fwd");
    return out;
}

torch::Tensor sine_embed_bwd(torch::Tensor pos, int64_t dim, torch::Tensor freq, torch::Tensor gout) {
    at::cuda::CUDAGuard guard(pos.device());
    auto p = pos.contiguous();
    auto g = aligned16(gout.to(torch::kBFloat16));
    const int n = static_cast<int>(p.size(-1));
    const int64_t rows = p.numel() / n;
    auto gpos = torch::empty_like(p);
    check_cuda(launch_sine_embed_bwd(p.data_ptr<float>(), rows, n, static_cast<int>(dim),
                                     freq.contiguous().data_ptr<float>(), g.data_ptr(), gpos.data_ptr<float>(),
                                     cur_stream()),
               "sine_embed_bwd");
    return gpos;
}

}  // namespace

void register_more_ops(pybind11::module& m) {
    m.def("sine_embed_fwd", &sine_embed_fwd, py::arg("pos"), py::arg("dim"), py::arg("freq"));
    m.def("sine_embed_bwd", &sine_embed_bwd, py::arg("pos"), py::arg("dim"), py::arg("freq"), py::arg("gout"));
    m.def("dense_focal_neg_fwd", &dense_focal_neg_fwd);
    m.def("dense_focal_neg_bwd", &dense_focal_neg_bwd);
    m.def("colsum", &colsum, py::arg("x"), py::arg("out_dtype") = py::none(), py::arg("out") = py::none());
    m.def("index_add_rows", &index_add_rows, py::arg("src"), py::arg("rows"), py::arg("R"));
    m.def("colsum_grouped", &colsum_grouped, py::arg("x"), py::arg("out_dtype") = py::none());
    m.def("patch_unfold", &patch_unfold, py::arg("img"), py::arg("p"));
    m.def("row_topk", &row_topk, py::arg("x"), py::arg("k"));
    m.def("scale_bwd", &scale_bwd, py::arg("gy"), py::arg("pre"), py::arg("gamma"),
          py::arg("gamma_grad") = py::none());
    m.def("scale_bias_bwd", &scale_bias_bwd, py::arg("gy"), py::arg("pre"), py::arg("gamma"),
          py::arg("gamma_grad") = py::none(), py::arg("bias_grad") = py::none(), py::arg("bias_dtype") = py::none());
    m.def("act_bwd_bias", &act_bwd_bias, py::arg("gy"), py::arg("pre"), py::arg("act"),
          py::arg("bias_grad") = py::none(), py::arg("dtype") = py::none());
    m.def("act_bwd", &act_bwd);
    m.def("gelu_fwd", &gelu_fwd);
    m.def("gelu_fwd_deriv", &gelu_fwd_deriv);
    register_ddp_ops(m);
    register_gemm_ops(m);
    register_aug_ops(m);
    register_loss_ops(m);
    register_image_ops(m);
    register_attn_ops(m);
    register_overlay_ops(m);
    register_debug_ops(m);
}

}  // namespace mmltk
