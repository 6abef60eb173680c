// Torch-facing wrappers and Python bindings of the sm_100a kernel library
// (`mmltk_b200._kernels`).  Shape/dtype checks and allocation happen here
// (g++); the kernels themselves are launched through launch_api.h.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <mutex>
#include <vector>

#include "launch_api.h"
#include "optim.cuh"
#include "torch_ops.h"

namespace mmltk {

int num_sms() {
    static std::mutex mu;
    static std::vector<int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    std::lock_guard<std::mutex> lk(mu);
    if (static_cast<int>(cache.size()) <= dev) cache.resize(dev + 1, 0);
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

DType dtype_of(const torch::Tensor& t) {
    if (t.scalar_type() == torch::kBFloat16) return DType::kBF16;
    TORCH_CHECK(t.scalar_type() == torch::kFloat32, "mmltk kernels support bf16 and fp32 tensors only, got ",
                t.scalar_type());
    return DType::kF32;
}

void check_cuda(cudaError_t e, const char* what) {
    TORCH_CHECK(e == cudaSuccess, what, ": ", cudaGetErrorString(e));
}

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

namespace {

// ---------------------------------------------------------------- LayerNorm
// res: normalise x + res (the sum is returned too); pos: also return y + pos.
// Returns {y, mean, rstd, sum (or undefined), y + pos (or undefined)}.
std::vector<torch::Tensor> layernorm_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor b, double eps,
                                         c10::optional<torch::Tensor> res, c10::optional<torch::Tensor> pos,
                                         c10::optional<torch::Tensor> rbias, c10::optional<torch::Tensor> rscale) {
    TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous(), "layernorm_fwd: x must be contiguous [rows, C]");
    TORCH_CHECK(w.scalar_type() == b.scalar_type() && w.numel() == x.size(1) && b.numel() == x.size(1),
                "layernorm_fwd: weight/bias must match C and share a dtype");
    const bool has_res = res && res->defined(), has_pos = pos && pos->defined();
    const bool has_rb = rbias && rbias->defined();
    if (has_rb)
        TORCH_CHECK(has_res && rbias->numel() == x.size(1) && rbias->is_contiguous() &&
                        rbias->scalar_type() == w.scalar_type(),
                    "layernorm_fwd: rbias needs res and must be a contiguous [C] vector of the weight dtype");
    const bool has_rs = rscale && rscale->defined();
    if (has_rs)
        TORCH_CHECK(has_res && rscale->numel() == x.size(1) && rscale->is_contiguous() &&
                        rscale->scalar_type() == w.scalar_type(),
                    "layernorm_fwd: rscale needs res and must be a contiguous [C] vector of the weight dtype");
    if (has_res)
        TORCH_CHECK(res->sizes() == x.sizes() && res->is_contiguous() && res->scalar_type() == x.scalar_type(),
                    "layernorm_fwd: res must match x");
    if (has_pos)
        TORCH_CHECK(pos->sizes() == x.sizes() && pos->is_contiguous() && pos->scalar_type() == x.scalar_type(),
                    "layernorm_fwd: pos must match x");
    at::cuda::CUDAGuard guard(x.device());
    const int64_t rows = x.size(0);
    const int C = static_cast<int>(x.size(1));
    auto y = torch::empty_like(x);
    auto opts = x.options().dtype(torch::kFloat32);
    auto mean = torch::empty({rows}, opts);
    auto rstd = torch::empty({rows}, opts);
    auto wc = w.contiguous(), bc = b.contiguous();
    torch::Tensor sum, y2;
    if (has_res) sum = torch::empty_like(x);
    if (has_pos) y2 = torch::empty_like(x);
    check_cuda(launch_layernorm_fwd(dtype_of(x), dtype_of(w), x.data_ptr(), wc.data_ptr(), bc.data_ptr(), y.data_ptr(),
                                    mean.data_ptr<float>(), rstd.data_ptr<float>(), rows, C, static_cast<float>(eps),
                                    cur_stream(), has_res ? res->data_ptr() : nullptr,
                                    has_res ? sum.data_ptr() : nullptr, has_pos ? pos->data_ptr() : nullptr,
                                    has_pos ? y2.data_ptr() : nullptr, has_rb ? rbias->data_ptr() : nullptr,
                                    has_rs ? rscale->data_ptr() : nullptr),
               "layernorm_fwd");
    return {y, mean, rstd, sum, y2};
}

// gw_acc / gb_acc: when given (a parameter's .grad view), the weight / bias gradients are added into them
// gy2: gradient of the forward's y + pos output, added to gy inside the kernel
std::vector<torch::Tensor> layernorm_bwd(torch::Tensor gy, torch::Tensor x, torch::Tensor w, torch::Tensor mean,
                                         torch::Tensor rstd, c10::optional<torch::Tensor> gw_acc,
                                         c10::optional<torch::Tensor> gb_acc, c10::optional<torch::Tensor> gy2,
                                         c10::optional<torch::Tensor> gres, bool want_gbias2,
                                         c10::optional<torch::Tensor> gbias2_acc) {
    const bool has_g2 = gy2 && gy2->defined();
    const bool has_res = gres && gres->defined();
    if (has_res)
        TORCH_CHECK(gres->sizes() == x.sizes() && gres->is_contiguous() && gres->scalar_type() == x.scalar_type(),
                    "layernorm_bwd: gres must match x");
    if (has_g2)
        TORCH_CHECK(gy2->sizes() == x.sizes() && gy2->is_contiguous() && gy2->scalar_type() == x.scalar_type(),
                    "layernorm_bwd: gy2 must match x");
    TORCH_CHECK(gy.sizes() == x.sizes() && gy.is_contiguous() && x.is_contiguous() &&
                    gy.scalar_type() == x.scalar_type(),
                "layernorm_bwd: grad/x mismatch");
    at::cuda::CUDAGuard guard(x.device());
    const int64_t rows = x.size(0);
    const int C = static_cast<int>(x.size(1));
    auto gx = torch::empty_like(x);
    auto wc = w.contiguous();
    const bool acc = gw_acc && gw_acc->defined() && gb_acc && gb_acc->defined();
    if (acc) {
        TORCH_CHECK(gw_acc->is_contiguous() && gb_acc->is_contiguous() && gw_acc->numel() == C &&
                        gb_acc->numel() == C && gw_acc->scalar_type() == w.scalar_type() &&
                        gb_acc->scalar_type() == w.scalar_type(),
                    "layernorm_bwd: accumulation targets must be contiguous [C] of the weight dtype");
    }
    auto gw = acc ? *gw_acc : torch::empty_like(wc);
    auto gb = acc ? *gb_acc : torch::empty_like(wc);
    const bool acc2 = gbias2_acc && gbias2_acc->defined();
    if (acc2)
        TORCH_CHECK(gbias2_acc->is_contiguous() && gbias2_acc->numel() == C && gbias2_acc->scalar_type() == w.scalar_type(),
                    "layernorm_bwd: gbias2 target must be a contiguous [C] of the weight dtype");
    torch::Tensor gb2;
    if (want_gbias2 || acc2) gb2 = acc2 ? *gbias2_acc : torch::empty_like(wc);
    check_cuda(launch_layernorm_bwd(dtype_of(x), dtype_of(w), gy.data_ptr(), x.data_ptr(), wc.data_ptr(),
                                    mean.data_ptr<float>(), rstd.data_ptr<float>(), gx.data_ptr(), gw.data_ptr(),
                                    gb.data_ptr(), rows, C, acc, cur_stream(), has_g2 ? gy2->data_ptr() : nullptr,
                                    has_res ? gres->data_ptr() : nullptr, gb2.defined() ? gb2.data_ptr() : nullptr, acc2),
               "layernorm_bwd");
    return {gx, gw, gb, gb2};
}

// LayerNorm whose row r lands in row ymap[r] (none when negative) of `out` [R, ld] at column `col`:
// e.g. the backbone taps, normalised straight into their un-windowed place in the projector's
// channel-concatenated input.  Returns {mean, rstd}.
std::vector<torch::Tensor> layernorm_fwd_map(torch::Tensor x, torch::Tensor w, torch::Tensor b, double eps,
                                             torch::Tensor ymap, torch::Tensor out, int64_t col) {
    TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous(), "layernorm_fwd_map: x must be contiguous [rows, C]");
    const int64_t rows = x.size(0), C = x.size(1);
    TORCH_CHECK(w.scalar_type() == b.scalar_type() && w.numel() == C && b.numel() == C,
                "layernorm_fwd_map: weight/bias must match C and share a dtype");
    TORCH_CHECK(ymap.is_cuda() && ymap.scalar_type() == torch::kInt32 && ymap.numel() == rows && ymap.is_contiguous(),
                "layernorm_fwd_map: ymap must be a contiguous int32 [rows] CUDA tensor");
    TORCH_CHECK(out.is_cuda() && out.dim() == 2 && out.stride(1) == 1 && out.scalar_type() == x.scalar_type() &&
                    col >= 0 && col + C <= out.size(1) && col % 4 == 0 && out.stride(0) % 4 == 0,
                "layernorm_fwd_map: out must be a row-major [R, >= col + C] tensor of the x dtype");
    at::cuda::CUDAGuard guard(x.device());
    auto opts = x.options().dtype(torch::kFloat32);
    auto mean = torch::empty({rows}, opts);
    auto rstd = torch::empty({rows}, opts);
    auto wc = w.contiguous(), bc = b.contiguous();
    void* y = static_cast<char*>(out.data_ptr()) + col * out.element_size();
    check_cuda(launch_layernorm_fwd(dtype_of(x), dtype_of(w), x.data_ptr(), wc.data_ptr(), bc.data_ptr(), y,
                                    mean.data_ptr<float>(), rstd.data_ptr<float>(), rows, static_cast<int>(C),
                                    static_cast<float>(eps), cur_stream(), nullptr, nullptr, nullptr, nullptr, nullptr,
                                    nullptr, ymap.data_ptr<int>(), out.stride(0)),
               "layernorm_fwd_map");
    return {mean, rstd};
}

// Backward of layernorm_fwd_map: the output gradient of row r is row gmap[r] of g [R, ld] at column
// `col` (zero when negative).  Returns {gx, gw, gb} (gw / gb added into gw_acc / gb_acc when given).
std::vector<torch::Tensor> layernorm_bwd_map(torch::Tensor g, int64_t col, torch::Tensor gmap, torch::Tensor x,
                                             torch::Tensor w, torch::Tensor mean, torch::Tensor rstd,
                                             c10::optional<torch::Tensor> gw_acc, c10::optional<torch::Tensor> gb_acc) {
    TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous(), "layernorm_bwd_map: x must be contiguous [rows, C]");
    const int64_t rows = x.size(0), C = x.size(1);
    TORCH_CHECK(gmap.is_cuda() && gmap.scalar_type() == torch::kInt32 && gmap.numel() == rows && gmap.is_contiguous(),
                "layernorm_bwd_map: gmap must be a contiguous int32 [rows] CUDA tensor");
    TORCH_CHECK(g.is_cuda() && g.dim() == 2 && g.stride(1) == 1 && g.scalar_type() == x.scalar_type() && col >= 0 &&
                    col + C <= g.size(1) && col % 4 == 0 && g.stride(0) % 4 == 0,
                "layernorm_bwd_map: g must be a row-major [R, >= col + C] tensor of the x dtype");
    at::cuda::CUDAGuard guard(x.device());
    auto gx = torch::empty_like(x);
    auto wc = w.contiguous();
    const bool acc = gw_acc && gw_acc->defined() && gb_acc && gb_acc->defined();
    if (acc)
        TORCH_CHECK(gw_acc->is_contiguous() && gb_acc->is_contiguous() && gw_acc->numel() == C && gb_acc->numel() == C &&
                        gw_acc->scalar_type() == w.scalar_type() && gb_acc->scalar_type() == w.scalar_type(),
                    "layernorm_bwd_map: accumulation targets must be contiguous [C] of the weight dtype");
    auto gw = acc ? *gw_acc : torch::empty_like(wc);
    auto gb = acc ? *gb_acc : torch::empty_like(wc);
    const void* gy = static_cast<const char*>(g.data_ptr()) + col * g.element_size();
    check_cuda(launch_layernorm_bwd(dtype_of(x), dtype_of(w), gy, x.data_ptr(), wc.data_ptr(), mean.data_ptr<float>(),
                                    rstd.data_ptr<float>(), gx.data_ptr(), gw.data_ptr(), gb.data_ptr(), rows,
                                    static_cast<int>(C), acc, cur_stream(), nullptr, nullptr, nullptr, false,
                                    gmap.data_ptr<int>(), g.stride(0)),
               "layernorm_bwd_map");
    return {gx, gw, gb};
}

// LayerNorm with one weight / bias row per group of rows: x [G * R, C] (group g = rows [g R, (g+1) R)),
// w / b [G, C] -- the two-stage head's per-group encoder-output norms.  Returns {y, mean, rstd}.
std::vector<torch::Tensor> layernorm_grouped_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor b, double eps) {
    TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous(), "layernorm_grouped_fwd: x must be contiguous [rows, C]");
    TORCH_CHECK(w.dim() == 2 && w.sizes() == b.sizes() && w.size(1) == x.size(1) && w.scalar_type() == b.scalar_type() &&
                    x.size(0) % w.size(0) == 0,
                "layernorm_grouped_fwd: weight / bias must be [G, C] with G dividing the rows");
    at::cuda::CUDAGuard guard(x.device());
    const int64_t rows = x.size(0);
    auto y = torch::empty_like(x);
    auto opts = x.options().dtype(torch::kFloat32);
    auto mean = torch::empty({rows}, opts);
    auto rstd = torch::empty({rows}, opts);
    auto wc = w.contiguous(), bc = b.contiguous();
    check_cuda(launch_layernorm_fwd(dtype_of(x), dtype_of(w), x.data_ptr(), wc.data_ptr(), bc.data_ptr(), y.data_ptr(),
                                    mean.data_ptr<float>(), rstd.data_ptr<float>(), rows, static_cast<int>(x.size(1)),
                                    static_cast<float>(eps), cur_stream(), nullptr, nullptr, nullptr, nullptr, nullptr,
                                    nullptr, nullptr, 0, rows / w.size(0)),
               "layernorm_grouped_fwd");
    return {y, mean, rstd};
}

// Backward of layernorm_grouped_fwd: {gx, gw [G, C], gb [G, C]} (added into gw_acc / gb_acc when given).
std::vector<torch::Tensor> layernorm_grouped_bwd(torch::Tensor gy, torch::Tensor x, torch::Tensor w, torch::Tensor mean,
                                                 torch::Tensor rstd, c10::optional<torch::Tensor> gw_acc,
                                                 c10::optional<torch::Tensor> gb_acc) {
    TORCH_CHECK(gy.sizes() == x.sizes() && gy.is_contiguous() && x.is_contiguous() && gy.scalar_type() == x.scalar_type(),
                "layernorm_grouped_bwd: grad/x mismatch");
    TORCH_CHECK(w.dim() == 2 && w.size(1) == x.size(1) && x.size(0) % w.size(0) == 0,
                "layernorm_grouped_bwd: weight must be [G, C] with G dividing the rows");
    at::cuda::CUDAGuard guard(x.device());
    const int64_t rows = x.size(0);
    auto gx = torch::empty_like(x);
    auto wc = w.contiguous();
    const bool acc = gw_acc && gw_acc->defined() && gb_acc && gb_acc->defined();
    if (acc)
        TORCH_CHECK(gw_acc->is_contiguous() && gb_acc->is_contiguous() && gw_acc->numel() == w.numel() &&
                        gb_acc->numel() == w.numel() && gw_acc->scalar_type() == w.scalar_type() &&
                        gb_acc->scalar_type() == w.scalar_type(),
                    "layernorm_grouped_bwd: accumulation targets must be contiguous [G, C] of the weight dtype");
    auto gw = acc ? *gw_acc : torch::empty_like(wc);
    auto gb = acc ? *gb_acc : torch::empty_like(wc);
    check_cuda(launch_layernorm_bwd(dtype_of(x), dtype_of(w), gy.data_ptr(), x.data_ptr(), wc.data_ptr(),
                                    mean.data_ptr<float>(), rstd.data_ptr<float>(), gx.data_ptr(), gw.data_ptr(),
                                    gb.data_ptr(), rows, static_cast<int>(x.size(1)), acc, cur_stream(), nullptr,
                                    nullptr, nullptr, false, nullptr, 0, rows / w.size(0)),
               "layernorm_grouped_bwd");
    return {gx, gw, gb};
}

// y = SiLU(LN(x)) (act 1): the projector's ConvX norm + activation in one pass.  Returns {y, mean, rstd}.
std::vector<torch::Tensor> layernorm_act_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor b, double eps,
                                             int64_t act) {
    TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous(), "layernorm_act_fwd: x must be contiguous [rows, C]");
    TORCH_CHECK(w.scalar_type() == b.scalar_type() && w.numel() == x.size(1) && b.numel() == x.size(1),
                "layernorm_act_fwd: weight/bias must match C and share a dtype");
    TORCH_CHECK(act == 1, "layernorm_act_fwd: act 1 (SiLU) only");
    at::cuda::CUDAGuard guard(x.device());
    const int64_t rows = x.size(0);
    auto y = torch::empty_like(x);
    auto opts = x.options().dtype(torch::kFloat32);
    auto mean = torch::empty({rows}, opts);
    auto rstd = torch::empty({rows}, opts);
    auto wc = w.contiguous(), bc = b.contiguous();
    check_cuda(launch_layernorm_fwd(dtype_of(x), dtype_of(w), x.data_ptr(), wc.data_ptr(), bc.data_ptr(), y.data_ptr(),
                                    mean.data_ptr<float>(), rstd.data_ptr<float>(), rows, static_cast<int>(x.size(1)),
                                    static_cast<float>(eps), cur_stream(), nullptr, nullptr, nullptr, nullptr, nullptr,
                                    nullptr, nullptr, 0, 0, static_cast<int>(act)),
               "layernorm_act_fwd");
    return {y, mean, rstd};
}

// Backward of layernorm_act_fwd: {gx, gw, gb} (added into gw_acc / gb_acc when given).
std::vector<torch::Tensor> layernorm_act_bwd(torch::Tensor gy, torch::Tensor x, torch::Tensor w, torch::Tensor b,
                                             torch::Tensor mean, torch::Tensor rstd, int64_t act,
                                             c10::optional<torch::Tensor> gw_acc, c10::optional<torch::Tensor> gb_acc) {
    TORCH_CHECK(gy.sizes() == x.sizes() && gy.is_contiguous() && x.is_contiguous() && gy.scalar_type() == x.scalar_type(),
                "layernorm_act_bwd: grad/x mismatch");
    TORCH_CHECK(act == 1 && b.numel() == x.size(1) && b.scalar_type() == w.scalar_type(), "layernorm_act_bwd: bad args");
    at::cuda::CUDAGuard guard(x.device());
    const int64_t rows = x.size(0);
    const int C = static_cast<int>(x.size(1));
    auto gx = torch::empty_like(x);
    auto wc = w.contiguous(), bc = b.contiguous();
    const bool acc = gw_acc && gw_acc->defined() && gb_acc && gb_acc->defined();
    if (acc)
        TORCH_CHECK(gw_acc->is_contiguous() && gb_acc->is_contiguous() && gw_acc->numel() == C && gb_acc->numel() == C &&
                        gw_acc->scalar_type() == w.scalar_type() && gb_acc->scalar_type() == w.scalar_type(),
                    "layernorm_act_bwd: accumulation targets must be contiguous [C] of the weight dtype");
    auto gw = acc ? *gw_acc : torch::empty_like(wc);
    auto gb = acc ? *gb_acc : torch::empty_like(wc);
    check_cuda(launch_layernorm_bwd(dtype_of(x), dtype_of(w), gy.data_ptr(), x.data_ptr(), wc.data_ptr(),
                                    mean.data_ptr<float>(), rstd.data_ptr<float>(), gx.data_ptr(), gw.data_ptr(),
                                    gb.data_ptr(), rows, C, acc, cur_stream(), nullptr, nullptr, nullptr, false, nullptr,
                                    0, 0, bc.data_ptr(), static_cast<int>(act)),
               "layernorm_act_bwd");
    return {gx, gw, gb};
}

// ---------------------------------------------------------------- MSDeformAttn
MsdaDims msda_dims(const torch::Tensor& value, const torch::Tensor& shapes, const torch::Tensor& starts,
                   const torch::Tensor& ref, const torch::Tensor& off, const torch::Tensor& logits) {
    TORCH_CHECK(value.is_cuda() && value.dim() == 4 && value.is_contiguous(), "msda: value must be [B,S,H,D]");
    TORCH_CHECK(off.dim() == 6 && off.is_contiguous() && off.size(5) == 2, "msda: offsets must be [B,Lq,H,L,P,2]");
    TORCH_CHECK(ref.dim() == 4 && ref.is_contiguous() && ref.size(3) == 4, "msda: ref must be [B,Lq,L,4]");
    TORCH_CHECK(logits.is_contiguous(), "msda: attention logits must be contiguous");
    TORCH_CHECK(shapes.scalar_type() == torch::kInt32 && starts.scalar_type() == torch::kInt32 && shapes.is_cuda(),
                "msda: shapes/starts must be CUDA int32");
    TORCH_CHECK(value.scalar_type() == ref.scalar_type() && value.scalar_type() == off.scalar_type() &&
                    value.scalar_type() == logits.scalar_type(),
                "msda: value/ref/offsets/logits must share one dtype");
    MsdaDims d;
    d.B = static_cast<int>(value.size(0));
    d.S = static_cast<int>(value.size(1));
    d.H = static_cast<int>(value.size(2));
    d.D = static_cast<int>(value.size(3));
    d.Lq = static_cast<int>(off.size(1));
    d.L = static_cast<int>(off.size(3));
    d.P = static_cast<int>(off.size(4));
    TORCH_CHECK(off.size(0) == d.B && off.size(2) == d.H, "msda: offsets batch/head mismatch");
    TORCH_CHECK(ref.size(0) == d.B && ref.size(1) == d.Lq && ref.size(2) == d.L, "msda: ref shape mismatch");
    TORCH_CHECK(logits.numel() == static_cast<int64_t>(d.B) * d.Lq * d.H * d.L * d.P, "msda: logits numel");
    TORCH_CHECK(d.L <= 8 && d.L * d.P <= 32, "msda: at most 8 levels and 32 points per head");
    TORCH_CHECK(d.D % 8 == 0 && d.D >= 8 && d.D <= 128, "msda: head dim must be 8, 16, 32, 64 or 128");
    TORCH_CHECK(shapes.size(0) == d.L && starts.numel() == d.L, "msda: level table mismatch");
    return d;
}

torch::Tensor msda_fwd(torch::Tensor value, torch::Tensor shapes, torch::Tensor starts, torch::Tensor ref,
                       torch::Tensor off, torch::Tensor logits) {
    MsdaDims d = msda_dims(value, shapes, starts, ref, off, logits);
    at::cuda::CUDAGuard guard(value.device());
    auto out = torch::empty({d.B, d.Lq, d.H * d.D}, value.options());
    check_cuda(launch_msda_fwd(dtype_of(value), value.data_ptr(), shapes.data_ptr<int>(), starts.data_ptr<int>(),
                               ref.data_ptr(), off.data_ptr(), logits.data_ptr(), out.data_ptr(), d, cur_stream()),
               "msda_fwd");
    return out;
}

std::vector<torch::Tensor> msda_bwd(torch::Tensor gout, torch::Tensor value, torch::Tensor shapes,
                                    torch::Tensor starts, torch::Tensor ref, torch::Tensor off, torch::Tensor logits) {
    MsdaDims d = msda_dims(value, shapes, starts, ref, off, logits);
    TORCH_CHECK(gout.is_contiguous() && gout.scalar_type() == value.scalar_type() &&
                    gout.numel() == static_cast<int64_t>(d.B) * d.Lq * d.H * d.D,
                "msda_bwd: grad dtype/layout");
    at::cuda::CUDAGuard guard(value.device());
    auto gvalue = torch::empty_like(value);
    auto gref = torch::empty_like(ref);
    auto goff = torch::empty_like(off);
    auto glogits = torch::empty_like(logits);
    auto acc = torch::empty({value.numel() + ref.numel()}, value.options().dtype(torch::kFloat32));
    check_cuda(launch_msda_bwd(dtype_of(value), gout.data_ptr(), value.data_ptr(), shapes.data_ptr<int>(),
                               starts.data_ptr<int>(), ref.data_ptr(), off.data_ptr(), logits.data_ptr(),
                               acc.data_ptr<float>(), acc.data_ptr<float>() + value.numel(), gvalue.data_ptr(),
                               gref.data_ptr(), goff.data_ptr(), glogits.data_ptr(), d, cur_stream()),
               "msda_bwd");
    return {gvalue, gref, goff, glogits};
}

// ---------------------------------------------------------------- matcher
torch::Tensor matcher_cost(std::vector<torch::Tensor> logits, std::vector<torch::Tensor> boxes, torch::Tensor labels,
                           torch::Tensor tboxes, torch::Tensor counts, double w_class, double w_bbox, double w_giou,
                           double alpha) {
    const int NL = static_cast<int>(logits.size());
    TORCH_CHECK(NL >= 1 && NL <= kMatcherMaxLayers && boxes.size() == logits.size(), "matcher_cost: 1..8 layers");
    const auto& l0 = logits[0];
    TORCH_CHECK(l0.is_cuda() && l0.dim() == 3, "matcher_cost: logits must be CUDA [B,Q,C]");
    const int B = static_cast<int>(l0.size(0)), Q = static_cast<int>(l0.size(1)), C = static_cast<int>(l0.size(2));
    TORCH_CHECK(labels.dim() == 2 && labels.size(0) == B && labels.scalar_type() == torch::kInt64,
                "matcher_cost: labels must be int64 [B,T]");
    const int T = static_cast<int>(labels.size(1));
    TORCH_CHECK(tboxes.scalar_type() == torch::kFloat32 && tboxes.is_contiguous() && tboxes.dim() == 3 &&
                    tboxes.size(0) == B && tboxes.size(1) == T,
                "matcher_cost: target boxes must be fp32 [B,T,4]");
    TORCH_CHECK(counts.scalar_type() == torch::kInt32 && counts.numel() == B, "matcher_cost: counts int32 [B]");
    at::cuda::CUDAGuard guard(l0.device());
    MatcherLayers lp{};
    std::vector<torch::Tensor> keep;
    for (int i = 0; i < NL; ++i) {
        TORCH_CHECK(logits[i].sizes() == l0.sizes() && logits[i].scalar_type() == l0.scalar_type(),
                    "matcher_cost: all layers must share shape/dtype");
        TORCH_CHECK(boxes[i].dim() == 3 && boxes[i].size(0) == B && boxes[i].size(1) == Q && boxes[i].size(2) == 4 &&
                        boxes[i].scalar_type() == boxes[0].scalar_type(),
                    "matcher_cost: boxes must be [B,Q,4] with one dtype");
        auto lc = logits[i].contiguous();
        auto bc = boxes[i].contiguous();
        keep.push_back(lc);
        keep.push_back(bc);
        lp.logits[i] = lc.data_ptr();
        lp.boxes[i] = bc.data_ptr();
    }
    auto cost = torch::empty({NL, B, Q, T}, l0.options().dtype(torch::kFloat32));
    auto lab = labels.contiguous();
    check_cuda(launch_matcher_cost(dtype_of(l0), dtype_of(boxes[0]), lp, NL, lab.data_ptr<int64_t>(),
                                   tboxes.data_ptr<float>(), counts.data_ptr<int32_t>(), cost.data_ptr<float>(), B, Q,
                                   C, T, static_cast<float>(w_class), static_cast<float>(w_bbox),
                                   static_cast<float>(w_giou), static_cast<float>(alpha), cur_stream()),
               "matcher_cost");
    return cost;
}

std::vector<torch::Tensor> lsap_batched(torch::Tensor cost, torch::Tensor counts, int64_t groups) {
    TORCH_CHECK(cost.is_cuda() && cost.dim() == 4 && cost.scalar_type() == torch::kFloat32 && cost.is_contiguous(),
                "lsap_batched: cost must be CUDA fp32 [NL,B,Q,T]");
    TORCH_CHECK(counts.scalar_type() == torch::kInt32 && counts.numel() == cost.size(1), "lsap_batched: counts");
    const int NL = static_cast<int>(cost.size(0)), B = static_cast<int>(cost.size(1));
    const int Q = static_cast<int>(cost.size(2)), T = static_cast<int>(cost.size(3));
    const int G = static_cast<int>(groups);
    TORCH_CHECK(G >= 1 && Q % G == 0, "lsap_batched: Q must be divisible by groups");
    const int Qg = Q / G;
    TORCH_CHECK(lsap_shared_bytes(Qg, T, lsap_warps_per_block(Qg, T)) <= 227 * 1024, "lsap_batched: too large");
    at::cuda::CUDAGuard guard(cost.device());
    auto match = torch::full({NL, B, G, T}, -1, cost.options().dtype(torch::kInt32));
    auto status = torch::zeros({1}, cost.options().dtype(torch::kInt32));
    check_cuda(launch_lsap(cost.data_ptr<float>(), counts.data_ptr<int32_t>(), match.data_ptr<int32_t>(), NL, B, G, Qg,
                           T, status.data_ptr<int32_t>(), cur_stream()),
               "lsap_batched");
    return {match, status};
}

// ---------------------------------------------------------------- optimizer
void adamw_ema_step(torch::Tensor chunks, torch::Tensor groups, torch::Tensor scalars, torch::Tensor grad,
                    torch::Tensor master, torch::Tensor m, torch::Tensor v, c10::optional<torch::Tensor> ema,
                    torch::Tensor param, torch::Tensor scratch, torch::Tensor flags) {
    TORCH_CHECK(grad.scalar_type() == torch::kBFloat16 && param.scalar_type() == torch::kBFloat16,
                "adamw_ema_step: grad/param must be bf16");
    TORCH_CHECK(master.scalar_type() == torch::kFloat32 && m.scalar_type() == torch::kFloat32 &&
                    v.scalar_type() == torch::kFloat32,
                "adamw_ema_step: master/m/v must be fp32");
    TORCH_CHECK(master.numel() == grad.numel() && param.numel() == grad.numel() && m.numel() == grad.numel() &&
                    v.numel() == grad.numel(),
                "adamw_ema_step: buffer sizes differ");
    TORCH_CHECK(chunks.scalar_type() == torch::kInt64 && chunks.dim() == 2 && chunks.size(1) == 3 && chunks.is_cuda(),
                "adamw_ema_step: chunks must be CUDA int64 [n,3]");
    TORCH_CHECK(scalars.scalar_type() == torch::kFloat32 && scalars.numel() >= kStepScalarFloats,
                "adamw_ema_step: scalars");
    TORCH_CHECK(groups.scalar_type() == torch::kFloat32 && groups.dim() == 2 && groups.size(1) == 2, "groups [G,2]");
    TORCH_CHECK(scratch.numel() >= optim_num_partials(), "adamw_ema_step: scratch too small");
    TORCH_CHECK(flags.scalar_type() == torch::kInt32 && flags.numel() >= 2, "adamw_ema_step: flags");
    at::cuda::CUDAGuard guard(grad.device());
    auto st = cur_stream();
    const int nparts = optim_num_partials();
    launch_grad_sumsq(reinterpret_cast<const __nv_bfloat16*>(grad.data_ptr()), grad.numel(), scratch.data_ptr<float>(),
                      nparts, st);
    check_cuda(cudaGetLastError(), "grad_sumsq");
    float* ema_ptr = ema.has_value() ? ema->data_ptr<float>() : nullptr;
    launch_adamw_ema(reinterpret_cast<const ChunkDesc*>(chunks.data_ptr<int64_t>()), static_cast<int>(chunks.size(0)),
                     reinterpret_cast<const __nv_bfloat16*>(grad.data_ptr()), master.data_ptr<float>(),
                     m.data_ptr<float>(), v.data_ptr<float>(), ema_ptr,
                     reinterpret_cast<__nv_bfloat16*>(param.data_ptr()),
                     reinterpret_cast<const GroupHyper*>(groups.data_ptr<float>()),
                     reinterpret_cast<const StepScalars*>(scalars.data_ptr<float>()), scratch.data_ptr<float>(), nparts,
                     flags.data_ptr<int>(), st);
    check_cuda(cudaGetLastError(), "adamw_ema");
}

}  // namespace

}  // namespace mmltk

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.doc() = "mmltk_b200 sm_100a CUDA kernels";
    m.def("num_sms", &mmltk::num_sms);
    m.def("layernorm_fwd", &mmltk::layernorm_fwd, py::arg("x"), py::arg("w"), py::arg("b"), py::arg("eps"),
          py::arg("res") = py::none(), py::arg("pos") = py::none(), py::arg("rbias") = py::none(),
          py::arg("rscale") = py::none());
    m.def("layernorm_bwd", &mmltk::layernorm_bwd, py::arg("gy"), py::arg("x"), py::arg("w"), py::arg("mean"),
          py::arg("rstd"), py::arg("gw_acc") = py::none(), py::arg("gb_acc") = py::none(), py::arg("gy2") = py::none(),
          py::arg("gres") = py::none(), py::arg("want_gbias2") = false, py::arg("gbias2_acc") = py::none());
    m.def("layernorm_fwd_map", &mmltk::layernorm_fwd_map, py::arg("x"), py::arg("w"), py::arg("b"), py::arg("eps"),
          py::arg("ymap"), py::arg("out"), py::arg("col"));
    m.def("layernorm_bwd_map", &mmltk::layernorm_bwd_map, py::arg("g"), py::arg("col"), py::arg("gmap"), py::arg("x"),
          py::arg("w"), py::arg("mean"), py::arg("rstd"), py::arg("gw_acc") = py::none(), py::arg("gb_acc") = py::none());
    m.def("layernorm_grouped_fwd", &mmltk::layernorm_grouped_fwd, py::arg("x"), py::arg("w"), py::arg("b"),
          py::arg("eps"));
    m.def("layernorm_grouped_bwd", &mmltk::layernorm_grouped_bwd, py::arg("gy"), py::arg("x"), py::arg("w"),
          py::arg("mean"), py::arg("rstd"), py::arg("gw_acc") = py::none(), py::arg("gb_acc") = py::none());
    m.def("layernorm_act_fwd", &mmltk::layernorm_act_fwd, py::arg("x"), py::arg("w"), py::arg("b"), py::arg("eps"),
          py::arg("act"));
    m.def("layernorm_act_bwd", &mmltk::layernorm_act_bwd, py::arg("gy"), py::arg("x"), py::arg("w"), py::arg("b"),
          py::arg("mean"), py::arg("rstd"), py::arg("act"), py::arg("gw_acc") = py::none(),
          py::arg("gb_acc") = py::none());
    m.def("msda_fwd", &mmltk::msda_fwd);
    m.def("msda_bwd", &mmltk::msda_bwd);
    m.def("matcher_cost", &mmltk::matcher_cost);
    m.def("lsap_batched", &mmltk::lsap_batched);
    m.def("adamw_ema_step", &mmltk::adamw_ema_step);
    m.def("optim_num_partials", &mmltk::optim_num_partials);
    m.def("step_scalar_floats", [] { return mmltk::kStepScalarFloats; });
    mmltk::register_more_ops(m);
}
