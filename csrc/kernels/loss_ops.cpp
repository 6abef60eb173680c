// Torch wrappers of the fused matched-pair loss kernels (csrc/kernels/matched_loss.cu).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "torch_ops.h"

namespace mmltk {

namespace {

struct Shapes {
    int NL, B, Q, C, G, T;
    DType lt, bt;
};

Shapes check(const std::vector<torch::Tensor>& logits, const std::vector<torch::Tensor>& boxes,
             const torch::Tensor& match, const torch::Tensor& tgt, const torch::Tensor& labels) {
    TORCH_CHECK(!logits.empty() && logits.size() == boxes.size() && int(logits.size()) <= kMatchedMaxLayers,
                "matched_loss: one logits and one boxes tensor per layer (at most 16 layers)");
    const auto& l0 = logits[0];
    const auto& b0 = boxes[0];
    for (size_t i = 0; i < logits.size(); ++i) {
        TORCH_CHECK(logits[i].is_cuda() && logits[i].is_contiguous() && logits[i].sizes() == l0.sizes() &&
                        logits[i].scalar_type() == l0.scalar_type() && logits[i].dim() == 3,
                    "matched_loss: logits must be contiguous [B,Q,C] of one dtype");
        TORCH_CHECK(boxes[i].is_contiguous() && boxes[i].sizes() == b0.sizes() &&
                        boxes[i].scalar_type() == b0.scalar_type() && boxes[i].dim() == 3 && boxes[i].size(2) == 4,
                    "matched_loss: boxes must be contiguous [B,Q,4] of one dtype");
    }
    Shapes s{int(logits.size()), int(l0.size(0)), int(l0.size(1)), int(l0.size(2)), int(match.size(2)),
             int(match.size(3)), dtype_of(l0), dtype_of(b0)};
    TORCH_CHECK(match.scalar_type() == torch::kInt32 && match.is_contiguous() && match.dim() == 4 &&
                    match.size(0) == s.NL && match.size(1) == s.B,
                "matched_loss: match [NL,B,G,T] int32");
    TORCH_CHECK(tgt.scalar_type() == torch::kFloat32 && tgt.is_contiguous() && tgt.size(0) == s.B &&
                    tgt.size(1) == s.T && tgt.size(2) == 4,
                "matched_loss: target boxes [B,T,4] fp32");
    TORCH_CHECK(labels.scalar_type() == torch::kInt64 && labels.is_contiguous() && labels.size(0) == s.B &&
                    labels.size(1) == s.T,
                "matched_loss: labels [B,T] int64");
    return s;
}

torch::Tensor matched_loss_fwd(std::vector<torch::Tensor> logits, std::vector<torch::Tensor> boxes,
                               torch::Tensor match, torch::Tensor tgt, torch::Tensor labels, int64_t mode,
                               double alpha) {
    const Shapes s = check(logits, boxes, match, tgt, labels);
    at::cuda::CUDAGuard guard(logits[0].device());
    MatchedLayers L{};
    for (int i = 0; i < s.NL; ++i) {
        L.logits[i] = logits[i].data_ptr();
        L.boxes[i] = boxes[i].data_ptr();
    }
    auto out = torch::zeros({s.NL, 3}, logits[0].options().dtype(torch::kFloat32));
    check_cuda(launch_matched_loss(false, s.lt, s.bt, L, s.NL, s.B, s.Q, s.C, s.G, s.T, match.data_ptr<int32_t>(),
                                   tgt.data_ptr<float>(), labels.data_ptr<int64_t>(), int(mode), float(alpha),
                                   out.data_ptr<float>(), cur_stream()),
               "matched_loss_fwd");
    return out;
}

// glogits: per-layer gradient tensors of the logits (the dense term's), updated in place;
// gboxes: per-layer zeroed box-gradient tensors, written in place.
void matched_loss_bwd(std::vector<torch::Tensor> logits, std::vector<torch::Tensor> boxes, torch::Tensor match,
                      torch::Tensor tgt, torch::Tensor labels, torch::Tensor gout, std::vector<torch::Tensor> glogits,
                      std::vector<torch::Tensor> gboxes, int64_t mode, double alpha) {
    const Shapes s = check(logits, boxes, match, tgt, labels);
    TORCH_CHECK(int(glogits.size()) == s.NL && int(gboxes.size()) == s.NL, "matched_loss_bwd: gradient lists");
    at::cuda::CUDAGuard guard(logits[0].device());
    MatchedLayers L{};
    for (int i = 0; i < s.NL; ++i) {
        TORCH_CHECK(glogits[i].sizes() == logits[i].sizes() && glogits[i].is_contiguous() &&
                        glogits[i].scalar_type() == logits[i].scalar_type(),
                    "matched_loss_bwd: logits gradient layout");
        TORCH_CHECK(gboxes[i].sizes() == boxes[i].sizes() && gboxes[i].is_contiguous() &&
                        gboxes[i].scalar_type() == boxes[i].scalar_type(),
                    "matched_loss_bwd: boxes gradient layout");
        L.logits[i] = logits[i].data_ptr();
        L.boxes[i] = boxes[i].data_ptr();
        L.glogits[i] = glogits[i].data_ptr();
        L.gboxes[i] = gboxes[i].data_ptr();
    }
    auto g = gout.to(torch::kFloat32).contiguous();
    TORCH_CHECK(g.numel() == 3 * s.NL, "matched_loss_bwd: upstream gradient [NL,3]");
    check_cuda(launch_matched_loss(true, s.lt, s.bt, L, s.NL, s.B, s.Q, s.C, s.G, s.T, match.data_ptr<int32_t>(),
                                   tgt.data_ptr<float>(), labels.data_ptr<int64_t>(), int(mode), float(alpha),
                                   g.data_ptr<float>(), cur_stream()),
               "matched_loss_bwd");
}

}  // namespace

void register_loss_ops(pybind11::module& m) {
    m.def("matched_loss_fwd", &matched_loss_fwd);
    m.def("matched_loss_bwd", &matched_loss_bwd);
}

}  // namespace mmltk
