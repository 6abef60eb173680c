// Torch wrappers of the fused augmentation kernels (csrc/kernels/augment.cu).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "torch_ops.h"

namespace mmltk {

namespace {

// images [B,3,H,W] uint8 or fp32 -> out (preallocated [>=B,3,H,W] bf16 / fp32)
void augment_images(torch::Tensor images, torch::Tensor out, c10::optional<torch::Tensor> records,
                    c10::optional<torch::Tensor> donors, c10::optional<torch::Tensor> donor_masks) {
    TORCH_CHECK(images.is_cuda() && images.dim() == 4 && images.size(1) == 3 && images.is_contiguous(),
                "augment_images: contiguous CUDA [B,3,H,W] images expected");
    TORCH_CHECK(images.scalar_type() == torch::kUInt8 || images.scalar_type() == torch::kFloat32,
                "augment_images: uint8 or float32 images");
    TORCH_CHECK(out.is_cuda() && out.is_contiguous() && out.dim() == 4 && out.size(0) >= images.size(0) &&
                    out.size(2) == images.size(2) && out.size(3) == images.size(3),
                "augment_images: output shape");
    TORCH_CHECK(out.scalar_type() == torch::kBFloat16 || out.scalar_type() == torch::kFloat32,
                "augment_images: bf16 or fp32 output");
    const int B = int(images.size(0)), H = int(images.size(2)), W = int(images.size(3));
    TORCH_CHECK(W % 8 != 0 || (reinterpret_cast<uintptr_t>(images.data_ptr()) % 16 == 0 &&
                               reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0),
                "augment_images: 16-byte aligned buffers expected");
    const float* rec = nullptr;
    if (records && records->defined()) {
        TORCH_CHECK(records->is_cuda() && records->scalar_type() == torch::kFloat32 && records->is_contiguous() &&
                        records->dim() == 2 && records->size(0) >= B && records->size(1) == 64,
                    "augment_images: records [B,64] fp32 on the device");
        rec = records->data_ptr<float>();
    }
    const void* dp = nullptr;
    if (donors && donors->defined()) {
        TORCH_CHECK(donors->scalar_type() == images.scalar_type() && donors->is_contiguous() &&
                        donors->size(2) == H && donors->size(3) == W,
                    "augment_images: donor cache must match the images");
        dp = donors->data_ptr();
    }
    const uint8_t* mp = nullptr;
    if (donor_masks && donor_masks->defined()) {
        TORCH_CHECK(donor_masks->scalar_type() == torch::kUInt8 && donor_masks->is_contiguous(), "donor masks u8");
        mp = donor_masks->data_ptr<uint8_t>();
    }
    at::cuda::CUDAGuard guard(images.device());
    check_cuda(launch_augment(out.scalar_type() == torch::kBFloat16 ? DType::kBF16 : DType::kF32,
                              images.scalar_type() == torch::kUInt8, images.data_ptr(), out.data_ptr(), rec, dp, mp,
                              B, H, W, cur_stream()),
               "augment_images");
}

// src [Ns,H,W] u8, donor_masks [slots,H,W] u8, rows [N,2] int32, records [B,64] -> [N,H,W] u8
torch::Tensor warp_masks(torch::Tensor src, torch::Tensor donor_masks, torch::Tensor rows, torch::Tensor records) {
    TORCH_CHECK(src.is_cuda() && src.scalar_type() == torch::kUInt8 && src.dim() == 3, "warp_masks: src [N,H,W] u8");
    TORCH_CHECK(rows.scalar_type() == torch::kInt32 && rows.dim() == 2 && rows.size(1) == 2, "warp_masks: rows");
    const int H = int(src.size(1)), W = int(src.size(2));
    at::cuda::CUDAGuard guard(src.device());
    auto s = src.contiguous();
    auto d = donor_masks.contiguous();
    auto r = rows.contiguous();
    auto rec = records.contiguous();
    auto out = torch::empty({rows.size(0), H, W}, src.options());
    check_cuda(launch_warp_masks(s.data_ptr<uint8_t>(), d.numel() ? d.data_ptr<uint8_t>() : nullptr,
                                 r.data_ptr<int32_t>(), rec.data_ptr<float>(), out.data_ptr<uint8_t>(),
                                 int(rows.size(0)), H, W, cur_stream()),
               "warp_masks");
    return out;
}

// logits [B,Q,C], boxes [B,Q,4] -> (scores [B,K], labels [B,K] int64, boxes [B,K,4] xyxy px, queries [B,K] int32)
std::vector<torch::Tensor> topk_postprocess(torch::Tensor logits, torch::Tensor boxes, int64_t K,
                                            c10::optional<torch::Tensor> sizes, double fixed_h, double fixed_w) {
    TORCH_CHECK(logits.is_cuda() && logits.dim() == 3 && boxes.dim() == 3 && boxes.size(2) == 4 &&
                    boxes.size(0) == logits.size(0) && boxes.size(1) == logits.size(1),
                "topk_postprocess: logits [B,Q,C], boxes [B,Q,4] on CUDA");
    at::cuda::CUDAGuard guard(logits.device());
    auto l = logits.contiguous();
    auto b = boxes.contiguous();
    TORCH_CHECK(l.scalar_type() == torch::kBFloat16 || l.scalar_type() == torch::kFloat32, "logits bf16/fp32");
    TORCH_CHECK(b.scalar_type() == torch::kBFloat16 || b.scalar_type() == torch::kFloat32, "boxes bf16/fp32");
    const int64_t B = l.size(0), Q = l.size(1), C = l.size(2);
    TORCH_CHECK(K > 0 && K <= 1024 && K <= Q * C, "topk_postprocess: 0 < K <= min(1024, Q*C)");
    const float* sp = nullptr;
    torch::Tensor sz;
    if (sizes && sizes->defined()) {
        sz = sizes->to(l.device(), torch::kFloat32).contiguous();
        TORCH_CHECK(sz.dim() == 2 && sz.size(0) == B && sz.size(1) == 2, "sizes [B,2] (h, w)");
        sp = sz.data_ptr<float>();
    }
    auto fo = l.options().dtype(torch::kFloat32);
    auto scores = torch::empty({B, K}, fo);
    auto labels = torch::empty({B, K}, l.options().dtype(torch::kInt64));
    auto ob = torch::empty({B, K, 4}, fo);
    auto qs = torch::empty({B, K}, l.options().dtype(torch::kInt32));
    check_cuda(launch_topk_postprocess(dtype_of(l), dtype_of(b), l.data_ptr(), b.data_ptr(), sp, int(B), int(Q),
                                       int(C), int(K), float(fixed_h), float(fixed_w), scores.data_ptr<float>(),
                                       labels.data_ptr<int64_t>(), ob.data_ptr<float>(), qs.data_ptr<int32_t>(),
                                       cur_stream()),
               "topk_postprocess");
    return {scores, labels, ob, qs};
}

}  // namespace

void register_aug_ops(pybind11::module& m) {
    m.def("topk_postprocess", &topk_postprocess, py::arg("logits"), py::arg("boxes"), py::arg("k"),
          py::arg("sizes") = py::none(), py::arg("fixed_h") = 1.0, py::arg("fixed_w") = 1.0);
    m.def("augment_images", &augment_images, py::arg("images"), py::arg("out"), py::arg("records") = py::none(),
          py::arg("donors") = py::none(), py::arg("donor_masks") = py::none());
    m.def("warp_masks", &warp_masks);
}

}  // namespace mmltk
