// Torch wrappers of the image-space kernels (csrc/kernels/imaging.cu).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "torch_ops.h"

namespace mmltk {

namespace {

void check_frame(const torch::Tensor& f, const char* what) {
    TORCH_CHECK(f.is_cuda() && f.scalar_type() == torch::kUInt8 && f.dim() == 3 && f.size(2) == 3 &&
                    f.stride(2) == 1 && f.stride(1) == 3,
                what, ": CUDA uint8 [H, W, 3] frame with packed pixels (rows may be pitched)");
}

// frame [H, W, 3] uint8 (BGR if bgr) -> [3, dh, dw] (fp32 [0,1] or normalised bf16)
torch::Tensor letterbox(torch::Tensor frame, int64_t dh, int64_t dw, bool bgr, bool normalize_bf16) {
    check_frame(frame, "letterbox");
    at::cuda::CUDAGuard guard(frame.device());
    auto out = torch::empty({3, dh, dw}, frame.options().dtype(normalize_bf16 ? torch::kBFloat16 : torch::kFloat32));
    check_cuda(launch_letterbox(frame.data_ptr<uint8_t>(), frame.stride(0), int(frame.size(1)), int(frame.size(0)), bgr,
                                out.data_ptr(), int(dw), int(dh), normalize_bf16, cur_stream()),
               "letterbox");
    return out;
}

void vflip_(torch::Tensor frame) {
    check_frame(frame, "vflip_");
    at::cuda::CUDAGuard guard(frame.device());
    check_cuda(launch_vflip(frame.data_ptr<uint8_t>(), frame.stride(0), int(frame.size(1)), int(frame.size(0)),
                            cur_stream()),
               "vflip_");
}

// draws in place; boxes [n,4] xyxy px (fp32), colors [n,3] uint8, masks [n,H,W] uint8, text [n, L] int8
void draw_(torch::Tensor img, torch::Tensor boxes, torch::Tensor colors, c10::optional<torch::Tensor> masks,
           c10::optional<torch::Tensor> text, int64_t thickness, double mask_alpha, int64_t scale) {
    check_frame(img, "draw_");
    at::cuda::CUDAGuard guard(img.device());
    auto b = boxes.to(img.device(), torch::kFloat32).contiguous();
    auto c = colors.to(img.device(), torch::kUInt8).contiguous();
    TORCH_CHECK(b.dim() == 2 && b.size(1) == 4 && c.dim() == 2 && c.size(1) == 3 && c.size(0) == b.size(0),
                "draw_: boxes [n,4], colors [n,3]");
    const int n = int(b.size(0));
    torch::Tensor m, t;
    if (masks && masks->defined()) {
        m = masks->to(img.device(), torch::kUInt8).contiguous();
        TORCH_CHECK(m.dim() == 3 && m.size(0) == n && m.size(1) == img.size(0) && m.size(2) == img.size(1),
                    "draw_: masks [n,H,W] at the image size");
    }
    if (text && text->defined()) {
        t = text->to(img.device(), torch::kInt8).contiguous();
        TORCH_CHECK(t.dim() == 2 && t.size(0) == n, "draw_: text [n, L]");
    }
    check_cuda(launch_draw(img.data_ptr<uint8_t>(), img.stride(0), int(img.size(1)), int(img.size(0)),
                           b.data_ptr<float>(), c.data_ptr<uint8_t>(), m.defined() ? m.data_ptr<uint8_t>() : nullptr,
                           t.defined() ? reinterpret_cast<const char*>(t.data_ptr<int8_t>()) : nullptr,
                           t.defined() ? int(t.size(1)) : 0, n, int(thickness), float(mask_alpha), int(scale),
                           cur_stream()),
               "draw_");
}

void composite_(torch::Tensor dst, torch::Tensor rgba, bool swap_rb) {
    check_frame(dst, "composite_");
    TORCH_CHECK(rgba.is_cuda() && rgba.scalar_type() == torch::kUInt8 && rgba.dim() == 3 && rgba.size(2) == 4 &&
                    rgba.size(0) == dst.size(0) && rgba.size(1) == dst.size(1) && rgba.stride(1) == 4,
                "composite_: rgba [H, W, 4] uint8 at the destination size");
    at::cuda::CUDAGuard guard(dst.device());
    check_cuda(launch_composite(dst.data_ptr<uint8_t>(), dst.stride(0), rgba.data_ptr<uint8_t>(), rgba.stride(0),
                                int(dst.size(1)), int(dst.size(0)), swap_rb, cur_stream()),
               "composite_");
}

torch::Tensor resize_masks(torch::Tensor masks, int64_t h, int64_t w) {
    TORCH_CHECK(masks.is_cuda() && masks.dim() == 3, "resize_masks: CUDA [n, h, w]");
    at::cuda::CUDAGuard guard(masks.device());
    auto m = masks.to(torch::kUInt8).contiguous();
    auto out = torch::empty({m.size(0), h, w}, m.options());
    check_cuda(launch_resize_masks(m.data_ptr<uint8_t>(), int(m.size(0)), int(m.size(1)), int(m.size(2)),
                                   out.data_ptr<uint8_t>(), int(h), int(w), cur_stream()),
               "resize_masks");
    return out;
}

torch::Tensor pack_masks(torch::Tensor masks) {
    TORCH_CHECK(masks.is_cuda() && masks.dim() == 3, "pack_masks: CUDA [n, H, W]");
    at::cuda::CUDAGuard guard(masks.device());
    auto m = masks.to(torch::kUInt8).contiguous();
    const int64_t pixels = m.size(1) * m.size(2);
    auto out = torch::empty({m.size(0), (pixels + 63) / 64}, m.options().dtype(torch::kInt64));
    check_cuda(launch_pack_masks(m.data_ptr<uint8_t>(), int(m.size(0)), pixels,
                                 reinterpret_cast<uint64_t*>(out.data_ptr<int64_t>()), cur_stream()),
               "pack_masks");
    return out;
}

torch::Tensor sample_packed_masks(torch::Tensor bits, int64_t h, int64_t w, torch::Tensor points) {
    TORCH_CHECK(bits.is_cuda() && bits.scalar_type() == torch::kInt64 && bits.dim() == 2, "sample_packed: bits");
    at::cuda::CUDAGuard guard(bits.device());
    auto p = points.to(bits.device(), torch::kFloat32).contiguous();
    TORCH_CHECK(p.dim() == 3 && p.size(0) == bits.size(0) && p.size(2) == 2, "sample_packed: points [n, P, 2]");
    auto out = torch::empty({p.size(0), p.size(1)}, p.options());
    check_cuda(launch_sample_packed(reinterpret_cast<const uint64_t*>(bits.contiguous().data_ptr<int64_t>()),
                                    int(bits.size(0)), int(h), int(w), p.data_ptr<float>(), int(p.size(1)),
                                    out.data_ptr<float>(), cur_stream()),
               "sample_packed_masks");
    return out;
}

// inp [N, C, H, W] (fp32 / bf16), pts [N or 1, P, 2] in [0, 1] (x, y) -> [N, C, P]
torch::Tensor point_sample(torch::Tensor inp, torch::Tensor pts) {
    TORCH_CHECK(inp.is_cuda() && inp.dim() == 4, "point_sample: CUDA [N, C, H, W] input");
    at::cuda::CUDAGuard guard(inp.device());
    auto x = inp.contiguous();
    auto p = pts.to(inp.device(), torch::kFloat32).contiguous();
    const int N = int(x.size(0)), C = int(x.size(1));
    TORCH_CHECK(p.dim() == 3 && p.size(2) == 2 && (p.size(0) == N || p.size(0) == 1), "point_sample: pts [N|1, P, 2]");
    const int P = int(p.size(1));
    auto out = torch::empty({N, C, P}, x.options());
    check_cuda(launch_point_sample_fwd(dtype_of(x), x.data_ptr(), N, C, int(x.size(2)), int(x.size(3)),
                                       p.data_ptr<float>(), P, p.size(0) == 1 && N != 1, out.data_ptr(), cur_stream()),
               "point_sample");
    return out;
}

// gradient w.r.t. the input map (fp32 [N, C, H, W])
torch::Tensor point_sample_bwd(torch::Tensor gout, torch::Tensor pts, int64_t H, int64_t W) {
    TORCH_CHECK(gout.is_cuda() && gout.dim() == 3, "point_sample_bwd: CUDA [N, C, P] gradient");
    at::cuda::CUDAGuard guard(gout.device());
    auto g = gout.contiguous();
    auto p = pts.to(g.device(), torch::kFloat32).contiguous();
    const int N = int(g.size(0)), C = int(g.size(1)), P = int(g.size(2));
    auto gin = torch::zeros({N, C, H, W}, g.options().dtype(torch::kFloat32));
    check_cuda(launch_point_sample_bwd(dtype_of(g), g.data_ptr(), N, C, int(H), int(W), p.data_ptr<float>(), P,
                                       p.size(0) == 1 && N != 1, gin.data_ptr<float>(), cur_stream()),
               "point_sample_bwd");
    return gin;
}

}  // namespace

void register_image_ops(pybind11::module& m) {
    m.def("point_sample", &point_sample, py::arg("inp"), py::arg("pts"));
    m.def("point_sample_bwd", &point_sample_bwd, py::arg("gout"), py::arg("pts"), py::arg("h"), py::arg("w"));
    m.def("letterbox", &letterbox, py::arg("frame"), py::arg("h"), py::arg("w"), py::arg("bgr") = true,
          py::arg("normalize_bf16") = true);
    m.def("vflip_", &vflip_);
    m.def("draw_", &draw_, py::arg("img"), py::arg("boxes"), py::arg("colors"), py::arg("masks") = py::none(),
          py::arg("text") = py::none(), py::arg("thickness") = 2, py::arg("mask_alpha") = 0.45,
          py::arg("scale") = 2);
    m.def("composite_", &composite_, py::arg("dst"), py::arg("rgba"), py::arg("swap_rb") = false);
    m.def("resize_masks", &resize_masks);
    m.def("pack_masks", &pack_masks);
    m.def("sample_packed_masks", &sample_packed_masks);
}

}  // namespace mmltk
