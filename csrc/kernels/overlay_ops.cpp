// Torch wrappers of the RGBA overlay kernels (csrc/kernels/overlay.cu).  Overlays are CUDA uint8
// [H, W, 4] tensors with packed pixels (rows may be pitched); colours are (r, g, b, a) tuples.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <array>

#include "torch_ops.h"

namespace mmltk {

namespace {

void check_surface(const torch::Tensor& t, int channels, const char* what) {
    TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kUInt8 && t.dim() == 3 && t.size(2) == channels &&
                    t.stride(2) == 1 && t.stride(1) == channels,
                what, ": CUDA uint8 [H, W, ", channels, "] surface with packed pixels (rows may be pitched)");
}

std::array<uint8_t, 4> rgba_of(const std::vector<int64_t>& c) {
    TORCH_CHECK(c.size() == 3 || c.size() == 4, "colour: (r, g, b) or (r, g, b, a)");
    std::array<uint8_t, 4> out{};
    for (int i = 0; i < 4; ++i) {
        const int64_t v = i < static_cast<int>(c.size()) ? c[i] : 255;
        TORCH_CHECK(v >= 0 && v <= 255, "colour components are 0..255");
        out[i] = static_cast<uint8_t>(v);
    }
    return out;
}

#define OV_ARGS(ov) ov.data_ptr<uint8_t>(), ov.stride(0), int(ov.size(1)), int(ov.size(0))

void overlay_detections_(torch::Tensor ov, torch::Tensor boxes, torch::Tensor colors, c10::optional<torch::Tensor> masks,
                         int64_t thickness, int64_t mask_alpha) {
    check_surface(ov, 4, "overlay_detections_");
    const int64_t n = boxes.size(0);
    TORCH_CHECK(boxes.is_cuda() && boxes.scalar_type() == torch::kFloat32 && boxes.is_contiguous() && boxes.dim() == 2 &&
                    boxes.size(1) == 4,
                "overlay_detections_: boxes [n, 4] fp32 xyxy px");
    TORCH_CHECK(colors.is_cuda() && colors.scalar_type() == torch::kUInt8 && colors.is_contiguous() &&
                    colors.numel() == 3 * n,
                "overlay_detections_: colors [n, 3] uint8");
    const uint8_t* mp = nullptr;
    if (masks.has_value()) {
        TORCH_CHECK(masks->is_cuda() && masks->scalar_type() == torch::kUInt8 && masks->is_contiguous() &&
                        masks->numel() == n * ov.size(0) * ov.size(1),
                    "overlay_detections_: masks [n, H, W] uint8");
        mp = masks->data_ptr<uint8_t>();
    }
    at::cuda::CUDAGuard guard(ov.device());
    check_cuda(launch_overlay_detections(OV_ARGS(ov), boxes.data_ptr<float>(), colors.data_ptr<uint8_t>(), mp,
                                         static_cast<int>(n), static_cast<int>(thickness),
                                         static_cast<uint8_t>(mask_alpha), cur_stream()),
               "overlay_detections_");
}

void composite_rgba_(torch::Tensor dst, torch::Tensor src, bool swap_rb) {
    TORCH_CHECK(dst.dim() == 3 && (dst.size(2) == 3 || dst.size(2) == 4), "composite_rgba_: dst [H, W, 3 or 4]");
    check_surface(dst, static_cast<int>(dst.size(2)), "composite_rgba_");
    check_surface(src, 4, "composite_rgba_");
    TORCH_CHECK(src.size(0) == dst.size(0) && src.size(1) == dst.size(1), "composite_rgba_: sizes differ");
    at::cuda::CUDAGuard guard(dst.device());
    check_cuda(launch_composite_rgba(dst.data_ptr<uint8_t>(), dst.stride(0), static_cast<int>(dst.size(2)),
                                     src.data_ptr<uint8_t>(), src.stride(0), int(dst.size(1)), int(dst.size(0)),
                                     swap_rb, cur_stream()),
               "composite_rgba_");
}

torch::Tensor copy_rgb_to_rgba(torch::Tensor src, bool swap_rb, int64_t alpha) {
    check_surface(src, 3, "copy_rgb_to_rgba");
    at::cuda::CUDAGuard guard(src.device());
    auto out = torch::empty({src.size(0), src.size(1), 4}, src.options());
    check_cuda(launch_copy_rgb_to_rgba(src.data_ptr<uint8_t>(), src.stride(0), out.data_ptr<uint8_t>(), out.stride(0),
                                       int(src.size(1)), int(src.size(0)), swap_rb, static_cast<uint8_t>(alpha),
                                       cur_stream()),
               "copy_rgb_to_rgba");
    return out;
}

void manual_mask_(torch::Tensor ov, int64_t x0, int64_t y0, torch::Tensor mask, std::vector<int64_t> color) {
    check_surface(ov, 4, "manual_mask_");
    TORCH_CHECK(mask.is_cuda() && mask.scalar_type() == torch::kUInt8 && mask.is_contiguous() && mask.dim() == 2,
                "manual_mask_: mask [h, w] uint8");
    const auto c = rgba_of(color);
    at::cuda::CUDAGuard guard(ov.device());
    check_cuda(launch_manual_mask(OV_ARGS(ov), int(x0), int(y0), int(mask.size(1)), int(mask.size(0)),
                                  mask.data_ptr<uint8_t>(), c.data(), cur_stream()),
               "manual_mask_");
}

void manual_mask_runs_(torch::Tensor ov, int64_t x0, int64_t y0, int64_t w, int64_t h, torch::Tensor runs,
                       std::vector<int64_t> color) {
    check_surface(ov, 4, "manual_mask_runs_");
    TORCH_CHECK(runs.is_cuda() && runs.scalar_type() == torch::kInt32 && runs.is_contiguous() && runs.dim() == 2 &&
                    runs.size(1) == 2,
                "manual_mask_runs_: runs [n, 2] int32 (start, length)");
    TORCH_CHECK(w > 0 && h > 0, "manual_mask_runs_: region size");
    const auto c = rgba_of(color);
    at::cuda::CUDAGuard guard(ov.device());
    check_cuda(launch_manual_mask_runs(OV_ARGS(ov), int(x0), int(y0), int(w), int(h),
                                       reinterpret_cast<const uint32_t*>(runs.data_ptr<int32_t>()),
                                       static_cast<int>(runs.size(0)), c.data(), cur_stream()),
               "manual_mask_runs_");
}

void box_outline_(torch::Tensor ov, std::vector<int64_t> box, int64_t thickness, std::vector<int64_t> color) {
    check_surface(ov, 4, "box_outline_");
    TORCH_CHECK(box.size() == 4, "box_outline_: box (x1, y1, x2, y2)");
    const auto c = rgba_of(color);
    at::cuda::CUDAGuard guard(ov.device());
    check_cuda(launch_box_outline(OV_ARGS(ov), int(box[0]), int(box[1]), int(box[2]), int(box[3]), int(thickness),
                                  c.data(), cur_stream()),
               "box_outline_");
}

void selection_handles_(torch::Tensor ov, std::vector<int64_t> box, int64_t radius, std::vector<int64_t> color) {
    check_surface(ov, 4, "selection_handles_");
    TORCH_CHECK(box.size() == 4, "selection_handles_: box (x1, y1, x2, y2)");
    const auto c = rgba_of(color);
    at::cuda::CUDAGuard guard(ov.device());
    check_cuda(launch_selection_handles(OV_ARGS(ov), int(box[0]), int(box[1]), int(box[2]), int(box[3]), int(radius),
                                        c.data(), cur_stream()),
               "selection_handles_");
}

void check_points(const torch::Tensor& pts, const char* what) {
    TORCH_CHECK(pts.is_cuda() && pts.scalar_type() == torch::kInt32 && pts.is_contiguous() && pts.dim() == 2 &&
                    pts.size(1) == 2,
                what, ": points [n, 2] int32 (x, y)");
}

void polyline_(torch::Tensor ov, torch::Tensor pts, bool closed, int64_t thickness, std::vector<int64_t> color) {
    check_surface(ov, 4, "polyline_");
    check_points(pts, "polyline_");
    const int n = static_cast<int>(pts.size(0));
    if (n < 2) return;
    const auto c = rgba_of(color);
    at::cuda::CUDAGuard guard(ov.device());
    check_cuda(launch_segments(OV_ARGS(ov), pts.data_ptr<int32_t>(), n, nullptr, closed ? n : n - 1, int(thickness),
                               c.data(), cur_stream()),
               "polyline_");
}

void points_(torch::Tensor ov, torch::Tensor pts, int64_t radius, std::vector<int64_t> color) {
    check_surface(ov, 4, "points_");
    check_points(pts, "points_");
    const auto c = rgba_of(color);
    at::cuda::CUDAGuard guard(ov.device());
    check_cuda(launch_points(OV_ARGS(ov), pts.data_ptr<int32_t>(), int(pts.size(0)), int(radius), c.data(),
                             cur_stream()),
               "points_");
}

void skeleton_(torch::Tensor ov, torch::Tensor pts, torch::Tensor edges, int64_t thickness, int64_t radius,
               std::vector<int64_t> color) {
    check_surface(ov, 4, "skeleton_");
    check_points(pts, "skeleton_");
    TORCH_CHECK(edges.is_cuda() && edges.scalar_type() == torch::kInt32 && edges.is_contiguous() && edges.dim() == 2 &&
                    edges.size(1) == 2,
                "skeleton_: edges [m, 2] int32 point indices");
    const auto c = rgba_of(color);
    at::cuda::CUDAGuard guard(ov.device());
    check_cuda(launch_segments(OV_ARGS(ov), pts.data_ptr<int32_t>(), int(pts.size(0)),
                               reinterpret_cast<const uint32_t*>(edges.data_ptr<int32_t>()), int(edges.size(0)),
                               int(thickness), c.data(), cur_stream()),
               "skeleton_ edges");
    if (radius > 0)
        check_cuda(launch_points(OV_ARGS(ov), pts.data_ptr<int32_t>(), int(pts.size(0)), int(radius), c.data(),
                                 cur_stream()),
                   "skeleton_ joints");
}

torch::Tensor label_colors(torch::Tensor labels) {
    TORCH_CHECK(labels.is_cuda() && labels.scalar_type() == torch::kInt32 && labels.is_contiguous(),
                "label_colors: labels int32");
    at::cuda::CUDAGuard guard(labels.device());
    auto out = torch::empty({labels.numel(), 3}, labels.options().dtype(torch::kUInt8));
    check_cuda(launch_label_colors(labels.data_ptr<int32_t>(), static_cast<int>(labels.numel()),
                                   out.data_ptr<uint8_t>(), cur_stream()),
               "label_colors");
    return out;
}

#undef OV_ARGS

}  // namespace

void register_overlay_ops(pybind11::module& m) {
    m.def("overlay_detections_", &overlay_detections_, py::arg("ov"), py::arg("boxes"), py::arg("colors"),
          py::arg("masks") = py::none(), py::arg("thickness") = 2, py::arg("mask_alpha") = 115);
    m.def("composite_rgba_", &composite_rgba_, py::arg("dst"), py::arg("src"), py::arg("swap_rb") = false);
    m.def("copy_rgb_to_rgba", &copy_rgb_to_rgba, py::arg("src"), py::arg("swap_rb") = false, py::arg("alpha") = 255);
    m.def("manual_mask_", &manual_mask_);
    m.def("manual_mask_runs_", &manual_mask_runs_);
    m.def("box_outline_", &box_outline_);
    m.def("selection_handles_", &selection_handles_);
    m.def("polyline_", &polyline_);
    m.def("points_", &points_);
    m.def("skeleton_", &skeleton_);
    m.def("label_colors", &label_colors);
}

}  // namespace mmltk
