// Python bindings of the augmentation planner (augment.h).
#include <torch/extension.h>

#include <memory>

#include "augment.h"
#include "native_api.h"

namespace mmltk {

namespace {

using aug::Planner;

aug::Group group_from(const py::dict& d, const char* name) {
    aug::Group g;
    if (!d.contains(name)) return g;
    auto t = d[name].cast<std::tuple<float, float, float>>();
    g.p = std::get<0>(t);
    g.lo = std::get<1>(t);
    g.hi = std::get<2>(t);
    return g;
}

aug::Config config_from(const py::dict& d) {
    aug::Config c;
    c.enabled = d.contains("enabled") ? d["enabled"].cast<bool>() : false;
    c.geometry = group_from(d, "geometry");
    c.resize = group_from(d, "resize");
    c.color = group_from(d, "color");
    c.noise = group_from(d, "noise");
    c.blur = group_from(d, "blur");
    c.occlusion = group_from(d, "occlusion");
    if (d.contains("copy_paste")) c.copy_paste = d["copy_paste"].cast<float>();
    return c;
}

void check_cpu(const torch::Tensor& t, torch::ScalarType st, const char* what) {
    TORCH_CHECK(!t.is_cuda() && t.is_contiguous() && t.scalar_type() == st, what);
}

}  // namespace

void register_aug_api(pybind11::module& m) {
    py::class_<Planner>(m, "AugmentPlanner")
        .def(py::init([](const py::dict& cfg, int capacity, int width, int height, bool masks) {
                 return std::make_unique<Planner>(config_from(cfg), capacity, width, height, masks);
             }),
             py::arg("config"), py::arg("capacity"), py::arg("width"), py::arg("height"), py::arg("masks") = false)
        .def("plan",
             [](Planner& p, std::vector<uint32_t> idx, uint64_t seed, int epoch, int rank, uint64_t seq,
                torch::Tensor rec) {
                 check_cpu(rec, torch::kFloat32, "plan: records must be a contiguous host fp32 tensor");
                 TORCH_CHECK(rec.numel() >= int64_t(idx.size()) * aug::kRecFloats, "plan: records too small");
                 p.plan(idx, seed, epoch, rank, seq, rec.data_ptr<float>());
             })
        // returns the (dataset_index, instance) list whose source masks the caller uploads
        .def("build_targets",
             [](Planner& p, std::shared_ptr<data::Reader> reader, int T, torch::Tensor boxes, torch::Tensor labels,
                torch::Tensor counts, torch::Tensor areas, c10::optional<torch::Tensor> src_rows) {
                 check_cpu(boxes, torch::kFloat32, "build_targets: boxes fp32 host");
                 check_cpu(labels, torch::kInt64, "build_targets: labels int64 host");
                 check_cpu(counts, torch::kInt32, "build_targets: counts int32 host");
                 check_cpu(areas, torch::kFloat32, "build_targets: areas fp32 host");
                 aug::TargetBuffers out{boxes.data_ptr<float>(), labels.data_ptr<int64_t>(),
                                        counts.data_ptr<int32_t>(), areas.data_ptr<float>(), nullptr};
                 if (src_rows && src_rows->defined()) {
                     check_cpu(*src_rows, torch::kInt32, "build_targets: src_rows int32 host");
                     out.src_rows = src_rows->data_ptr<int32_t>();
                 }
                 std::vector<std::pair<uint32_t, uint32_t>> srcs;
                 p.build_targets(*reader, T, out, out.src_rows ? &srcs : nullptr);
                 return srcs;
             },
             py::arg("reader"), py::arg("slots"), py::arg("boxes"), py::arg("labels"), py::arg("counts"),
             py::arg("areas"), py::arg("src_rows") = py::none())
        .def("replacements", &Planner::replacements)
        .def("commit_donors", &Planner::commit_donors)
        .def("dropped", &Planner::dropped)
        .def("remaps", &Planner::remaps);
    m.def("aug_uniform", &aug::uniform);
    m.def("aug_image_key", &aug::image_key);
    m.def("aug_record_floats", [] { return int(aug::kRecFloats); });
}

}  // namespace mmltk
