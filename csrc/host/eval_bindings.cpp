// Python bindings of the COCO evaluator (coco_eval.h).
#include <torch/extension.h>

#include <memory>

#include "coco_eval.h"
#include "native_api.h"
#include "worker_pool.h"

namespace mmltk {

namespace {

using eval::Evaluator;

// Keeps the reader alive as long as the evaluator that points into its mapping.
struct PyEvaluator {
    std::shared_ptr<data::Reader> reader;
    std::unique_ptr<Evaluator> ev;
};

py::dict metric_dict(const eval::Metric& m) {
    py::dict d;
    d["ap"] = m.ap;
    d["ap50"] = m.ap50;
    d["ap75"] = m.ap75;
    py::list t;
    for (double v : m.per_threshold) t.append(v);
    d["per_threshold"] = t;
    return d;
}

// batch: indices [B]; scores [B,K] f32; labels [B,K] i64; boxes [B,K,4] f32 (xyxy pixels); masks [B,K,H,W] u8 or None
void add_batch(PyEvaluator& e, std::vector<uint32_t> idx, torch::Tensor scores, torch::Tensor labels,
               torch::Tensor boxes, c10::optional<torch::Tensor> masks) {
    auto s = scores.to(torch::kFloat32).contiguous().cpu();
    auto l = labels.to(torch::kInt64).contiguous().cpu();
    auto b = boxes.to(torch::kFloat32).contiguous().cpu();
    TORCH_CHECK(s.dim() == 2 && l.sizes() == s.sizes() && b.dim() == 3 && b.size(0) == s.size(0) &&
                    b.size(1) == s.size(1) && b.size(2) == 4 && int64_t(idx.size()) == s.size(0),
                "add_batch: scores [B,K], labels [B,K], boxes [B,K,4]");
    torch::Tensor m;
    if (masks && masks->defined()) {
        m = masks->to(torch::kUInt8).contiguous().cpu();
        TORCH_CHECK(m.dim() == 4 && m.size(0) == s.size(0) && m.size(1) == s.size(1), "add_batch: masks [B,K,H,W]");
    }
    const int64_t B = s.size(0), K = s.size(1);
    const int64_t plane = m.defined() ? m.size(2) * m.size(3) : 0;
    py::gil_scoped_release nogil;
    WorkerPool::global().parallel_for(B, [&](int64_t i) {
        e.ev->add_image(idx[i], s.data_ptr<float>() + i * K, l.data_ptr<int64_t>() + i * K,
                        b.data_ptr<float>() + i * K * 4, int(K),
                        m.defined() ? m.data_ptr<uint8_t>() + i * K * plane : nullptr);
    });
}

}  // namespace

void register_eval_api(pybind11::module& m) {
    py::class_<PyEvaluator>(m, "CocoEvaluator")
        .def(py::init([](std::shared_ptr<data::Reader> reader, bool masks, int max_dets) {
                 auto e = std::make_unique<PyEvaluator>();
                 e->reader = reader;
                 e->ev = std::make_unique<Evaluator>(*reader, masks, max_dets);
                 return e;
             }),
             py::arg("reader"), py::arg("masks") = false, py::arg("max_dets") = 500)
        .def("add_batch", &add_batch, py::arg("indices"), py::arg("scores"), py::arg("labels"), py::arg("boxes"),
             py::arg("masks") = py::none())
        .def("summarize", [](PyEvaluator& e, bool mask) { return metric_dict(e.ev->summarize(mask)); },
             py::arg("mask") = false)
        .def("num_images", [](PyEvaluator& e) { return e.ev->num_images(); })
        .def("num_matches", [](PyEvaluator& e, bool mask) { return e.ev->num_matches(mask); },
             py::arg("mask") = false)
        .def("export_matches",
             [](PyEvaluator& e, bool mask) {
                 auto v = e.ev->export_matches(mask);
                 auto t = torch::empty({int64_t(v.size() / 5), 5}, torch::kFloat64);
                 std::copy(v.begin(), v.end(), t.data_ptr<double>());
                 return t;
             },
             py::arg("mask") = false)
        .def("import_matches",
             [](PyEvaluator& e, torch::Tensor t, bool mask) {
                 auto c = t.to(torch::kFloat64).contiguous().cpu();
                 TORCH_CHECK(c.dim() == 2 && c.size(1) == 5, "import_matches: [n, 5]");
                 e.ev->import_matches(mask, c.data_ptr<double>(), size_t(c.size(0)));
             },
             py::arg("rows"), py::arg("mask") = false);
}

}  // namespace mmltk
