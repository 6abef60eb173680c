// Python bindings of the data path: compiler, reader, loader, target packer,
// PNG codec.  Target packing follows the reference's `build_targets`
// (`src/rfdetr/target_builder.cpp:338-615`): xyxy pixel boxes -> normalised
// cxcywh, labels = stored class ids, per-instance areas, masks from runs.
#include <torch/extension.h>

#include <algorithm>
#include <memory>

#include "dataset.h"
#include "image_io.h"
#include "native_api.h"

namespace mmltk {

namespace {

using data::Loader;
using data::Reader;
using data::PackedInstance;

template <typename T>
std::vector<T> to_vec(const torch::Tensor& t) {
    auto c = t.contiguous().cpu();
    return std::vector<T>(c.data_ptr<T>(), c.data_ptr<T>() + c.numel());
}

py::dict compile_py(const std::string& out_path, std::vector<std::string> paths, torch::Tensor counts,
                    torch::Tensor classes, torch::Tensor boxes, torch::Tensor rle_begin, torch::Tensor rle_count,
                    torch::Tensor rle, std::vector<std::string> class_names, int width, int height, int workers) {
    data::CompileInput in;
    in.image_paths = std::move(paths);
    in.counts = to_vec<int32_t>(counts.to(torch::kInt32));
    in.classes = to_vec<uint8_t>(classes.to(torch::kUInt8));
    in.boxes = to_vec<float>(boxes.to(torch::kFloat32));
    in.rle_begin = to_vec<int64_t>(rle_begin.to(torch::kInt64));
    in.rle_count = to_vec<int64_t>(rle_count.to(torch::kInt64));
    auto r = rle.to(torch::kInt64).contiguous();
    in.rle.resize(r.numel());
    for (int64_t i = 0; i < r.numel(); ++i) in.rle[i] = uint32_t(r.data_ptr<int64_t>()[i]);
    in.class_names = std::move(class_names);
    in.width = width;
    in.height = height;
    in.workers = workers;
    data::CompileStats st;
    {
        py::gil_scoped_release nogil;
        st = data::compile_dataset(in, out_path);
    }
    py::dict d;
    d["images"] = st.images;
    d["instances"] = st.instances;
    d["dropped_instances"] = st.dropped_instances;
    d["rle_pairs"] = st.rle_pairs;
    d["bytes"] = st.bytes;
    return d;
}

py::dict header_dict(const Reader& r) {
    const auto& h = r.header();
    py::dict d;
    d["num_images"] = h.num_images;
    d["width"] = h.width;
    d["height"] = h.height;
    d["channels"] = h.channels;
    d["num_classes"] = h.num_classes;
    d["image_stride"] = h.image_stride;
    d["total_size"] = h.total_size;
    d["version"] = h.version;
    d["instances"] = r.total_instances();
    d["rle_pairs"] = r.total_rle_pairs();
    py::list names;
    for (uint32_t c = 0; c < h.num_classes; ++c) names.append(std::string(h.class_names[c].data()));
    d["class_names"] = names;
    return d;
}

// [n, 4] xyxy pixels, [n] class ids, [n] rle pair counts for one image
py::tuple instances_py(const Reader& r, uint32_t i) {
    if (i >= r.num_images()) throw std::out_of_range("image index");
    const auto& e = r.entry(i);
    const auto* p = r.instances(i);
    auto boxes = torch::empty({e.num_instances, 4}, torch::kInt16);
    auto cls = torch::empty({e.num_instances}, torch::kUInt8);
    auto npairs = torch::empty({e.num_instances}, torch::kInt64);
    for (int k = 0; k < e.num_instances; ++k) {
        int16_t* b = boxes.data_ptr<int16_t>() + 4 * k;
        b[0] = p[k].x1;
        b[1] = p[k].y1;
        b[2] = p[k].x2;
        b[3] = p[k].y2;
        cls.data_ptr<uint8_t>()[k] = p[k].class_id;
        npairs.data_ptr<int64_t>()[k] = p[k].rle_pairs;
    }
    return py::make_tuple(boxes, cls, npairs);
}

// Padded targets of a batch: boxes [B,T,4] normalised cxcywh (pad box (0.5,0.5,0.25,0.25)),
// labels [B,T] int64, counts [B] int32, areas [B,T] (mask area or box area, pixels).
py::tuple targets_py(const Reader& r, std::vector<uint32_t> idx, int T) {
    const int B = int(idx.size());
    const float W = float(r.header().width), H = float(r.header().height);
    auto boxes = torch::empty({B, T, 4}, torch::kFloat32);
    auto labels = torch::zeros({B, T}, torch::kInt64);
    auto counts = torch::zeros({B}, torch::kInt32);
    auto areas = torch::zeros({B, T}, torch::kFloat32);
    float* bp = boxes.data_ptr<float>();
    for (int64_t k = 0; k < int64_t(B) * T; ++k) {
        bp[4 * k] = 0.5f;
        bp[4 * k + 1] = 0.5f;
        bp[4 * k + 2] = 0.25f;
        bp[4 * k + 3] = 0.25f;
    }
    for (int b = 0; b < B; ++b) {
        const auto& e = r.entry(idx[b]);
        const auto* p = r.instances(idx[b]);
        const int n = std::min<int>(e.num_instances, T);
        counts.data_ptr<int32_t>()[b] = n;
        for (int k = 0; k < n; ++k) {
            float* o = bp + 4 * (int64_t(b) * T + k);
            o[0] = 0.5f * (p[k].x1 + p[k].x2) / W;
            o[1] = 0.5f * (p[k].y1 + p[k].y2) / H;
            o[2] = (p[k].x2 - p[k].x1) / W;
            o[3] = (p[k].y2 - p[k].y1) / H;
            labels.data_ptr<int64_t>()[int64_t(b) * T + k] = p[k].class_id;
            double area = double(p[k].x2 - p[k].x1) * (p[k].y2 - p[k].y1);
            if (p[k].rle_pairs) {
                area = 0;
                for (int q = 0; q < p[k].rle_pairs; ++q) area += r.rle()[p[k].rle_offset + q].length;
            }
            areas.data_ptr<float>()[int64_t(b) * T + k] = float(area);
        }
    }
    return py::make_tuple(boxes, labels, counts, areas);
}

// One instance's binary mask (runs, or the box when it has none) into m [H, W] (zeroed by the caller).
void fill_mask(const Reader& r, const PackedInstance& p, uint8_t* m) {
    const int W = int(r.header().width), H = int(r.header().height);
    if (!p.rle_pairs) {
        for (int y = std::max<int>(0, p.y1); y < std::min<int>(H, p.y2); ++y)
            std::fill(m + int64_t(y) * W + std::max<int>(0, p.x1), m + int64_t(y) * W + std::min<int>(W, p.x2), 1);
        return;
    }
    for (int q = 0; q < p.rle_pairs; ++q) {
        const auto& rp = r.rle()[p.rle_offset + q];
        const uint64_t s = rp.start, l = rp.length, lim = uint64_t(W) * H;
        std::fill(m + std::min(s, lim), m + std::min(s + l, lim), 1);
    }
}

// Binary masks of the first T instances of each image, concatenated image-major: [sum(counts), H, W] uint8.
torch::Tensor masks_py(const Reader& r, std::vector<uint32_t> idx, int T) {
    const int W = int(r.header().width), H = int(r.header().height);
    int64_t total = 0;
    for (auto i : idx) total += std::min<int>(r.entry(i).num_instances, T);
    auto out = torch::zeros({total, H, W}, torch::kUInt8);
    uint8_t* o = out.data_ptr<uint8_t>();
    int64_t row = 0;
    for (auto i : idx) {
        const auto* p = r.instances(i);
        for (int k = 0; k < std::min<int>(r.entry(i).num_instances, T); ++k, ++row)
            fill_mask(r, p[k], o + row * int64_t(H) * W);
    }
    return out;
}

// Masks of (image, instance) pairs into a caller-owned [>= n, H, W] uint8 host tensor (pinned for upload).
void instance_masks_py(const Reader& r, const std::vector<std::pair<uint32_t, uint32_t>>& pairs, torch::Tensor out) {
    const int W = int(r.header().width), H = int(r.header().height);
    TORCH_CHECK(!out.is_cuda() && out.is_contiguous() && out.scalar_type() == torch::kUInt8 &&
                    out.numel() >= int64_t(pairs.size()) * H * W,
                "instance_masks: contiguous host uint8 [n, H, W] expected");
    uint8_t* o = out.data_ptr<uint8_t>();
    const int64_t plane = int64_t(H) * W;
    std::memset(o, 0, size_t(pairs.size()) * size_t(plane));
    for (size_t n = 0; n < pairs.size(); ++n) {
        const auto [img, k] = pairs[n];
        if (img >= r.num_images() || k >= r.entry(img).num_instances) throw std::out_of_range("instance_masks");
        fill_mask(r, r.instances(img)[k], o + int64_t(n) * plane);
    }
}

torch::Tensor image_py(const Reader& r, uint32_t i) {
    if (i >= r.num_images()) throw std::out_of_range("image index");
    const auto& h = r.header();
    auto out = torch::empty({3, int64_t(h.height), int64_t(h.width)}, torch::kFloat32);
    std::memcpy(out.data_ptr<float>(), r.pixels(i), h.image_stride);
    return out;
}

torch::Tensor decode_png_py(py::bytes data) {
    std::string s = data;
    img::Image im = img::decode_png(reinterpret_cast<const uint8_t*>(s.data()), s.size());
    auto t = torch::empty({im.height, im.width, 3}, torch::kUInt8);
    std::memcpy(t.data_ptr<uint8_t>(), im.rgb.data(), im.rgb.size());
    return t;
}

py::bytes encode_png_py(torch::Tensor hwc) {
    auto t = hwc.to(torch::kUInt8).contiguous().cpu();
    TORCH_CHECK(t.dim() == 3 && (t.size(2) == 3 || t.size(2) == 4), "encode_png: [H, W, 3|4] uint8");
    auto v = img::encode_png(t.data_ptr<uint8_t>(), int(t.size(1)), int(t.size(0)), int(t.size(2)));
    return py::bytes(reinterpret_cast<const char*>(v.data()), v.size());
}

}  // namespace

void register_data_api(pybind11::module& m) {
    m.def("compile_dataset", &compile_py);
    py::class_<Reader, std::shared_ptr<Reader>>(m, "DatasetReader")
        .def(py::init<const std::string&>())
        .def("header", &header_dict)
        .def("__len__", [](const Reader& r) { return r.num_images(); })
        .def("image", &image_py)
        .def("instances", &instances_py)
        .def("targets", &targets_py)
        .def("masks", &masks_py)
        .def("instance_masks", &instance_masks_py)
        .def("instance_counts", [](const Reader& r) {
            auto t = torch::empty({int64_t(r.num_images())}, torch::kInt32);
            for (uint32_t i = 0; i < r.num_images(); ++i) t.data_ptr<int32_t>()[i] = r.entry(i).num_instances;
            return t;
        });
    py::class_<Loader>(m, "DatasetLoader")
        .def(py::init([](const std::string& path, int batch, bool shuffle, uint64_t seed, int rank, int count,
                         bool drop_last, int workers, int format, std::vector<int64_t> slot_ptrs, size_t slot_bytes,
                         std::vector<int> cpus) {
                 Loader::Config c;
                 c.cpus = std::move(cpus);
                 c.path = path;
                 c.batch = batch;
                 c.shuffle = shuffle;
                 c.seed = seed;
                 c.shard_rank = rank;
                 c.shard_count = count;
                 c.drop_last = drop_last;
                 c.workers = workers;
                 c.format = format;
                 std::vector<void*> slots;
                 for (auto p : slot_ptrs) slots.push_back(reinterpret_cast<void*>(p));
                 return std::make_unique<Loader>(c, slots, slot_bytes);
             }),
             py::arg("path"), py::arg("batch"), py::arg("shuffle"), py::arg("seed"), py::arg("rank"), py::arg("count"),
             py::arg("drop_last"), py::arg("workers"), py::arg("format"), py::arg("slot_ptrs"), py::arg("slot_bytes"),
             py::arg("cpus") = std::vector<int>{})
        .def("begin_epoch", &Loader::begin_epoch)
        .def("num_batches", &Loader::num_batches)
        .def("next", [](Loader& l) -> py::object {
            int slot = -1;
            std::vector<uint32_t> idx;
            bool ok;
            {
                py::gil_scoped_release nogil;
                ok = l.next(slot, idx);
            }
            if (!ok) return py::none();
            return py::make_tuple(slot, idx);
        })
        .def("release", &Loader::release)
        .def("targets", [](Loader& l, std::vector<uint32_t> idx, int T) { return targets_py(l.reader(), idx, T); })
        .def("masks", [](Loader& l, std::vector<uint32_t> idx, int T) { return masks_py(l.reader(), idx, T); })
        .def("header", [](Loader& l) { return header_dict(l.reader()); });
    m.def("decode_png", &decode_png_py);
    m.def("encode_png", &encode_png_py);
}

}  // namespace mmltk
