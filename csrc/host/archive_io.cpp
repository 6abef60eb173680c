// libtorch serialize-archive bridge: nested Python dicts <-> the archive files
// written by `torch::serialize::OutputArchive` (a TorchScript-module zip).
//
// The reference's native checkpoints (`src/rfdetr/checkpoint.cpp:26-106`,
// resume state `src/rfdetr/training/train.cpp:1154-1348`) are such archives: a
// flat set of typed keys plus nested sub-archives ("state" -> "entry_000000" ->
// {name, tensor}).  Reading and writing them through the same libtorch classes
// keeps the files interchangeable; the key layout itself lives in Python
// (mmltk_b200/ckpt/native.py).
//
// Value mapping: str <-> string, bool <-> bool, int <-> int, float <-> double,
// torch.Tensor <-> tensor (written as a buffer), dict <-> sub-archive.
#include <torch/extension.h>
#include <torch/serialize.h>

#include <string>

#include "native_api.h"

namespace mmltk {

namespace {

void write_dict(torch::serialize::OutputArchive& ar, const py::dict& d) {
    for (auto item : d) {
        const std::string key = py::str(item.first);
        py::handle v = item.second;
        if (py::isinstance<py::dict>(v)) {
            torch::serialize::OutputArchive sub;
            write_dict(sub, v.cast<py::dict>());
            ar.write(key, sub);
        } else if (THPVariable_Check(v.ptr())) {
            ar.write(key, v.cast<torch::Tensor>().detach().cpu(), /*is_buffer=*/true);
        } else if (py::isinstance<py::bool_>(v)) {
            ar.write(key, c10::IValue(v.cast<bool>()));
        } else if (py::isinstance<py::int_>(v)) {
            ar.write(key, c10::IValue(v.cast<int64_t>()));
        } else if (py::isinstance<py::float_>(v)) {
            ar.write(key, c10::IValue(v.cast<double>()));
        } else if (py::isinstance<py::str>(v)) {
            ar.write(key, c10::IValue(v.cast<std::string>()));
        } else {
            throw std::invalid_argument("archive_save: unsupported value type for key '" + key + "'");
        }
    }
}

py::dict read_dict(torch::serialize::InputArchive& ar) {
    py::dict d;
    for (const auto& key : ar.keys()) {
        c10::IValue v;
        if (!ar.try_read(key, v)) continue;
        if (v.isTensor()) {
            d[py::str(key)] = v.toTensor();
        } else if (v.isBool()) {
            d[py::str(key)] = v.toBool();
        } else if (v.isInt()) {
            d[py::str(key)] = v.toInt();
        } else if (v.isDouble()) {
            d[py::str(key)] = v.toDouble();
        } else if (v.isString()) {
            d[py::str(key)] = v.toStringRef();
        } else if (v.isObject() || v.isModule()) {
            torch::serialize::InputArchive sub;
            ar.read(key, sub);
            d[py::str(key)] = read_dict(sub);
        }
        // other IValue kinds (none written by either side) are skipped
    }
    return d;
}

}  // namespace

void register_archive_api(pybind11::module& m) {
    m.def("archive_save", [](const std::string& path, const py::dict& d) {
        torch::serialize::OutputArchive ar;
        write_dict(ar, d);
        ar.save_to(path);
    });
    m.def("archive_load", [](const std::string& path) {
        torch::serialize::InputArchive ar;
        ar.load_from(path, c10::Device(c10::kCPU));
        return read_dict(ar);
    });
}

}  // namespace mmltk
