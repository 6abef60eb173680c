// Registration hooks of the host-side modules bound into `mmltk_b200._native`.
#pragma once

#include <torch/extension.h>

namespace mmltk {
void register_native_api(pybind11::module& m);
}  // namespace mmltk
