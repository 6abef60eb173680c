// Helpers shared by the torch-facing wrapper files (g++ only).
#pragma once

#include <torch/extension.h>

#include "launch_api.h"

namespace mmltk {

DType dtype_of(const torch::Tensor& t);
void check_cuda(cudaError_t e, const char* what);
cudaStream_t cur_stream();

// Ops defined in other wrapper files (GEMM, attention, DDP, ...) register here.
void register_more_ops(pybind11::module& m);
void register_ddp_ops(pybind11::module& m);
void register_gemm_ops(pybind11::module& m);
void register_aug_ops(pybind11::module& m);
void register_loss_ops(pybind11::module& m);
void register_image_ops(pybind11::module& m);
void register_attn_ops(pybind11::module& m);
void register_overlay_ops(pybind11::module& m);
void register_debug_ops(pybind11::module& m);

}  // namespace mmltk
