// Benchmark harness for the reference arm of bench.py.
//
// It drives the UNMODIFIED rlewkowicz/mmltk libtorch sources (compiled next to this file by
// baseline/build_reference.py) through their public API, in the order the reference's own training
// loop runs one single-lane step (src/rfdetr/training/train.cpp:2381-2458 and the optimizer step at
// :2295-2344):
//
//   AutocastGuard(bf16) -> NativeRfDetrModel::forward -> detection_loss_dict -> weighted_detection_loss
//   -> backward -> [gradient all-reduce, N > 1] -> GradScaler::check_and_unscale_ (finite check)
//   -> clip_grad_norm_(0.1) -> one pinned metric read-back + event sync -> NativeAdamW::step (fused
//   backend) -> zero_grad -> ModelEma::update.
//
// What is restated here rather than called: the reference's run_training needs its compiled-dataset
// loader, whose sources are not in the reference snapshot, so the harness builds the per-step inputs
// (normalised float32 images, the padding mask, the PreparedTargets views) the way
// src/rfdetr/target_builder.cpp:587-611 lays them out; the parameter-group rule of
// train.cpp:889-938, the DetectionConfig mapping of train.cpp:1350-1378 and the 8-float metric
// handoff of train.cpp:295-372 are file-local there, so they are restated with the same values.
// The gradient all-reduce (train.cpp:1389-1410: allreduce_coalesced over every gradient, then
// x 1/world) is passed in from Python as a callable that issues the same NCCL collective.
#include <torch/extension.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>

#include <cmath>
#include <memory>
#include <optional>
#include <string>
#include <vector>

#include "mmltk/rfdetr/detection_ops.h"
#include "mmltk/rfdetr/model.h"
#include "mmltk/rfdetr/model_config.h"
#include "mmltk/rfdetr/postprocess.h"
#include "mmltk/rfdetr/training_ops.h"
#include "rfdetr/gpu_augment.h"
#include "rfdetr/ms_deform_attn_op.h"
#include "rfdetr/native_optimizer.h"

namespace py = pybind11;
namespace R = mmltk::rfdetr;

namespace {

R::NativeRfDetrConfig config_for(const std::string& preset_name, int resolution, int patch_size, int num_windows,
                                 int pos_size, int dec_layers, int num_classes) {
    const R::ModelPresetConfig* preset = R::find_model_preset(preset_name);
    R::NativeRfDetrConfig c;
    if (preset != nullptr) {
        // the same field mapping as make_config_from_preset (model.cpp:1374-1401)
        c.preset_name = std::string(preset->preset_name);
        c.resolution = preset->resolution;
        c.segmentation = preset->segmentation_head;
        c.num_classes = preset->num_classes;
        c.num_queries = preset->num_queries;
        c.num_select = preset->num_select;
        c.dec_layers = preset->dec_layers;
        c.group_detr = preset->group_detr;
        c.two_stage = preset->two_stage;
        c.hidden_dim = preset->hidden_dim;
        c.patch_size = preset->patch_size;
        c.num_windows = preset->num_windows;
        c.positional_encoding_size = preset->positional_encoding_size;
        c.cls_loss_coef = preset->cls_loss_coef;
        c.bbox_loss_coef = preset->bbox_loss_coef;
        c.giou_loss_coef = preset->giou_loss_coef;
        c.mask_ce_loss_coef = preset->mask_ce_loss_coef;
        c.mask_dice_loss_coef = preset->mask_dice_loss_coef;
    } else {
        // a configuration the reference has no preset for (e.g. RF-DETR-Base 560 at patch 14): every
        // field the model reads is given explicitly, the rest keep NativeRfDetrConfig's defaults
        c.preset_name = preset_name;
        c.num_classes = 91;
        c.num_queries = 300;
        c.num_select = 300;
        c.group_detr = 13;
    }
    if (resolution > 0) c.resolution = resolution;
    if (patch_size > 0) c.patch_size = patch_size;
    if (num_windows > 0) c.num_windows = num_windows;
    if (pos_size > 0) c.positional_encoding_size = pos_size;
    if (dec_layers > 0) c.dec_layers = dec_layers;
    if (num_classes > 0) c.num_classes = num_classes;
    return c;
}

torch::Device device_for(int device_id) {
    return device_id < 0 ? torch::Device(torch::kCPU)
                         : torch::Device(torch::kCUDA, static_cast<c10::DeviceIndex>(device_id));
}

// a device guard that does nothing on the CPU
struct MaybeCudaGuard {
    std::optional<c10::cuda::CUDAGuard> g;
    explicit MaybeCudaGuard(const torch::Device& d) {
        if (d.is_cuda()) g.emplace(d);
    }
};

R::CompilationMode mode_for(const std::string& m) {
    if (m == "none") return R::CompilationMode::kNone;
    if (m == "full") return R::CompilationMode::kFullTrace;
    return R::CompilationMode::kSelective;
}

}  // namespace

// One rank's training state: model, fused NativeAdamW, ModelEma, the metric read-back buffers.
class RefTrainer {
   public:
    RefTrainer(const std::string& preset, int batch, int device_id, const std::string& compile_mode, int resolution,
               int patch_size, int num_windows, int pos_size, int dec_layers, int world_size, double lr,
               double lr_encoder, double weight_decay, double component_decay, double layer_decay,
               double clip_max_norm, double ema_decay, double ema_tau, int num_classes)
        : device_(device_for(device_id)),
          batch_(batch),
          world_(world_size),
          clip_(clip_max_norm) {
        // device_id < 0: the reference's CPU training step (fp32, no autocast)
        MaybeCudaGuard guard(device_);
        config_ = config_for(preset, resolution, patch_size, num_windows, pos_size, dec_layers, num_classes);
        const auto mode = mode_for(compile_mode);
        model_ = std::make_shared<R::NativeRfDetrModel>(config_);
        model_->to(device_);
        model_->optimize_for_inference(batch, true, mode);
        model_->train();

        // DetectionConfig, as train.cpp:1350-1378 maps it
        det_.num_classes = config_.num_classes;
        det_.group_detr = config_.group_detr;
        det_.dec_layers = config_.dec_layers;
        det_.num_select = config_.num_select;
        det_.world_size = std::max(1, world_size);
        det_.sum_group_losses = config_.sum_group_losses;
        det_.use_varifocal_loss = config_.use_varifocal_loss;
        det_.use_position_supervised_loss = config_.use_position_supervised_loss;
        det_.ia_bce_loss = config_.ia_bce_loss;
        det_.aux_loss = config_.aux_loss;
        det_.two_stage = config_.two_stage;
        det_.include_masks = config_.segmentation;
        det_.use_jit_traced_loss_ops = (mode == R::CompilationMode::kSelective);
        det_.mask_point_sample_ratio = config_.mask_point_sample_ratio;
        det_.focal_alpha = config_.focal_alpha;
        det_.cls_loss_coef = config_.cls_loss_coef;
        det_.bbox_loss_coef = config_.bbox_loss_coef;
        det_.giou_loss_coef = config_.giou_loss_coef;
        det_.mask_ce_loss_coef = config_.mask_ce_loss_coef;
        det_.mask_dice_loss_coef = config_.mask_dice_loss_coef;
        det_.set_cost_class = config_.set_cost_class;
        det_.set_cost_bbox = config_.set_cost_bbox;
        det_.set_cost_giou = config_.set_cost_giou;
        R::populate_default_detection_weight_dict(det_);

        // parameter groups keyed by (lr, weight decay), the rule of train.cpp:889-938 and :1000-1043
        std::vector<R::NativeAdamW::NamedParameter> named;
        std::vector<R::NativeAdamW::Group> groups;
        std::vector<std::pair<double, double>> keys;
        for (const auto& item : model_->named_parameters(true)) {
            if (!item.value().requires_grad()) continue;
            const std::string& name = item.key();
            const bool encoder = name.find("backbone.0.encoder") != std::string::npos;
            double p_lr = lr;
            double p_wd = weight_decay;
            if (encoder) {
                int layer_id = 13 + 1;
                if (name.find("embeddings") != std::string::npos) {
                    layer_id = 0;
                } else {
                    const auto pos = name.find(".layer.");
                    if (pos != std::string::npos && name.find(".residual.") == std::string::npos) {
                        size_t p = pos + 7, n = 0;
                        while (p + n < name.size() && std::isdigit(static_cast<unsigned char>(name[p + n]))) ++n;
                        if (n > 0) layer_id = std::stoi(name.substr(p, n)) + 1;
                    }
                }
                p_lr = lr_encoder * std::pow(layer_decay, static_cast<double>(13 + 1 - layer_id)) * component_decay *
                       component_decay;
                const bool no_wd = name.find("gamma") != std::string::npos ||
                                   name.find("bias") != std::string::npos || name.find("norm") != std::string::npos ||
                                   name.find("embeddings") != std::string::npos ||
                                   name.find("rel_pos") != std::string::npos;
                p_wd = no_wd ? 0.0 : weight_decay;
            } else if (name.find("transformer.decoder") != std::string::npos) {
                p_lr = lr * component_decay;
            }
            size_t g = 0;
            for (; g < keys.size(); ++g) {
                if (keys[g].first == p_lr && keys[g].second == p_wd) break;
            }
            if (g == keys.size()) {
                keys.emplace_back(p_lr, p_wd);
                groups.push_back(R::NativeAdamW::Group{R::NativeAdamWGroupConfig{p_lr, p_wd, false}, {}});
                base_lrs_.push_back(p_lr);
            }
            named.push_back(R::NativeAdamW::NamedParameter{name, item.value()});
            groups[g].param_indices.push_back(named.size() - 1);
        }
        std::vector<torch::Tensor> trainable;
        for (const auto& n : named) trainable.push_back(n.tensor);
        const auto backend = R::native_optimizer_supports_fused(trainable) ? R::NativeOptimizerBackend::fused
                             : R::native_optimizer_supports_foreach(trainable)
                                 ? R::NativeOptimizerBackend::foreach
                                 : R::NativeOptimizerBackend::eager;
        optimizer_.emplace(R::NativeAdamW(std::move(groups), std::move(named), backend));
        if (ema_decay > 0.0) ema_.emplace(optimizer_->parameters(), ema_decay, ema_tau);
        scaler_ = std::make_unique<R::GradScaler>(false);

        // the 8-float metric handoff: device accumulators, one pinned copy + event sync per step
        metrics_ = torch::zeros({8}, torch::TensorOptions().dtype(torch::kFloat32).device(device_));
        metrics_.select(0, 6).fill_(1.0f);
        host_metrics_ =
            torch::empty({8}, torch::TensorOptions().dtype(torch::kFloat32).pinned_memory(device_.is_cuda()));
        if (device_.is_cuda()) TORCH_CHECK(cudaEventCreateWithFlags(&copy_done_, cudaEventDisableTiming) == cudaSuccess);
        nested_mask_ = torch::zeros({batch, config_.resolution, config_.resolution},
                                    torch::TensorOptions().dtype(torch::kBool).device(device_));
        sizes_ = torch::tensor({static_cast<int64_t>(config_.resolution), static_cast<int64_t>(config_.resolution)},
                               torch::TensorOptions().dtype(torch::kInt64))
                     .repeat({batch, 1})
                     .to(device_);
        image_ids_ = torch::arange(batch, torch::TensorOptions().dtype(torch::kInt64).device(device_));
        target_indices_ = torch::arange(4096, torch::TensorOptions().dtype(torch::kInt64).device(device_));
    }

    ~RefTrainer() {
        if (copy_done_ != nullptr) cudaEventDestroy(copy_done_);
    }

    const char* backend_name() const { return optimizer_->backend_name(); }
    int64_t num_parameters() const {
        int64_t n = 0;
        for (const auto& p : optimizer_->parameters()) n += p.numel();
        return n;
    }
    int resolution() const { return config_.resolution; }

    // images: [B,3,H,W] float32 normalised, on the device; boxes [T,4] float32 cxcywh normalised and
    // labels [T] int64 on the device (all images' targets concatenated); counts: per-image target count.
    // allreduce: None at world size 1, else a callable(list[Tensor]) that sums the tensors over ranks in
    // place.  Returns the step loss read back to the host (the metric handoff's read-back).
    double step(const torch::Tensor& images, const torch::Tensor& boxes, const torch::Tensor& labels,
                const std::vector<int64_t>& counts, const py::object& allreduce) {
        // libtorch's autograd engine must not run under the GIL; the all-reduce callbacks take it back
        const bool reduce = world_ > 1 && !allreduce.is_none();
        py::gil_scoped_release nogil;
        MaybeCudaGuard guard(device_);
        const int64_t batch = images.size(0);
        R::PreparedTargets prepared = make_targets(boxes, labels, counts, batch);

        metrics_.narrow(0, 3, 3).zero_();
        torch::Tensor loss, class_loss, box_loss;
        {
            R::AutocastGuard autocast(device_.is_cuda(), device_.is_cuda() ? R::resolve_cuda_autocast_dtype() : at::kFloat);
            R::ModelOutputs outputs = model_->forward(R::NestedTensor{images, nested_mask_.narrow(0, 0, batch)});
            R::AllReduceTensorFn reduce_fn;
            if (reduce) {
                reduce_fn = [&allreduce](torch::Tensor& value) {
                    py::gil_scoped_acquire gil;
                    py::list l;
                    l.append(value);
                    allreduce(l);
                };
            }
            R::TensorMap loss_dict =
                R::detection_loss_dict(outputs, prepared, det_, true, reduce, reduce_fn);
            loss = R::weighted_detection_loss(loss_dict, det_, images.device());
            class_loss = loss_dict.count("loss_ce") ? loss_dict.at("loss_ce") : torch::zeros_like(loss);
            box_loss = loss_dict.count("loss_bbox") ? loss_dict.at("loss_bbox") : torch::zeros_like(loss);
        }
        {
            const auto l = loss.detach(), c = class_loss.detach(), b = box_loss.detach();
            metrics_.select(0, 0).add_(l);
            metrics_.select(0, 1).add_(c);
            metrics_.select(0, 2).add_(b);
            metrics_.select(0, 3).add_(l);
            metrics_.select(0, 4).add_(c);
            metrics_.select(0, 5).add_(b);
            metrics_.select(0, 6).mul_(torch::isfinite(l).to(torch::kFloat32));
        }
        scaler_->scale(loss).backward();

        // optimizer step (train.cpp:2295-2344)
        optimizer_->set_lrs(base_lrs_, 1.0);
        auto& params = optimizer_->parameters();
        if (reduce) {
            std::vector<torch::Tensor> gs;
            for (auto& p : params)
                if (p.grad().defined()) gs.push_back(p.grad());
            {
                py::gil_scoped_acquire gil;
                py::list grads;
                for (auto& g : gs) grads.append(g);
                allreduce(grads);
            }
            for (auto& g : gs) g.mul_(1.0 / static_cast<double>(world_));
        }
        const auto found_inf = scaler_->check_and_unscale_(*optimizer_);
        if (clip_ > 0.0) torch::nn::utils::clip_grad_norm_(params, clip_);
        metrics_.select(0, 7).copy_(found_inf);
        if (device_.is_cuda()) {
            host_metrics_.copy_(metrics_, true);
            const auto stream = at::cuda::getCurrentCUDAStream(device_.index());
            TORCH_CHECK(cudaEventRecord(copy_done_, stream.stream()) == cudaSuccess);
            TORCH_CHECK(cudaEventSynchronize(copy_done_) == cudaSuccess);
        } else {
            host_metrics_.copy_(metrics_);
        }
        const float* v = host_metrics_.data_ptr<float>();
        const double step_loss = v[3];
        const bool loss_finite = v[6] != 0.0f;
        const bool grads_finite = v[7] == 0.0f;
        metrics_.select(0, 6).fill_(1.0f);
        metrics_.select(0, 7).zero_();
        TORCH_CHECK(loss_finite && grads_finite, "non-finite RF-DETR loss or gradients in the reference arm");
        scaler_->step(*optimizer_, false);
        scaler_->update(false);
        optimizer_->zero_grad(true);
        if (ema_.has_value()) ema_->update(params, steps_);
        ++steps_;
        return step_loss;
    }

   private:
    R::PreparedTargets make_targets(const torch::Tensor& boxes, const torch::Tensor& labels,
                                    const std::vector<int64_t>& counts, int64_t batch) {
        // the views build_targets hands to the loss (target_builder.cpp:587-611)
        R::PreparedTargets prepared;
        std::vector<int64_t> offsets(static_cast<size_t>(batch), 0);
        int64_t total = 0;
        for (int64_t i = 0; i < batch; ++i) {
            offsets[static_cast<size_t>(i)] = total;
            total += counts[static_cast<size_t>(i)];
        }
        const auto i64 = torch::TensorOptions().dtype(torch::kInt64);
        const auto area = (boxes.select(1, 2) * boxes.select(1, 3)).contiguous();
        const auto iscrowd = torch::zeros({total}, i64.device(device_));
        prepared.orig_sizes = sizes_.narrow(0, 0, batch);
        prepared.nested_mask = nested_mask_.narrow(0, 0, batch);
        prepared.all_boxes = boxes;
        prepared.all_labels = labels;
        prepared.all_area = area;
        prepared.all_iscrowd = iscrowd;
        prepared.target_offsets = torch::tensor(offsets, i64).to(device_, true);
        prepared.target_counts = torch::tensor(counts, i64).to(device_, true);
        prepared.target_indices = target_indices_.narrow(0, 0, total);
        prepared.offsets = offsets;
        prepared.counts = counts;
        for (int64_t i = 0; i < batch; ++i) {
            R::PreparedTarget t;
            const int64_t o = offsets[static_cast<size_t>(i)], n = counts[static_cast<size_t>(i)];
            t.image_id = image_ids_.narrow(0, i, 1);
            t.orig_size = prepared.orig_sizes.select(0, i);
            t.size = prepared.orig_sizes.select(0, i);
            t.boxes = boxes.narrow(0, o, n);
            t.labels = labels.narrow(0, o, n);
            t.area = area.narrow(0, o, n);
            t.iscrowd = iscrowd.narrow(0, o, n);
            prepared.targets.push_back(std::move(t));
        }
        return prepared;
    }

    torch::Device device_;
    int batch_;
    int world_;
    double clip_;
    int64_t steps_ = 0;
    R::NativeRfDetrConfig config_;
    std::shared_ptr<R::NativeRfDetrModel> model_;
    R::DetectionConfig det_;
    std::optional<R::NativeAdamW> optimizer_;
    std::optional<R::ModelEma> ema_;
    std::unique_ptr<R::GradScaler> scaler_;
    std::vector<double> base_lrs_;
    torch::Tensor metrics_, host_metrics_, nested_mask_, sizes_, image_ids_, target_indices_;
    cudaEvent_t copy_done_ = nullptr;
};

// Eval-mode model + fixed-size post-process: the reference's weights-backend prediction lane
// (src/rfdetr/inference/predict.cpp:626-657 with --fp16: AutocastGuard(bf16) around forward, then
// postprocess_output_batch_fixed_size, src/rfdetr/inference/postprocess.cpp:123-156).
class RefPredictor {
   public:
    RefPredictor(const std::string& preset, int batch, int device_id, const std::string& compile_mode, int resolution,
                 int patch_size, int num_windows, int pos_size, int dec_layers, int num_select)
        : device_(torch::kCUDA, static_cast<c10::DeviceIndex>(device_id)), num_select_(num_select) {
        c10::cuda::CUDAGuard guard(device_);
        config_ = config_for(preset, resolution, patch_size, num_windows, pos_size, dec_layers, 0);
        model_ = std::make_shared<R::NativeRfDetrModel>(config_);
        model_->to(device_);
        model_->optimize_for_inference(batch, false, mode_for(compile_mode));
        model_->eval();
        nested_mask_ = torch::zeros({batch, config_.resolution, config_.resolution},
                                    torch::TensorOptions().dtype(torch::kBool).device(device_));
    }

    int resolution() const { return config_.resolution; }

    // images: [B,3,H,W] float32 normalised on the device.  Returns (scores, labels, boxes) on the device.
    std::vector<torch::Tensor> run(const torch::Tensor& images) {
        py::gil_scoped_release nogil;
        c10::cuda::CUDAGuard guard(device_);
        torch::NoGradGuard no_grad;
        R::OutputTensors out;
        {
            R::AutocastGuard autocast(true, R::resolve_cuda_autocast_dtype());
            R::ModelOutputs o = model_->forward(R::NestedTensor{images, nested_mask_.narrow(0, 0, images.size(0))});
            out.pred_logits = o.main.pred_logits;
            out.pred_boxes = o.main.pred_boxes;
        }
        const auto b = R::postprocess_output_batch_fixed_size(out, config_.resolution, config_.resolution, num_select_);
        return {b.scores, b.labels, b.boxes};
    }

   private:
    torch::Device device_;
    int num_select_;
    R::NativeRfDetrConfig config_;
    std::shared_ptr<R::NativeRfDetrModel> model_;
    torch::Tensor nested_mask_;
};

// The reference's loader hands the trainer float32 planar RGB in [0, 1]; GpuBatchPreprocessor
// (src/rfdetr/gpu_augment.cpp:149-211) normalises it on the device into the model input.
class RefPreprocessor {
   public:
    RefPreprocessor(int64_t batch, int height, int width, int device_id)
        : p_(std::make_unique<R::GpuBatchPreprocessor>(batch, height, width, device_id, at::kFloat)) {}

    torch::Tensor run(const torch::Tensor& images01) {
        TORCH_CHECK(images01.is_cuda() && images01.scalar_type() == torch::kFloat32 && images01.is_contiguous(),
                    "RefPreprocessor: float32 contiguous CUDA images in [0, 1]");
        mmltk::Batch b{};
        b.num_images = static_cast<size_t>(images01.size(0));
        b.device_images = images01.data_ptr<float>();
        return p_->run(b);
    }

   private:
    std::unique_ptr<R::GpuBatchPreprocessor> p_;
};

// MSDeformAttn forward + backward through the reference's autograd op (ms_deform_attn_op.cpp:12-82:
// bf16 inputs are upcast to fp32 for the kernels, gradients cast back), im2col_step 64 as the model
// uses it (model.cpp:808-907).  Returns (out, grad_value, grad_loc, grad_attn).
std::vector<torch::Tensor> ref_msda_fwd_bwd(const torch::Tensor& value, const torch::Tensor& shapes,
                                            const torch::Tensor& level_start, const torch::Tensor& loc,
                                            const torch::Tensor& attn, const torch::Tensor& grad_out,
                                            int64_t im2col_step) {
    py::gil_scoped_release nogil;
    auto v = value.detach().requires_grad_(true);
    auto l = loc.detach().requires_grad_(true);
    auto a = attn.detach().requires_grad_(true);
    auto out = R::ms_deform_attn_cuda_autograd(v, shapes, level_start, l, a, im2col_step);
    out.backward(grad_out);
    return {out.detach(), v.grad(), l.grad(), a.grad()};
}

torch::Tensor ref_msda_fwd(const torch::Tensor& value, const torch::Tensor& shapes, const torch::Tensor& level_start,
                           const torch::Tensor& loc, const torch::Tensor& attn, int64_t im2col_step) {
    torch::NoGradGuard no_grad;
    return R::ms_deform_attn_cuda_autograd(value, shapes, level_start, loc, attn, im2col_step);
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.doc() = "rlewkowicz/mmltk reference (unmodified libtorch sources) driven for benchmarking";
    py::class_<RefTrainer>(m, "RefTrainer")
        .def(py::init<const std::string&, int, int, const std::string&, int, int, int, int, int, int, double, double,
                      double, double, double, double, double, double, int>(),
             py::arg("preset"), py::arg("batch"), py::arg("device_id"), py::arg("compile_mode") = "selective",
             py::arg("resolution") = 0, py::arg("patch_size") = 0, py::arg("num_windows") = 0,
             py::arg("pos_size") = 0, py::arg("dec_layers") = 0, py::arg("world_size") = 1, py::arg("lr") = 1e-4,
             py::arg("lr_encoder") = 1.5e-4, py::arg("weight_decay") = 1e-4, py::arg("component_decay") = 0.7,
             py::arg("layer_decay") = 0.8, py::arg("clip_max_norm") = 0.1, py::arg("ema_decay") = 0.993,
             py::arg("ema_tau") = 100.0, py::arg("num_classes") = 0)
        .def("step", &RefTrainer::step, py::arg("images"), py::arg("boxes"), py::arg("labels"), py::arg("counts"),
             py::arg("allreduce") = py::none())
        .def_property_readonly("backend", &RefTrainer::backend_name)
        .def_property_readonly("num_parameters", &RefTrainer::num_parameters)
        .def_property_readonly("resolution", &RefTrainer::resolution);
    py::class_<RefPredictor>(m, "RefPredictor")
        .def(py::init<const std::string&, int, int, const std::string&, int, int, int, int, int, int>(),
             py::arg("preset"), py::arg("batch"), py::arg("device_id"), py::arg("compile_mode") = "selective",
             py::arg("resolution") = 0, py::arg("patch_size") = 0, py::arg("num_windows") = 0,
             py::arg("pos_size") = 0, py::arg("dec_layers") = 0, py::arg("num_select") = 300)
        .def("run", &RefPredictor::run)
        .def_property_readonly("resolution", &RefPredictor::resolution);
    py::class_<RefPreprocessor>(m, "RefPreprocessor")
        .def(py::init<int64_t, int, int, int>(), py::arg("batch"), py::arg("height"), py::arg("width"),
             py::arg("device_id"))
        .def("run", &RefPreprocessor::run);
    m.def("msda_fwd_bwd", &ref_msda_fwd_bwd);
    m.def("msda_fwd", &ref_msda_fwd);
}
