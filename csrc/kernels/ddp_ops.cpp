// Torch-facing side of the fused data-parallel step: CUDA IPC allocation /
// mapping of the peer-visible buffers and the DdpComm object that launches the
// reduce-scatter, update/all-gather and small all-reduce kernels.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cstring>
#include <string>
#include <vector>

#include "ddp_fused.h"
#include "torch_ops.h"

namespace mmltk {

namespace {

// cudaMalloc'd buffer that other processes can map; returned as a uint8 tensor
// (freed with cudaFree when the tensor dies) plus its 64-byte IPC handle.
std::tuple<torch::Tensor, py::bytes> ipc_alloc(int64_t nbytes, int64_t device) {
    TORCH_CHECK(nbytes > 0, "ipc_alloc: size must be positive");
    c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
    void* p = nullptr;
    check_cuda(cudaMalloc(&p, static_cast<size_t>(nbytes)), "ipc_alloc: cudaMalloc");
    check_cuda(cudaMemset(p, 0, static_cast<size_t>(nbytes)), "ipc_alloc: cudaMemset");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        check_cuda(e, "ipc_alloc: cudaIpcGetMemHandle");
    }
    auto t = torch::from_blob(
        p, {nbytes}, [](void* q) { cudaFree(q); },
        torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, static_cast<c10::DeviceIndex>(device)));
    return {t, py::bytes(reinterpret_cast<const char*>(&h), sizeof(h))};
}

int64_t ipc_open(py::bytes handle, int64_t device) {
    std::string s = handle;
    TORCH_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "ipc_open: bad handle size");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, s.data(), sizeof(h));
    c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
    void* p = nullptr;
    check_cuda(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "ipc_open: cudaIpcOpenMemHandle");
    return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr) { cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)); }

class DdpComm {
   public:
    DdpComm(std::vector<int64_t> grad, std::vector<int64_t> param, std::vector<int64_t> flags,
            std::vector<int64_t> small, int64_t rank, int64_t world, torch::Tensor flags_local,
            torch::Tensor small_local, torch::Tensor ctrl, int64_t spin_limit)
        : flags_local_(flags_local), small_local_(small_local), ctrl_(ctrl) {
        TORCH_CHECK(world >= 1 && world <= kDdpMaxWorld, "DdpComm: world size 1..16");
        TORCH_CHECK(static_cast<int64_t>(grad.size()) == world && static_cast<int64_t>(param.size()) == world &&
                        static_cast<int64_t>(flags.size()) == world && static_cast<int64_t>(small.size()) == world,
                    "DdpComm: one pointer per rank expected");
        TORCH_CHECK(ctrl.scalar_type() == torch::kInt32 && ctrl.numel() >= 5 && ctrl.is_cuda(), "DdpComm: ctrl");
        std::memset(&peers_, 0, sizeof(peers_));
        for (int j = 0; j < world; ++j) {
            peers_.grad[j] = reinterpret_cast<const __nv_bfloat16*>(grad[j]);
            peers_.param[j] = reinterpret_cast<__nv_bfloat16*>(param[j]);
            peers_.flags[j] = reinterpret_cast<uint32_t*>(flags[j]);
            peers_.small[j] = reinterpret_cast<float*>(small[j]);
        }
        peers_.world = static_cast<int>(world);
        peers_.rank = static_cast<int>(rank);
        int32_t* c = ctrl.data_ptr<int32_t>();
        st_.flags_local = reinterpret_cast<uint32_t*>(flags_local.data_ptr());
        st_.small_local = reinterpret_cast<float*>(small_local.data_ptr());
        st_.epoch = reinterpret_cast<uint32_t*>(c + 0);
        st_.small_epoch = reinterpret_cast<uint32_t*>(c + 1);
        st_.ticket = reinterpret_cast<unsigned int*>(c + 2);
        st_.status = c + 3;
        st_.gather_epoch = reinterpret_cast<uint32_t*>(c + 4);
        st_.spin_limit = spin_limit;
    }

    // reduce-scatter of bucket `bucket`: this rank's slice [g_off, g_off + len) of the flat gradient into
    // gshard[l_off, l_off + len), per-CTA sums of squares into partials[p_off, p_off + blocks)
    void rs(int64_t g_off, int64_t len, torch::Tensor gshard, int64_t l_off, torch::Tensor partials, int64_t p_off,
            int64_t bucket, int64_t blocks) {
        TORCH_CHECK(gshard.scalar_type() == torch::kFloat32 && l_off >= 0 && gshard.numel() >= l_off + len,
                    "ddp rs: gshard");
        TORCH_CHECK(partials.scalar_type() == torch::kFloat32 && p_off >= 0 && partials.numel() >= p_off + blocks,
                    "ddp rs: partials");
        check_cuda(launch_ddp_rs(peers_, st_, g_off, len, gshard.data_ptr<float>() + l_off,
                                 partials.data_ptr<float>() + p_off, static_cast<int>(bucket), static_cast<int>(blocks),
                                 cur_stream()),
                   "ddp_rs");
    }

    void grad_allgather(std::vector<int64_t> g_off, std::vector<int64_t> len, std::vector<int64_t> l_off,
                        torch::Tensor gshard) {
        TORCH_CHECK(g_off.size() == len.size() && len.size() == l_off.size(), "grad_allgather: one entry per slice");
        TORCH_CHECK(gshard.scalar_type() == torch::kFloat32 && gshard.is_cuda(), "grad_allgather: fp32 shard");
        check_cuda(launch_ddp_grad_allgather(peers_, st_, g_off.data(), len.data(), l_off.data(),
                                             static_cast<int>(g_off.size()), gshard.data_ptr<float>(), cur_stream()),
                   "ddp_grad_allgather");
    }

    void publish(torch::Tensor partials, int64_t n) {
        TORCH_CHECK(partials.scalar_type() == torch::kFloat32 && partials.numel() >= n, "ddp publish: partials");
        check_cuda(launch_ddp_publish(peers_, st_, partials.data_ptr<float>(), static_cast<int>(n), cur_stream()),
                   "ddp_publish");
    }

    void update(torch::Tensor chunks, torch::Tensor gdelta, torch::Tensor gshard, torch::Tensor master,
                torch::Tensor m, torch::Tensor v, c10::optional<torch::Tensor> ema, torch::Tensor groups,
                torch::Tensor scalars, torch::Tensor flags) {
        TORCH_CHECK(chunks.scalar_type() == torch::kInt64 && chunks.is_cuda() && chunks.dim() == 2, "ddp: chunks");
        TORCH_CHECK(gdelta.scalar_type() == torch::kInt64 && gdelta.is_cuda() && gdelta.numel() == chunks.size(0),
                    "ddp: one flat-offset delta per chunk");
        TORCH_CHECK(scalars.numel() >= kStepScalarFloats, "ddp: scalars");
        check_cuda(launch_ddp_update(peers_, st_, reinterpret_cast<const ChunkDesc*>(chunks.data_ptr<int64_t>()),
                                     gdelta.data_ptr<int64_t>(), static_cast<int>(chunks.size(0)),
                                     gshard.data_ptr<float>(),
                                     master.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
                                     ema.has_value() ? ema->data_ptr<float>() : nullptr,
                                     reinterpret_cast<const GroupHyper*>(groups.data_ptr<float>()),
                                     reinterpret_cast<const StepScalars*>(scalars.data_ptr<float>()),
                                     flags.data_ptr<int>(), cur_stream()),
                   "ddp_update");
    }

    void small_allreduce(torch::Tensor data) {
        TORCH_CHECK(data.is_cuda() && data.scalar_type() == torch::kFloat32 && data.is_contiguous() &&
                        data.numel() <= kSmallMax,
                    "small_allreduce: contiguous CUDA fp32 with at most 16 elements");
        check_cuda(launch_small_allreduce(peers_, st_, data.data_ptr<float>(), static_cast<int>(data.numel()),
                                          cur_stream()),
                   "small_allreduce");
    }

    // Byte all-gather between steps (see launch_gather_bytes): this rank's payload must already be
    // staged at the start of its gradient buffer; len16[j] 16-byte words of rank j land at out + off16[j].
    void gather_bytes(torch::Tensor out, std::vector<int64_t> off16, std::vector<int64_t> len16) {
        TORCH_CHECK(out.is_cuda() && out.is_contiguous(), "gather_bytes: contiguous CUDA output");
        TORCH_CHECK(static_cast<int>(off16.size()) == peers_.world && static_cast<int>(len16.size()) == peers_.world,
                    "gather_bytes: one offset and length per rank");
        int64_t end = 0;
        for (int j = 0; j < peers_.world; ++j) end = std::max(end, (off16[j] + len16[j]) * 16);
        TORCH_CHECK(end <= out.numel() * out.element_size(), "gather_bytes: output too small");
        check_cuda(launch_gather_bytes(peers_, st_, out.data_ptr(), off16.data(), len16.data(), cur_stream()),
                   "gather_bytes");
    }

   private:
    DdpPeers peers_;
    DdpState st_;
    torch::Tensor flags_local_, small_local_, ctrl_;
};

}  // namespace

void register_ddp_ops(pybind11::module& m) {
    m.def("ipc_alloc", &ipc_alloc);
    m.def("ipc_open", &ipc_open);
    m.def("ipc_close", &ipc_close);
    m.def("ddp_rs_blocks", &ddp_rs_blocks, py::arg("overlapped") = false);
    m.def("ddp_max_buckets", [] { return kDdpMaxBuckets; });
    m.def("ddp_flag_words", [] { return kFlagWords; });
    m.def("ddp_small_floats", [] { return 2 * kDdpMaxWorld * kSmallMax; });
    py::class_<DdpComm>(m, "DdpComm")
        .def(py::init<std::vector<int64_t>, std::vector<int64_t>, std::vector<int64_t>, std::vector<int64_t>, int64_t,
                      int64_t, torch::Tensor, torch::Tensor, torch::Tensor, int64_t>())
        .def("rs", &DdpComm::rs)
        .def("publish", &DdpComm::publish)
        .def("grad_allgather", &DdpComm::grad_allgather)
        .def("update", &DdpComm::update)
        .def("small_allreduce", &DdpComm::small_allreduce)
        .def("gather_bytes", &DdpComm::gather_bytes);
}

}  // namespace mmltk
