// Torch wrapper of the tcgen05 GEMM.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <mutex>
#include <vector>

#include "gemm_tc.h"
#include "torch_ops.h"

namespace mmltk {

namespace {

// One status word per device, shared by every GEMM launch (checked by gemm_tc_status()).
torch::Tensor& status_word(const torch::Device& dev) {
    static std::mutex mu;
    static std::vector<torch::Tensor> words(64);
    std::lock_guard<std::mutex> lk(mu);
    auto& t = words.at(dev.index());
    if (!t.defined()) t = torch::zeros({1}, torch::TensorOptions().dtype(torch::kInt32).device(dev));
    return t;
}

bool aligned16(const torch::Tensor& t) { return reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0; }

// C = opA(a) opB(b) (+ bias) with an optional fused epilogue.
//   a_mn=false: a is [M, K]; a_mn=true: a is [K, M].   b_mn=false: b is [N, K]; b_mn=true: b is [K, N].
//   epi: 0 none, 1 GELU, 2 ReLU, 3 res + gamma * (acc + bias).  want_aux: also return acc + bias.
//   epi 4 / 5 (activation backward: C = acc * GELU'(res) / acc * [res > 0]): res = pre-activation [M, N].
//   colsum: optional [N] output that receives (or, colsum_acc, accumulates) the column sums of C.
std::vector<torch::Tensor> gemm_tc(torch::Tensor a, torch::Tensor b, c10::optional<torch::Tensor> bias, bool a_mn,
                                   bool b_mn, int64_t epi, bool want_aux, c10::optional<torch::Tensor> res,
                                   c10::optional<torch::Tensor> gamma, c10::optional<torch::Tensor> colsum,
                                   bool colsum_acc) {
    TORCH_CHECK(a.is_cuda() && b.is_cuda() && a.dim() == 2 && b.dim() == 2, "gemm_tc: 2-D CUDA tensors expected");
    TORCH_CHECK(a.scalar_type() == torch::kBFloat16 && b.scalar_type() == torch::kBFloat16, "gemm_tc: bf16 only");
    TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1, "gemm_tc: operands must be row-major");
    const int64_t M = a_mn ? a.size(1) : a.size(0);
    const int64_t K = a_mn ? a.size(0) : a.size(1);
    const int64_t N = b_mn ? b.size(1) : b.size(0);
    const int64_t Kb = b_mn ? b.size(0) : b.size(1);
    TORCH_CHECK(K == Kb, "gemm_tc: reduction sizes differ (", K, " vs ", Kb, ")");
    TORCH_CHECK(a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0 && aligned16(a) && aligned16(b),
                "gemm_tc: rows must be 16-byte aligned");
    TORCH_CHECK(N % 16 == 0, "gemm_tc: N must be a multiple of 16");
    TORCH_CHECK(!a_mn || M % 128 == 0, "gemm_tc: MN-major A needs M % 128 == 0");
    TORCH_CHECK(!b_mn || N % 128 == 0, "gemm_tc: MN-major B needs N % 128 == 0");
    TORCH_CHECK(M > 0 && N > 0 && K > 0, "gemm_tc: empty problem");
    at::cuda::CUDAGuard guard(a.device());
    auto C = torch::empty({M, N}, a.options());
    torch::Tensor aux;
    GemmArgs g{};
    g.A = reinterpret_cast<const __nv_bfloat16*>(a.data_ptr());
    g.B = reinterpret_cast<const __nv_bfloat16*>(b.data_ptr());
    g.C = reinterpret_cast<__nv_bfloat16*>(C.data_ptr());
    if (want_aux) {
        aux = torch::empty({M, N}, a.options());
        g.aux = reinterpret_cast<__nv_bfloat16*>(aux.data_ptr());
    }
    torch::Tensor bias_c, res_c, gamma_c;
    if (bias.has_value() && bias->defined()) {
        bias_c = bias->contiguous();
        if (!aligned16(bias_c)) bias_c = bias_c.clone();  // vector loads in the epilogue
        TORCH_CHECK(bias_c.numel() == N && bias_c.scalar_type() == torch::kBFloat16, "gemm_tc: bias must be bf16 [N]");
        g.bias = reinterpret_cast<const __nv_bfloat16*>(bias_c.data_ptr());
    }
    if (epi == 3) {
        TORCH_CHECK(res.has_value() && gamma.has_value(), "gemm_tc: epilogue 3 needs res and gamma");
        res_c = res->contiguous();
        gamma_c = gamma->contiguous();
        if (!aligned16(gamma_c)) gamma_c = gamma_c.clone();
        TORCH_CHECK(res_c.numel() == M * N && res_c.scalar_type() == torch::kBFloat16 && aligned16(res_c),
                    "gemm_tc: res must be bf16 [M, N]");
        TORCH_CHECK(gamma_c.numel() == N && gamma_c.scalar_type() == torch::kBFloat16, "gemm_tc: gamma bf16 [N]");
        g.res = reinterpret_cast<const __nv_bfloat16*>(res_c.data_ptr());
        g.gamma = reinterpret_cast<const __nv_bfloat16*>(gamma_c.data_ptr());
    }
    if (epi == 4 || epi == 5) {
        TORCH_CHECK(res.has_value() && res->defined(), "gemm_tc: epilogues 4/5 need the pre-activation (res)");
        res_c = res->contiguous();
        TORCH_CHECK(res_c.numel() == M * N && res_c.scalar_type() == torch::kBFloat16 && aligned16(res_c),
                    "gemm_tc: pre-activation must be bf16 [M, N]");
        g.res = reinterpret_cast<const __nv_bfloat16*>(res_c.data_ptr());
    }
    TORCH_CHECK(epi >= 0 && epi <= 5, "gemm_tc: unknown epilogue");
    torch::Tensor colsum_t;
    if (colsum.has_value() && colsum->defined()) {
        colsum_t = *colsum;
        TORCH_CHECK(colsum_t.is_cuda() && colsum_t.is_contiguous() && colsum_t.numel() == N &&
                        (colsum_t.scalar_type() == torch::kBFloat16 || colsum_t.scalar_type() == torch::kFloat32),
                    "gemm_tc: colsum must be a contiguous bf16/fp32 [N] tensor");
        TORCH_CHECK(N <= kReduceAccFloats, "gemm_tc: colsum supports N <= ", kReduceAccFloats);
        const ReduceScratch rs = reduce_scratch();
        TORCH_CHECK(rs.acc != nullptr, "gemm_tc: reduction scratch unavailable");
        g.colacc = rs.acc;   // zero on entry; the finalize below writes the result and clears it
    }
    g.status = status_word(a.device()).data_ptr<int>();
    g.M = static_cast<int>(M);
    g.N = static_cast<int>(N);
    g.K = static_cast<int>(K);
    g.ldc = N;
    g.epi = static_cast<int>(epi);
    torch::Tensor ws;
    if (epi == 0 && !want_aux && g.bias == nullptr && g.colacc == nullptr) {
        const int splits = gemm_tc_splits(g.M, g.N, g.K, b_mn);
        if (splits > 1) {  // few output tiles, long reduction: split K, sum partials in fp32
            ws = torch::empty({M, N}, a.options().dtype(torch::kFloat32));
            g.ws = ws.data_ptr<float>();
            g.splits = splits;
        }
    }
    check_cuda(launch_gemm_tc(g, a_mn, b_mn, a.stride(0), b.stride(0), cur_stream()), "gemm_tc");
    if (g.colacc != nullptr)
        check_cuda(launch_colacc_finalize(g.colacc, dtype_of(colsum_t), colsum_t.data_ptr(), static_cast<int>(N),
                                          colsum_acc, cur_stream()),
                   "gemm_tc colsum");
    if (want_aux) return {C, aux};
    return {C};
}

int64_t gemm_tc_status(int64_t device) {
    auto& t = status_word(torch::Device(torch::kCUDA, static_cast<c10::DeviceIndex>(device)));
    return t.item<int>();
}

}  // namespace

void register_gemm_ops(pybind11::module& m) {
    m.def("gemm_tc", &gemm_tc, py::arg("a"), py::arg("b"), py::arg("bias") = py::none(), py::arg("a_mn") = false,
          py::arg("b_mn") = false, py::arg("epi") = 0, py::arg("want_aux") = false, py::arg("res") = py::none(),
          py::arg("gamma") = py::none(), py::arg("colsum") = py::none(), py::arg("colsum_acc") = false);
    m.def("gemm_tc_status", &gemm_tc_status);
    m.def("gemm_tc_smem_bytes", &gemm_tc_smem_bytes);
    m.def("gemm_tc_set_variant", &gemm_tc_set_variant, py::arg("variant"));
    m.def("gemm_tc_variant", &gemm_tc_variant);
}

}  // namespace mmltk
