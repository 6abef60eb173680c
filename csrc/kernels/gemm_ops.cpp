// Torch wrapper of the tcgen05 GEMM.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <limits>
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
//   epi 4 / 5 (activation backward: C = acc * GELU'(res) / acc * [res > 0]): res = pre-activation [M, N];
//   epi 8: C = acc * res (res = a stored activation derivative [M, N]).
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
    // MN-major operands are read as 64-wide boxes (a box past the extent is skipped, a partial one
    // zero-filled), so their extents only need the 16-byte row pitch checked above
    TORCH_CHECK(!a_mn || M % 8 == 0, "gemm_tc: MN-major A needs M % 8 == 0");
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
    if (epi == 4 || epi == 5 || epi == 8) {
        TORCH_CHECK(res.has_value() && res->defined(), "gemm_tc: epilogues 4/5/8 need the pre-activation (res)");
        res_c = res->contiguous();
        TORCH_CHECK(res_c.numel() == M * N && res_c.scalar_type() == torch::kBFloat16 && aligned16(res_c),
                    "gemm_tc: pre-activation must be bf16 [M, N]");
        g.res = reinterpret_cast<const __nv_bfloat16*>(res_c.data_ptr());
    }
    TORCH_CHECK((epi >= 0 && epi <= 5) || epi == 8, "gemm_tc: unknown epilogue");
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

// out += opA(a) opB(b): the product added into an existing bf16 [M, N] tensor (weight gradients
// accumulated straight into the flat gradient buffer).  Split-K products sum their fp32 partials
// and the conversion adds the old value; unsplit ones read it in the epilogue (alpha = beta = 1).
void gemm_tc_acc(torch::Tensor a, torch::Tensor b, bool a_mn, bool b_mn, torch::Tensor out) {
    TORCH_CHECK(a.is_cuda() && b.is_cuda() && a.dim() == 2 && b.dim() == 2, "gemm_tc_acc: 2-D CUDA tensors expected");
    TORCH_CHECK(a.scalar_type() == torch::kBFloat16 && b.scalar_type() == torch::kBFloat16 &&
                    out.scalar_type() == torch::kBFloat16,
                "gemm_tc_acc: bf16 only");
    TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1, "gemm_tc_acc: operands must be row-major");
    const int64_t M = a_mn ? a.size(1) : a.size(0);
    const int64_t K = a_mn ? a.size(0) : a.size(1);
    const int64_t N = b_mn ? b.size(1) : b.size(0);
    TORCH_CHECK(K == (b_mn ? b.size(0) : b.size(1)), "gemm_tc_acc: reduction sizes differ");
    TORCH_CHECK(a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0 && aligned16(a) && aligned16(b),
                "gemm_tc_acc: rows must be 16-byte aligned");
    TORCH_CHECK(N % 16 == 0 && (!a_mn || M % 128 == 0) && (!b_mn || N % 128 == 0) && M > 0 && K > 0,
                "gemm_tc_acc: unsupported shape");
    TORCH_CHECK(out.is_cuda() && out.is_contiguous() && out.size(0) == M && out.size(1) == N && aligned16(out),
                "gemm_tc_acc: out must be a contiguous, 16-byte aligned bf16 [M, N] tensor");
    at::cuda::CUDAGuard guard(a.device());
    GemmArgs g{};
    g.A = reinterpret_cast<const __nv_bfloat16*>(a.data_ptr());
    g.B = reinterpret_cast<const __nv_bfloat16*>(b.data_ptr());
    g.C = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
    g.status = status_word(a.device()).data_ptr<int>();
    g.M = static_cast<int>(M);
    g.N = static_cast<int>(N);
    g.K = static_cast<int>(K);
    g.ldc = N;
    torch::Tensor ws;
    const int splits = gemm_tc_splits(g.M, g.N, g.K, b_mn);
    if (splits > 1) {
        ws = torch::empty({M, N}, a.options().dtype(torch::kFloat32));
        g.ws = ws.data_ptr<float>();
        g.splits = splits;
        g.ws_acc = 1;
    } else {
        g.epi = 6;
        g.alpha = 1.f;
        g.beta = 1.f;
        g.res = g.C;
    }
    check_cuda(launch_gemm_tc(g, a_mn, b_mn, a.stride(0), b.stride(0), cur_stream()), "gemm_tc_acc");
}

// 3 x 3 convolution, stride 1, zero padding 1, of a channels-last input x [B, H, W, C] with weights
// w [N, 3, 3, C] (taps row-major, channel fastest) on the tcgen05 GEMM: each tile of `rows` image rows
// is one product of [rows * W pixels, 9 C] x [9 C, N] whose A tiles are read straight from x (one
// 4-D tensor load per tap and 64-channel chunk; the padding is the loads' zero fill).  Returns y
// [B, H, W, N].  Needs C % 64 == 0, N % 16 == 0 and rows * W <= 128 for a row count dividing H.
torch::Tensor conv3x3_tc(torch::Tensor x, torch::Tensor w) {
    TORCH_CHECK(x.is_cuda() && w.is_cuda() && x.dim() == 4 && w.dim() == 4, "conv3x3_tc: 4-D CUDA tensors expected");
    TORCH_CHECK(x.scalar_type() == torch::kBFloat16 && w.scalar_type() == torch::kBFloat16, "conv3x3_tc: bf16 only");
    TORCH_CHECK(x.is_contiguous() && w.is_contiguous() && aligned16(x) && aligned16(w),
                "conv3x3_tc: contiguous, 16-byte aligned tensors expected");
    const int64_t B = x.size(0), H = x.size(1), W = x.size(2), C = x.size(3), N = w.size(0);
    TORCH_CHECK(w.size(1) == 3 && w.size(2) == 3 && w.size(3) == C, "conv3x3_tc: weights must be [N, 3, 3, C]");
    TORCH_CHECK(C % 64 == 0 && N % 16 == 0 && B > 0 && H > 0 && W > 0, "conv3x3_tc: C % 64 and N % 16 required");
    const int rows = conv3x3_tc_rows(static_cast<int>(H), static_cast<int>(W));
    TORCH_CHECK(rows > 0, "conv3x3_tc: no row count r with r * W <= 128 divides H");
    at::cuda::CUDAGuard guard(x.device());
    auto y = torch::empty({B, H, W, N}, x.options());
    GemmArgs g{};
    g.A = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
    g.B = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
    g.C = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
    g.status = status_word(x.device()).data_ptr<int>();
    g.M = static_cast<int>(rows * W);
    g.N = static_cast<int>(N);
    g.K = static_cast<int>(9 * C);
    g.ldc = N;
    g.batch = static_cast<int>(B * (H / rows));
    g.bs_c = static_cast<int64_t>(rows) * W * N;
    g.conv_w = static_cast<int>(W);
    g.conv_rows = rows;
    g.conv_groups = static_cast<int>(H / rows);
    g.conv_c = static_cast<int>(C);
    check_cuda(launch_gemm_tc(g, false, false, 9 * C, 9 * C, cur_stream()), "conv3x3_tc");
    return y;
}

// Batched products through 2-D tensor maps (see GemmArgs): a / b are the whole operand matrices
// (row-major, unit column stride); batch i reads them at tile coordinates shifted by
// i * (a_bk, a_bm) and i * (b_bk, b_bn).  Returns C [batch, M, N] bf16, or for epi 7 the row
// maxima of acc + bias as fp32 [2, batch, M] (one per half of the columns; take the larger).
//   epi 0: acc + bias;  6: alpha * (acc + bias) + beta * res (res [batch, M, N]);  7: row max.
std::vector<torch::Tensor> gemm_tc_batched(torch::Tensor a, torch::Tensor b, c10::optional<torch::Tensor> bias,
                                           bool a_mn, bool b_mn, int64_t batch, int64_t M, int64_t N, int64_t K,
                                           int64_t a_bk, int64_t a_bm, int64_t b_bk, int64_t b_bn, int64_t epi,
                                           double alpha, double beta, c10::optional<torch::Tensor> res) {
    TORCH_CHECK(a.is_cuda() && b.is_cuda() && a.dim() == 2 && b.dim() == 2, "gemm_tc_batched: 2-D CUDA tensors");
    TORCH_CHECK(a.scalar_type() == torch::kBFloat16 && b.scalar_type() == torch::kBFloat16, "gemm_tc_batched: bf16");
    TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0 &&
                    aligned16(a) && aligned16(b),
                "gemm_tc_batched: row-major operands with 16-byte aligned rows");
    TORCH_CHECK(batch >= 1 && M > 0 && N > 0 && K > 0 && N % 16 == 0, "gemm_tc_batched: bad sizes");
    TORCH_CHECK(batch == 1 || K % 64 == 0, "gemm_tc_batched: K must be a multiple of 64 when batch > 1");
    TORCH_CHECK(epi == 0 || epi == 6 || epi == 7, "gemm_tc_batched: epilogue 0, 6 or 7");
    TORCH_CHECK(!a_mn || M % 128 == 0, "gemm_tc_batched: MN-major A needs M % 128 == 0");
    TORCH_CHECK(!b_mn || N % 128 == 0, "gemm_tc_batched: MN-major B needs N % 128 == 0");
    at::cuda::CUDAGuard guard(a.device());
    GemmArgs g{};
    g.A = reinterpret_cast<const __nv_bfloat16*>(a.data_ptr());
    g.B = reinterpret_cast<const __nv_bfloat16*>(b.data_ptr());
    g.a_inner = a.size(1);
    g.a_outer = a.size(0);
    g.b_inner = b.size(1);
    g.b_outer = b.size(0);
    g.M = static_cast<int>(M);
    g.N = static_cast<int>(N);
    g.K = static_cast<int>(K);
    g.ldc = N;
    g.epi = static_cast<int>(epi);
    g.batch = static_cast<int>(batch);
    g.a_bk = static_cast<int>(a_bk);
    g.a_bm = static_cast<int>(a_bm);
    g.b_bk = static_cast<int>(b_bk);
    g.b_bn = static_cast<int>(b_bn);
    g.bs_c = M * N;
    g.alpha = static_cast<float>(alpha);
    g.beta = static_cast<float>(beta);
    g.status = status_word(a.device()).data_ptr<int>();
    torch::Tensor bias_c, res_c, C, rmax;
    if (bias.has_value() && bias->defined()) {
        bias_c = bias->contiguous();
        TORCH_CHECK(bias_c.scalar_type() == torch::kBFloat16 && bias_c.numel() == batch * N,
                    "gemm_tc_batched: bias bf16 [batch, N]");
        if (!aligned16(bias_c)) bias_c = bias_c.clone();
        g.bias = reinterpret_cast<const __nv_bfloat16*>(bias_c.data_ptr());
        g.bs_bias = N;
    }
    if (epi == 6) {
        TORCH_CHECK(res.has_value() && res->defined(), "gemm_tc_batched: epilogue 6 needs res");
        res_c = res->contiguous();
        TORCH_CHECK(res_c.scalar_type() == torch::kBFloat16 && res_c.numel() == batch * M * N && aligned16(res_c),
                    "gemm_tc_batched: res bf16 [batch, M, N]");
        g.res = reinterpret_cast<const __nv_bfloat16*>(res_c.data_ptr());
    }
    if (epi == 7) {
        TORCH_CHECK(N <= 256, "gemm_tc_batched: the row maximum takes N <= 256");
        rmax = torch::full({2, batch, M}, -std::numeric_limits<float>::infinity(),
                           a.options().dtype(torch::kFloat32));
        g.rmax = rmax.data_ptr<float>();
        C = torch::empty({1}, a.options());
    } else {
        C = torch::empty({batch, M, N}, a.options());
    }
    g.C = reinterpret_cast<__nv_bfloat16*>(C.data_ptr());
    check_cuda(launch_gemm_tc(g, a_mn, b_mn, a.stride(0), b.stride(0), cur_stream()), "gemm_tc_batched");
    return {epi == 7 ? rmax : C};
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
    m.def("gemm_tc_acc", &gemm_tc_acc, py::arg("a"), py::arg("b"), py::arg("a_mn"), py::arg("b_mn"),
          py::arg("out"));
    m.def("conv3x3_tc", &conv3x3_tc, py::arg("x"), py::arg("w"));
    m.def("conv3x3_tc_rows", &conv3x3_tc_rows, py::arg("H"), py::arg("W"));
    m.def("gemm_tc_status", &gemm_tc_status);
    m.def("gemm_tc_batched", &gemm_tc_batched, py::arg("a"), py::arg("b"), py::arg("bias"), py::arg("a_mn"),
          py::arg("b_mn"), py::arg("batch"), py::arg("M"), py::arg("N"), py::arg("K"), py::arg("a_bk"), py::arg("a_bm"),
          py::arg("b_bk"), py::arg("b_bn"), py::arg("epi") = 0, py::arg("alpha") = 1.0, py::arg("beta") = 0.0,
          py::arg("res") = py::none());
    m.def("gemm_tc_smem_bytes", &gemm_tc_smem_bytes);
    m.def("gemm_tc_set_variant", &gemm_tc_set_variant, py::arg("variant"));
    m.def("gemm_tc_variant", &gemm_tc_variant);
}

}  // namespace mmltk
