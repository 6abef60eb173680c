// No-allocation variant of the MSDeformAttn backward (see msda_noalloc.h for
// who needs it and the rules of use).  It has no counterpart in the reference
// implementation.  Built into its own library (libmmltk_noalloc.so) so the
// fixed scratch array below is only reserved in processes that load it.
#include <cstdio>
#include <mutex>

#include "launch_api.h"
#include "msda_noalloc.h"

namespace {

constexpr unsigned kValueElems = MMLTK_NOALLOC_MAX_VALUE_ELEMS;
constexpr unsigned kRefElems = MMLTK_NOALLOC_MAX_REF_ELEMS;

// fp32 accumulators of the backward pass: grad_value first, then grad_ref.
static __device__ __align__(256) float g_msda_scratch[kValueElems + kRefElems];

constexpr int kMaxDevices = 64;

// Device address of g_msda_scratch per device.  In host code the symbol
// itself is only a host-side handle; the kernel needs the address that the
// runtime reports for the current device.
float* scratch_address(cudaError_t* err) {
    static std::mutex mu;
    static float* addr[kMaxDevices] = {};
    int dev = 0;
    *err = cudaGetDevice(&dev);
    if (*err != cudaSuccess) return nullptr;
    if (dev < 0 || dev >= kMaxDevices) {
        *err = cudaErrorInvalidDevice;
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(mu);
    if (addr[dev] == nullptr) {
        void* p = nullptr;
        *err = cudaGetSymbolAddress(&p, g_msda_scratch);
        if (*err != cudaSuccess) return nullptr;
        addr[dev] = static_cast<float*>(p);
    }
    return addr[dev];
}

}  // namespace

extern "C" int mmltk_msda_bwd_noalloc(int dtype, const void* grad_out, const void* value, const int* shapes,
                                      const int* starts, const void* ref, const void* offsets, const void* logits,
                                      void* grad_value, void* grad_ref, void* grad_offsets, void* grad_logits, int B,
                                      int S, int Lq, int H, int L, int P, int D, void* stream) {
    if ((dtype != 0 && dtype != 1) || B < 0 || S < 0 || Lq < 0 || H < 1 || L < 1 || L > 8 || P < 1 || L * P > 32 ||
        !(D == 8 || D == 16 || D == 32 || D == 64 || D == 128)) {
        std::fprintf(stderr, "mmltk_msda_bwd_noalloc: unsupported arguments (dtype %d, L %d, P %d, D %d)\n", dtype, L,
                     P, D);
        return MMLTK_NOALLOC_ERR_BAD_ARG;
    }
    const unsigned long long nv = 1ull * B * S * H * D;
    const unsigned long long nr = 1ull * B * Lq * L * 4;
    if (nv > kValueElems || nr > kRefElems) {
        std::fprintf(stderr,
                     "mmltk_msda_bwd_noalloc: problem needs %llu value and %llu reference-box accumulator elements; "
                     "the fixed scratch holds at most %u and %u\n",
                     nv, nr, kValueElems, kRefElems);
        return MMLTK_NOALLOC_ERR_TOO_LARGE;
    }
    cudaError_t err = cudaSuccess;
    float* scratch = scratch_address(&err);
    if (scratch == nullptr) return static_cast<int>(err);
    mmltk::MsdaDims d{B, S, Lq, H, L, P, D};
    // launch_msda_bwd clears both accumulators on the stream before using them
    err = mmltk::launch_msda_bwd(dtype == 1 ? mmltk::DType::kBF16 : mmltk::DType::kF32, grad_out, value, shapes,
                                 starts, ref, offsets, logits, scratch, scratch + kValueElems, grad_value, grad_ref,
                                 grad_offsets, grad_logits, d, static_cast<cudaStream_t>(stream));
    return static_cast<int>(err);
}
