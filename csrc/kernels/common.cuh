// Shared helpers for the mmltk_b200 sm_100a kernels.
#pragma once

// Device-side only: no torch headers here, so nvcc stays fast.  Torch-facing
// wrappers live in the g++-compiled *_ops.cpp files.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <type_traits>

#include "launch_api.h"

namespace mmltk {

// ---------------------------------------------------------------- debug bounds checks
// Built with -DMMLTK_DEBUG_BOUNDS=1 (the `_kernels_dbg` variant, `python -m mmltk_b200.build
// --debug-bounds`), MMLTK_DEBUG_CHECK(cond, code) records `code` in this translation unit's device
// status word when a data-dependent index is out of range; the kernel itself keeps its release
// behaviour (the index is clamped or the element skipped), so a bad input is reported instead of
// trapping or reading out of bounds.  Each kernel file that checks declares
// MMLTK_DEBUG_STATUS_TU(name) once; `debug_status()` (debug_status.cpp) reads and clears every
// registered word.  Release builds compile the checks to nothing.
#if defined(MMLTK_DEBUG_BOUNDS) && MMLTK_DEBUG_BOUNDS
static __device__ unsigned int g_mmltk_debug_status = 0;
__device__ __forceinline__ void debug_flag(unsigned code) { atomicCAS(&g_mmltk_debug_status, 0u, code); }
#define MMLTK_DEBUG_CHECK(cond, code)            \
    do {                                         \
        if (!(cond)) ::mmltk::debug_flag(code);  \
    } while (0)
#define MMLTK_DEBUG_STATUS_TU(name)                                                         \
    namespace {                                                                             \
    unsigned debug_read_##name() {                                                          \
        unsigned v = 0;                                                                     \
        const unsigned zero = 0;                                                            \
        if (cudaMemcpyFromSymbol(&v, g_mmltk_debug_status, sizeof(v)) != cudaSuccess) return 0u; \
        if (v) cudaMemcpyToSymbol(g_mmltk_debug_status, &zero, sizeof(zero));               \
        return v;                                                                           \
    }                                                                                       \
    const bool debug_registered_##name = ::mmltk::register_debug_reader(&debug_read_##name); \
    }
#else
#define MMLTK_DEBUG_CHECK(cond, code) \
    do {                              \
    } while (0)
#define MMLTK_DEBUG_STATUS_TU(name)
#endif

// debug status codes
constexpr unsigned kDbgMatcherLabel = 0x101;      // matcher: target label outside [0, C)
constexpr unsigned kDbgMatcherCount = 0x102;      // matcher: target count above the slot count T
constexpr unsigned kDbgLossLabel = 0x201;         // matched losses: target label outside [0, C)
constexpr unsigned kDbgLossQuery = 0x202;         // matched losses: matched query index outside [0, Q)
constexpr unsigned kDbgMaskIndex = 0x301;         // packed-mask sampling: mask index outside the mask table

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f(__half x) { return __half2float(x); }

template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ float from_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }

// Standard normal CDF Phi(x) and density phi(x), for GELU(erf) forward and backward.
// Phi comes from erf(|x|/sqrt 2) by Abramowitz & Stegun, Handbook of Mathematical
// Functions, formula 7.1.26 (|erf error| <= 1.5e-7): 1 - t(a1 + t(a2 + ...)) exp(-z^2) with
// t = 1/(1 + p z).  exp(-z^2) = exp(-x^2/2) is the exponential phi needs anyway, so one
// exponential and one reciprocal replace the erf evaluation.
struct NormalCdfPdf {
    float cdf, pdf;
};
__device__ __forceinline__ NormalCdfPdf normal_cdf_pdf(float x) {
    const float e = __expf(-0.5f * x * x);
    const float z = fabsf(x) * 0.70710678118654752f;
    const float t = __fdividef(1.f, fmaf(0.3275911f, z, 1.f));   // approximate reciprocal; 1 <= divisor
    const float poly =
        t * fmaf(t, fmaf(t, fmaf(t, fmaf(t, 1.061405429f, -1.453152027f), 1.421413741f), -0.284496736f), 0.254829592f);
    const float half_erf = 0.5f - 0.5f * poly * e;   // erf(z) / 2, z >= 0
    NormalCdfPdf r;
    r.cdf = 0.5f + copysignf(half_erf, x);
    r.pdf = 0.39894228040143268f * e;
    return r;
}
// GELU(x) = x Phi(x);  GELU'(x) = Phi(x) + x phi(x)
__device__ __forceinline__ float gelu_fwd(float x) { return x * normal_cdf_pdf(x).cdf; }
__device__ __forceinline__ float gelu_bwd(float x) {
    const NormalCdfPdf n = normal_cdf_pdf(x);
    return fmaf(x, n.pdf, n.cdf);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// 8 x bf16 <-> 8 x float through one 16-byte vector.  The data moves as raw
// uint4 / uint2 words: assigning __nv_bfloat162 structs member-wise would split
// every 16-byte access into four 4-byte ones.
__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float2 unpack_bf16x2(uint32_t u) {
    return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u));
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* f) {
    const uint4 raw = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 t = unpack_bf16x2(w[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float* f) {
    uint4 raw;
    raw.x = pack_bf16x2(f[0], f[1]);
    raw.y = pack_bf16x2(f[2], f[3]);
    raw.z = pack_bf16x2(f[4], f[5]);
    raw.w = pack_bf16x2(f[6], f[7]);
    *reinterpret_cast<uint4*>(p) = raw;
}

__device__ __forceinline__ void load8(const float* p, float* f) {
    float4 a = reinterpret_cast<const float4*>(p)[0];
    float4 b = reinterpret_cast<const float4*>(p)[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

__device__ __forceinline__ void store8(float* p, const float* f) {
    reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
}

// 4 elements <-> float4
__device__ __forceinline__ float4 load4(const __nv_bfloat16* p) {
    const uint2 raw = *reinterpret_cast<const uint2*>(p);
    const float2 a = unpack_bf16x2(raw.x), b = unpack_bf16x2(raw.y);
    return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ float4 load4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void store4(__nv_bfloat16* p, float4 v) {
    uint2 raw;
    raw.x = pack_bf16x2(v.x, v.y);
    raw.y = pack_bf16x2(v.z, v.w);
    *reinterpret_cast<uint2*>(p) = raw;
}
__device__ __forceinline__ void store4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }

}  // namespace mmltk

// dtype dispatch for the two activation dtypes used by the framework
#define MMLTK_DISPATCH_DT(dt, ...)                   \
    [&]() -> cudaError_t {                           \
        if ((dt) == ::mmltk::DType::kBF16) {         \
            using scalar_t = __nv_bfloat16;          \
            return __VA_ARGS__();                    \
        } else if ((dt) == ::mmltk::DType::kF32) {   \
            using scalar_t = float;                  \
            return __VA_ARGS__();                    \
        }                                            \
        return cudaErrorInvalidValue;                \
    }()
