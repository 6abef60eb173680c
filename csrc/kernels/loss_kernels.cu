// Dense negative term of the sigmoid classification losses:
//   fwd: sum(coef * s^2 * softplus(x)), s = sigmoid(x), over every logit
//   bwd: dx = g * coef * s^2 * (2 (1 - s) softplus(x) + s)
// Forward: grid-stride 8-wide vector loads, fp32 math, per-CTA partials, and a
// last-CTA-done final sum (no atomics on the value, deterministic order).
#include "common.cuh"

namespace mmltk {

namespace {

__device__ __forceinline__ float softplus_f(float x) { return fmaxf(x, 0.f) + log1pf(__expf(-fabsf(x))); }

__device__ __forceinline__ float sig(float x) { return 1.f / (1.f + __expf(-x)); }

template <typename T>
__global__ void __launch_bounds__(256) dense_neg_fwd_kernel(const T* __restrict__ x, int64_t n, float coef,
                                                           float* __restrict__ partials,
                                                           unsigned int* __restrict__ counter,
                                                           float* __restrict__ out) {
    __shared__ float red[8];
    __shared__ bool last;
    float s = 0.f;
    const int64_t n8 = n / 8;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float v[8];
        load8(x + 8 * i, v);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const float p = sig(v[c]);
            s += p * p * softplus_f(v[c]);
        }
    }
    if (blockIdx.x == 0)
        for (int64_t i = n8 * 8 + threadIdx.x; i < n; i += blockDim.x) {
            const float xv = to_f(x[i]);
            const float p = sig(xv);
            s += p * p * softplus_f(xv);
        }
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int w = 0; w < (blockDim.x >> 5); ++w) t += red[w];
        partials[blockIdx.x] = t;
        __threadfence();
        const unsigned int done = atomicAdd(counter, 1u);
        last = (done == gridDim.x - 1);
    }
    __syncthreads();
    if (last && threadIdx.x < 32) {
        __threadfence();
        float t = 0.f;
        for (int i = threadIdx.x; i < static_cast<int>(gridDim.x); i += 32) t += partials[i];
        t = warp_sum(t);
        if (threadIdx.x == 0) {
            out[0] = t * coef;
            *counter = 0u;  // ready for the next launch (also inside graph replays)
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(256) dense_neg_bwd_kernel(const T* __restrict__ x, const float* __restrict__ g,
                                                           int64_t n, float coef, T* __restrict__ dx) {
    const float gc = g[0] * coef;
    const int64_t n8 = n / 8;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float v[8], o[8];
        load8(x + 8 * i, v);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const float p = sig(v[c]);
            o[c] = gc * p * p * (2.f * (1.f - p) * softplus_f(v[c]) + p);
        }
        store8(dx + 8 * i, o);
    }
    if (blockIdx.x == 0)
        for (int64_t i = n8 * 8 + threadIdx.x; i < n; i += blockDim.x) {
            const float xv = to_f(x[i]);
            const float p = sig(xv);
            dx[i] = from_f<T>(gc * p * p * (2.f * (1.f - p) * softplus_f(xv) + p));
        }
}

}  // namespace

int dense_neg_blocks(int64_t n) {
    const int64_t want = (n / 8 + 255) / 256;
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, static_cast<int64_t>(num_sms()) * 4)));
}

cudaError_t launch_dense_neg_fwd(DType t, const void* x, int64_t n, float coef, float* partials,
                                 unsigned int* counter, float* out, cudaStream_t st) {
    const int blocks = dense_neg_blocks(n);
    return MMLTK_DISPATCH_DT(t, [&] {
        dense_neg_fwd_kernel<scalar_t><<<blocks, 256, 0, st>>>(static_cast<const scalar_t*>(x), n, coef, partials,
                                                               counter, out);
        return cudaGetLastError();
    });
}

cudaError_t launch_dense_neg_bwd(DType t, const void* x, const float* g, int64_t n, float coef, void* dx,
                                 cudaStream_t st) {
    const int blocks = dense_neg_blocks(n);
    return MMLTK_DISPATCH_DT(t, [&] {
        dense_neg_bwd_kernel<scalar_t><<<blocks, 256, 0, st>>>(static_cast<const scalar_t*>(x), g, n, coef,
                                                               static_cast<scalar_t*>(dx));
        return cudaGetLastError();
    });
}

}  // namespace mmltk
