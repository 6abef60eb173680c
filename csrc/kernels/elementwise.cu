// Memory-bound helpers of the dense layers:
//   colsum        out[n] = sum_m x[m, n]                       (bias gradients)
//   scale_bwd     g_pre = gy * gamma ; g_gamma[n] = sum_m gy*pre (LayerScale backward)
//   act_bwd       g_pre = gy * act'(pre)  for GELU(erf) / ReLU
// Column reductions run in two levels with no atomics: a row-chunk per CTA
// writes one fp32 partial row, then a reduce kernel with one warp per 32
// columns sums the partials with 8 loads in flight per lane.
#include "common.cuh"

namespace mmltk {

namespace {

constexpr int kColThreads = 256;

// Block = 256 threads = (256 / (N/8)) row lanes x (N/8) column lanes when N/8 <= 256,
// otherwise the block covers a 2048-column slab.  Each thread owns 8 columns.
template <typename T, int MODE>  // MODE 0: colsum(x) ; 1: colsum(gy*pre) + g_pre = gy*gamma
__global__ void __launch_bounds__(kColThreads) colsum_partial_kernel(const T* __restrict__ x,
                                                                     const T* __restrict__ pre,
                                                                     const T* __restrict__ gamma,
                                                                     T* __restrict__ gout, int64_t M, int N,
                                                                     int rows_per_cta, float* __restrict__ part) {
    const int vec_cols = N / 8;
    const int col_lanes = vec_cols < kColThreads ? vec_cols : kColThreads;
    const int row_lanes = kColThreads / col_lanes;
    const int tid = threadIdx.x;
    const int cl = tid % col_lanes, rl = tid / col_lanes;
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_cta;
    const int64_t r1 = r0 + rows_per_cta < M ? r0 + rows_per_cta : M;
    __shared__ float red[kColThreads * 8];
    const int vc = cl + blockIdx.y * kColThreads;
    // every thread reaches both barriers; idle threads just contribute nothing
    const bool active = tid < col_lanes * row_lanes && vc < vec_cols;
    {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        float gm[8];
        if (MODE == 1 && active) load8(gamma + 8 * vc, gm);
        for (int64_t r = r0 + rl; active && r < r1; r += row_lanes) {
            float a[8];
            load8(x + r * N + 8 * vc, a);
            if (MODE == 1) {
                float p[8], o[8];
                load8(pre + r * N + 8 * vc, p);
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    acc[c] += a[c] * p[c];
                    o[c] = a[c] * gm[c];
                }
                store8(gout + r * N + 8 * vc, o);
            } else {
#pragma unroll
                for (int c = 0; c < 8; ++c) acc[c] += a[c];
            }
        }
        // reduce over the row lanes through shared memory
        if (tid < col_lanes * row_lanes) {
#pragma unroll
            for (int c = 0; c < 8; ++c) red[(rl * col_lanes + cl) * 8 + c] = acc[c];
        }
        __syncthreads();
        if (active && rl == 0) {
            for (int q = 1; q < row_lanes; ++q)
#pragma unroll
                for (int c = 0; c < 8; ++c) acc[c] += red[(q * col_lanes + cl) * 8 + c];
            store8(part + static_cast<int64_t>(blockIdx.x) * N + 8 * vc, acc);
        }
    }
}

template <typename TO>
__global__ void __launch_bounds__(256) reduce_partials_kernel(const float* __restrict__ part, int nparts, int N,
                                                              TO* __restrict__ out) {
    // 8 warps x 32 lanes: lane -> column, warp -> strided subset of partial rows
    __shared__ float red[8][33];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int col = blockIdx.x * 32 + lane;
    float s = 0.f;
    if (col < N) {
        int p = w;
        for (; p + 24 < nparts; p += 32) {
            const float a = part[static_cast<int64_t>(p) * N + col];
            const float b = part[static_cast<int64_t>(p + 8) * N + col];
            const float c = part[static_cast<int64_t>(p + 16) * N + col];
            const float d = part[static_cast<int64_t>(p + 24) * N + col];
            s += (a + b) + (c + d);
        }
        for (; p < nparts; p += 8) s += part[static_cast<int64_t>(p) * N + col];
    }
    red[w][lane] = s;
    __syncthreads();
    if (w == 0 && col < N) {
        float t = 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q) t += red[q][lane];
        out[col] = from_f<TO>(t);
    }
}

__device__ __forceinline__ float gelu_grad(float x) {
    // d/dx [x * Phi(x)] = Phi(x) + x * phi(x)
    const float cdf = 0.5f * (1.f + erff(x * 0.70710678118654752f));
    const float pdf = 0.39894228040143268f * __expf(-0.5f * x * x);
    return cdf + x * pdf;
}

template <typename T>
__global__ void __launch_bounds__(256) act_bwd_kernel(const T* __restrict__ gy, const T* __restrict__ pre,
                                                     T* __restrict__ gx, int64_t n8, int act) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float g[8], p[8], o[8];
        load8(gy + 8 * i, g);
        load8(pre + 8 * i, p);
#pragma unroll
        for (int c = 0; c < 8; ++c) o[c] = act == 1 ? g[c] * gelu_grad(p[c]) : (p[c] > 0.f ? g[c] : 0.f);
        store8(gx + 8 * i, o);
    }
}

}  // namespace

int colsum_parts(int64_t M, int N) {
    const int64_t slabs = (N / 8 + kColThreads - 1) / kColThreads;
    int64_t want = static_cast<int64_t>(num_sms()) * 2 / slabs;
    want = std::max<int64_t>(1, std::min<int64_t>(want, (M + 63) / 64));
    return static_cast<int>(want);
}

cudaError_t launch_colsum(DType t, DType out_t, int mode, const void* x, const void* pre, const void* gamma,
                          void* gout, int64_t M, int N, float* part, void* out, cudaStream_t st) {
    if (N % 8 != 0) return cudaErrorInvalidValue;
    const int parts = colsum_parts(M, N);
    const int rows_per_cta = static_cast<int>((M + parts - 1) / parts);
    dim3 grid(parts, (N / 8 + kColThreads - 1) / kColThreads);
    cudaError_t e = MMLTK_DISPATCH_DT(t, [&] {
        using T = scalar_t;
        if (mode == 0)
            colsum_partial_kernel<T, 0><<<grid, kColThreads, 0, st>>>(static_cast<const T*>(x), nullptr, nullptr,
                                                                      nullptr, M, N, rows_per_cta, part);
        else
            colsum_partial_kernel<T, 1><<<grid, kColThreads, 0, st>>>(
                static_cast<const T*>(x), static_cast<const T*>(pre), static_cast<const T*>(gamma),
                static_cast<T*>(gout), M, N, rows_per_cta, part);
        return cudaGetLastError();
    });
    if (e != cudaSuccess) return e;
    return MMLTK_DISPATCH_DT(out_t, [&] {
        reduce_partials_kernel<scalar_t><<<(N + 31) / 32, 256, 0, st>>>(part, parts, N, static_cast<scalar_t*>(out));
        return cudaGetLastError();
    });
}

cudaError_t launch_reduce_partials(DType out_t, const float* part, int nparts, int N, void* out, cudaStream_t st) {
    return MMLTK_DISPATCH_DT(out_t, [&] {
        reduce_partials_kernel<scalar_t><<<(N + 31) / 32, 256, 0, st>>>(part, nparts, N, static_cast<scalar_t*>(out));
        return cudaGetLastError();
    });
}

cudaError_t launch_act_bwd(DType t, const void* gy, const void* pre, void* gx, int64_t n, int act, cudaStream_t st) {
    if (n % 8 != 0) return cudaErrorInvalidValue;
    const int64_t n8 = n / 8;
    const int blocks = static_cast<int>(std::min<int64_t>((n8 + 255) / 256, static_cast<int64_t>(num_sms()) * 8));
    return MMLTK_DISPATCH_DT(t, [&] {
        using T = scalar_t;
        act_bwd_kernel<T><<<std::max(blocks, 1), 256, 0, st>>>(static_cast<const T*>(gy), static_cast<const T*>(pre),
                                                              static_cast<T*>(gx), n8, act);
        return cudaGetLastError();
    });
}

}  // namespace mmltk
