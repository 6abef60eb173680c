// Memory-bound helpers of the dense layers, each ONE launch:
//   colsum        out[n] (+)= sum_m x[m, n]                              (bias gradients)
//   scale_bwd     g_pre = gy * gamma ; g_gamma[n] (+)= sum_m gy * pre     (LayerScale backward)
//   act_bwd       g_pre = gy * act'(pre) ; optionally gb[n] (+)= sum_m g_pre   (GELU(erf) / ReLU + bias grad)
//
// Column reductions: the columns are cut into 256-wide slabs (grid.y) and the
// rows into chunks (grid.x).  Each CTA (32 column lanes x 8 row lanes, 8
// columns per thread) reduces its rows in shared memory and adds its partial
// row into a per-device fp32 accumulator with vector atomics (the sum happens
// in L2, spread over all slices); the last CTA of a slab to arrive (counter)
// writes -- or, for gradient accumulation, adds into -- the output and clears
// the accumulator and counter for the next launch.  No second reduction
// launch, and a parameter's gradient accumulates in place in the flat
// gradient buffer (no AccumulateGrad add).  Float atomics make the summation
// order, and so the last bits of the result, run dependent.
#include <mutex>

#include "common.cuh"

namespace mmltk {

namespace {

constexpr int kColThreads = 256;
constexpr int kSlabCols = 256;     // columns per slab = 32 lanes x 8
constexpr int kColCtasPerSm = 4;   // resident CTAs per SM (64 registers per thread)
// rows per row lane with loads in flight together (two with the GELU derivative or a second sum, to
// fit 64 registers)
__host__ __device__ constexpr int col_unroll(int mode) { return mode >= 2 ? 2 : 4; }

__device__ __forceinline__ float gelu_grad(float x) { return gelu_bwd(x); }

__device__ __forceinline__ void ldcg8(const float* p, float* f) {
    const float4 a = __ldcg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldcg(reinterpret_cast<const float4*>(p + 4));
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

template <typename TO>
__device__ __forceinline__ void write_out8(TO* out, const float* s, int n_valid, bool accumulate) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        if (c < n_valid) {
            const float base = accumulate ? to_f(out[c]) : 0.f;
            out[c] = from_f<TO>(base + s[c]);
        }
    }
}

// 8 elements as loaded (not yet widened): loads of several rows can be in flight while only
// their raw registers are live
template <typename T>
struct Raw8;
template <>
struct Raw8<__nv_bfloat16> {
    uint4 v;
    __device__ __forceinline__ void load(const __nv_bfloat16* p) { v = *reinterpret_cast<const uint4*>(p); }
    __device__ __forceinline__ void widen(float* f) const {
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 t = unpack_bf16x2(w[i]);
            f[2 * i] = t.x;
            f[2 * i + 1] = t.y;
        }
    }
};
template <>
struct Raw8<float> {
    float4 a, b;
    __device__ __forceinline__ void load(const float* p) {
        a = reinterpret_cast<const float4*>(p)[0];
        b = reinterpret_cast<const float4*>(p)[1];
    }
    __device__ __forceinline__ void widen(float* f) const {
        f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
        f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    }
};

template <typename T, int MODE>
__device__ __forceinline__ void colreduce_row(const T* __restrict__ x, const T* __restrict__ pre,
                                              T* __restrict__ gout, const float* a, const float* p,
                                              const float* gm, float* acc, float* acc2, int act, int64_t off) {
    if constexpr (MODE == 0) {
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[c] += a[c];
    } else {
        float o[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            if (MODE == 1 || MODE == 3) {
                acc[c] += a[c] * p[c];
                o[c] = a[c] * gm[c];
            } else {
                // act 1: GELU' from the pre-activation; 3: p is the stored GELU'; 2: ReLU (p's sign)
                o[c] = act == 3 ? a[c] * p[c] : act == 1 ? a[c] * gelu_grad(p[c]) : (p[c] > 0.f ? a[c] : 0.f);
            }
        }
        if (MODE == 3) {
            // second column sum: the bias gradient of the scaled product, as stored
#pragma unroll
            for (int c = 0; c < 8; ++c) acc2[c] += to_f(from_f<T>(o[c]));
        }
        if (MODE == 2) {
            // the bias gradient sums g_pre as stored (rounded to T), i.e. what the GEMMs consume
#pragma unroll
            for (int c = 0; c < 8; ++c) acc[c] += to_f(from_f<T>(o[c]));
        }
        store8(gout + off, o);
    }
}

// MODE 0: colsum(x) ; 1: gout = x * gamma, colsum(x * pre) ; 2: gout = x * act'(pre), colsum(gout) ;
// 3: MODE 1 plus a second column sum colsum(gout) into out2 (LayerScale and bias gradients in one pass)
// Each row lane keeps col_unroll(MODE) rows' loads in flight (issued before any is consumed) and
// four CTAs share an SM: a memory-bound pass needs tens of KB in flight per SM to cover DRAM
// latency, which one 16-byte load per thread per iteration does not give.
template <typename T, int MODE, typename TO>
__global__ void __launch_bounds__(kColThreads, kColCtasPerSm) colreduce_kernel(const T* __restrict__ x, const T* __restrict__ pre,
                                                                   const T* __restrict__ gamma, T* __restrict__ gout,
                                                                   int64_t M, int N, int rows_per_cta, int act,
                                                                   float* acc_buf, unsigned* counters,
                                                                   TO* __restrict__ out, int accumulate,
                                                                   TO* __restrict__ out2, int accumulate2) {
    // groups (gridDim.z > 1): group g = blockIdx.z reduces its own M rows (x, pre and gout advanced by
    // g * M rows) into its own accumulators, arrival counters and output row g (out / out2 [G, N])
    if (gridDim.z > 1) {
        const int64_t g = blockIdx.z;
        x += g * M * N;
        if (pre != nullptr) pre += g * M * N;
        if (gout != nullptr) gout += g * M * N;
        if (acc_buf != nullptr) acc_buf += g * (MODE == 3 ? 2 : 1) * static_cast<int64_t>(N);
        counters += g * gridDim.y;
        if (out != nullptr) out += g * N;
        if (out2 != nullptr) out2 += g * N;
    }
    __shared__ float red[kColThreads * 8];
    __shared__ unsigned s_last;
    const int tid = threadIdx.x, cl = tid & 31, rl = tid >> 5;
    const int col = blockIdx.y * kSlabCols + 8 * cl;   // first of this thread's 8 columns
    const bool cols_ok = col < N;                       // N % 8 == 0, so all 8 or none
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_cta;
    const int64_t r1 = r0 + rows_per_cta < M ? r0 + rows_per_cta : M;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float acc2[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float gm[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if ((MODE == 1 || MODE == 3) && cols_ok) load8(gamma + col, gm);
    int64_t r = r0 + rl;
    if (cols_ok) {
        constexpr int U = col_unroll(MODE);
        for (; r + 8 * (U - 1) < r1; r += 8 * U) {
            Raw8<T> ra[U], rp[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                ra[u].load(x + (r + 8 * u) * N + col);
                if (MODE != 0) rp[u].load(pre + (r + 8 * u) * N + col);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                float a[8], p[8];
                ra[u].widen(a);
                if (MODE != 0) rp[u].widen(p);
                colreduce_row<T, MODE>(x, pre, gout, a, p, gm, acc, acc2, act, (r + 8 * u) * N + col);
            }
        }
        for (; r < r1; r += 8) {
            float a[8], p[8];
            load8(x + r * N + col, a);
            if (MODE != 0) load8(pre + r * N + col, p);
            colreduce_row<T, MODE>(x, pre, gout, a, p, gm, acc, acc2, act, r * N + col);
        }
    }
    if (acc_buf == nullptr) return;   // act_bwd without a bias gradient
#pragma unroll
    for (int c = 0; c < 8; ++c) red[tid * 8 + c] = acc[c];
    __syncthreads();
    if (rl == 0 && cols_ok) {
        for (int q = 1; q < 8; ++q)
#pragma unroll
            for (int c = 0; c < 8; ++c) acc[c] += red[(q * 32 + cl) * 8 + c];
        atomicAdd(reinterpret_cast<float4*>(acc_buf + col), make_float4(acc[0], acc[1], acc[2], acc[3]));
        atomicAdd(reinterpret_cast<float4*>(acc_buf + col + 4), make_float4(acc[4], acc[5], acc[6], acc[7]));
    }
    if constexpr (MODE == 3) {   // the second sum through the same shared buffer, into acc_buf + N
        __syncthreads();
#pragma unroll
        for (int c = 0; c < 8; ++c) red[tid * 8 + c] = acc2[c];
        __syncthreads();
        if (rl == 0 && cols_ok) {
            for (int q = 1; q < 8; ++q)
#pragma unroll
                for (int c = 0; c < 8; ++c) acc2[c] += red[(q * 32 + cl) * 8 + c];
            float* a2 = acc_buf + N;
            atomicAdd(reinterpret_cast<float4*>(a2 + col), make_float4(acc2[0], acc2[1], acc2[2], acc2[3]));
            atomicAdd(reinterpret_cast<float4*>(a2 + col + 4), make_float4(acc2[4], acc2[5], acc2[6], acc2[7]));
        }
    }
    // arrival: the last CTA of this slab writes the result and clears the scratch.  One thread
    // fences after the barrier (the barrier orders the CTA's atomics before it), as in a grid sync.
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        s_last = atomicAdd(&counters[blockIdx.y], 1u) == gridDim.x - 1;
        if (s_last) __threadfence();
    }
    __syncthreads();
    if (!s_last) return;
    if (rl == 0 && cols_ok) {
        float s[8];
        ldcg8(acc_buf + col, s);
        write_out8(out + col, s, 8, accumulate != 0);
        *reinterpret_cast<float4*>(acc_buf + col) = make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(acc_buf + col + 4) = make_float4(0.f, 0.f, 0.f, 0.f);
        if constexpr (MODE == 3) {
            float* a2 = acc_buf + N;
            ldcg8(a2 + col, s);
            write_out8(out2 + col, s, 8, accumulate2 != 0);
            *reinterpret_cast<float4*>(a2 + col) = make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4*>(a2 + col + 4) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    if (tid == 0) counters[blockIdx.y] = 0u;   // ready for the next launch (and graph replay)
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
        for (int c = 0; c < 8; ++c)
            o[c] = act == 3 ? g[c] * p[c] : act == 1 ? g[c] * gelu_grad(p[c]) : (p[c] > 0.f ? g[c] : 0.f);
        store8(gx + 8 * i, o);
    }
}

// y = GELU(x) (erf form) and, when d != nullptr, d = GELU'(x) -- the forward already evaluates the
// normal cdf / density, so storing the derivative (instead of x) leaves the backward a multiply.
// 8 elements per vector, four vectors in flight per thread.
template <typename T>
__global__ void __launch_bounds__(256) gelu_fwd_kernel(const T* __restrict__ x, T* __restrict__ y, T* __restrict__ d,
                                                       int64_t n8) {
    constexpr int U = 4;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8; i += U * stride) {
        Raw8<T> r[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (i + u * stride < n8) r[u].load(x + 8 * (i + u * stride));
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (i + u * stride < n8) {
                float a[8], o[8], g[8];
                r[u].widen(a);
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const NormalCdfPdf n = normal_cdf_pdf(a[c]);
                    o[c] = a[c] * n.cdf;
                    g[c] = fmaf(a[c], n.pdf, n.cdf);
                }
                store8(y + 8 * (i + u * stride), o);
                if (d != nullptr) store8(d + 8 * (i + u * stride), g);
            }
        }
    }
}


// out[rows[i]] += src[i] for every row i of src [n, C] (bf16; out zeroed by the caller): the backward of
// a row gather whose rows may repeat.  One thread per 8 columns of a row, four packed bf16 pair
// reductions into L2 (red.global.add.noftz.bf16x2).
__global__ void index_add_rows_kernel(const __nv_bfloat16* __restrict__ src, const int64_t* __restrict__ rows,
                                      __nv_bfloat16* __restrict__ out, int64_t n, int C) {
    const int c8 = C / 8;
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < n * c8;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t i = t / c8;
        const int c = static_cast<int>(t % c8) * 8;
        const uint4 v = *reinterpret_cast<const uint4*>(src + i * C + c);
        __nv_bfloat16* dst = out + rows[i] * C + c;
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 4; ++k)
            asm volatile("red.global.add.noftz.bf16x2 [%0], %1;" ::"l"(dst + 2 * k), "r"(w[k]) : "memory");
    }
}

// Non-overlapping p x p patches of a planar image [B, Cin, H, W] as GEMM rows: out[(b, py, px), (c, ky, kx)]
// (the patch-embedding convolution's im2col, with no copy of overlapping windows).  One thread per
// 8-pixel run of a patch row: a 16-byte read of the image row and a 16-byte write of the output row.
template <typename T>
__global__ void patch_unfold_kernel(const T* __restrict__ img, T* __restrict__ out, int B, int Cin, int H, int W,
                                    int p) {
    // 32-bit index decomposition (the launcher keeps the work count below 2^31); the pointer
    // offsets themselves are formed in 64 bits.
    const int hp = H / p, wp = W / p, runs = p / 8;
    const int per_patch = Cin * p * runs;
    const int total = B * hp * wp * per_patch;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += gridDim.x * blockDim.x) {
        const int patch = t / per_patch;                 // (b, py, px)
        const int rem = t - patch * per_patch;
        const int c = rem / (p * runs);
        const int ky = (rem / runs) % p;
        const int run = rem % runs;
        const int px = patch % wp, py = (patch / wp) % hp;
        const int b = patch / (wp * hp);
        const T* src = img + ((static_cast<int64_t>(b) * Cin + c) * H + py * p + ky) * W + px * p + run * 8;
        T* dst = out + static_cast<int64_t>(patch) * (Cin * p * p) + (c * p + ky) * p + run * 8;
        if constexpr (sizeof(T) == 2) {
            *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
        } else {
            reinterpret_cast<float4*>(dst)[0] = reinterpret_cast<const float4*>(src)[0];
            reinterpret_cast<float4*>(dst)[1] = reinterpret_cast<const float4*>(src)[1];
        }
    }
}

// out (+)= acc, then acc = 0 (finishes a column sum accumulated by another kernel's atomics)
template <typename TO>
__global__ void colacc_finalize_kernel(float* acc, TO* out, int N, int accumulate) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= N) return;
    const float s = acc[c];
    out[c] = from_f<TO>((accumulate ? to_f(out[c]) : 0.f) + s);
    acc[c] = 0.f;
}

std::mutex g_scratch_mu;
void* g_scratch[64] = {nullptr};

}  // namespace

// Per-device zero-initialised scratch of the single-launch reductions: kMaxCounters arrival
// counters followed by kReduceAccFloats fp32 accumulators.  Every launch leaves it zeroed.
ReduceScratch reduce_scratch() {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return {nullptr, nullptr};
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (g_scratch[dev] == nullptr) {
        const size_t bytes = kMaxCounters * sizeof(unsigned) + kReduceAccFloats * sizeof(float);
        void* p = nullptr;
        if (cudaMalloc(&p, bytes) != cudaSuccess) return {nullptr, nullptr};
        if (cudaMemset(p, 0, bytes) != cudaSuccess) return {nullptr, nullptr};
        g_scratch[dev] = p;
    }
    unsigned* c = static_cast<unsigned*>(g_scratch[dev]);
    return {c, reinterpret_cast<float*>(c + kMaxCounters)};
}

static int colsum_parts(int64_t M, int N, int mode) {
    const int64_t slabs = (N + kSlabCols - 1) / kSlabCols;
    int64_t want = static_cast<int64_t>(num_sms()) * kColCtasPerSm / slabs;
    want = std::max<int64_t>(1, std::min<int64_t>(want, (M + 8 * col_unroll(mode) - 1) / (8 * col_unroll(mode))));
    return static_cast<int>(want);
}

static cudaError_t launch_colreduce(DType t, DType out_t, int mode, const void* x, const void* pre,
                                    const void* gamma, void* gout, int64_t M, int N, int act, void* out,
                                    bool accumulate, cudaStream_t st, void* out2 = nullptr, bool accumulate2 = false,
                                    int groups = 1) {
    if (N % 8 != 0 || groups < 1 || groups > 65535) return cudaErrorInvalidValue;
    const int slabs = (N + kSlabCols - 1) / kSlabCols;
    if (static_cast<int64_t>(slabs) * groups > kMaxCounters ||
        (out != nullptr && static_cast<int64_t>(N) * groups > kReduceAccFloats))
        return cudaErrorInvalidValue;
    if (mode == 3 && (out2 == nullptr || out == nullptr || 2 * static_cast<int64_t>(N) * groups > kReduceAccFloats))
        return cudaErrorInvalidValue;
    const ReduceScratch rs = reduce_scratch();
    if (rs.counters == nullptr) return cudaErrorMemoryAllocation;
    unsigned* counters = rs.counters;
    float* acc_buf = out != nullptr ? rs.acc : nullptr;   // null: no column sum wanted
    const int parts = std::max(1, colsum_parts(M, N, mode) / groups);
    const int rows_per_cta = static_cast<int>((M + parts - 1) / parts);
    const dim3 grid(parts, slabs, groups);
    return MMLTK_DISPATCH_DT(t, [&] {
        using T = scalar_t;
        return MMLTK_DISPATCH_DT(out_t, [&] {
            using TO = scalar_t;
            const T* xx = static_cast<const T*>(x);
            const T* pp = static_cast<const T*>(pre);
            const T* gg = static_cast<const T*>(gamma);
            T* go = static_cast<T*>(gout);
            TO* oo = static_cast<TO*>(out);
            TO* o2 = static_cast<TO*>(out2);
            const int a1 = accumulate ? 1 : 0, a2 = accumulate2 ? 1 : 0;
            if (mode == 0)
                colreduce_kernel<T, 0, TO><<<grid, kColThreads, 0, st>>>(xx, pp, gg, go, M, N, rows_per_cta, act,
                                                                        acc_buf, counters, oo, a1, o2, a2);
            else if (mode == 1)
                colreduce_kernel<T, 1, TO><<<grid, kColThreads, 0, st>>>(xx, pp, gg, go, M, N, rows_per_cta, act,
                                                                        acc_buf, counters, oo, a1, o2, a2);
            else if (mode == 2)
                colreduce_kernel<T, 2, TO><<<grid, kColThreads, 0, st>>>(xx, pp, gg, go, M, N, rows_per_cta, act,
                                                                        acc_buf, counters, oo, a1, o2, a2);
            else
                colreduce_kernel<T, 3, TO><<<grid, kColThreads, 0, st>>>(xx, pp, gg, go, M, N, rows_per_cta, act,
                                                                        acc_buf, counters, oo, a1, o2, a2);
            return cudaGetLastError();
        });
    });
}

cudaError_t launch_colsum(DType t, DType out_t, int mode, const void* x, const void* pre, const void* gamma,
                          void* gout, int64_t M, int N, void* out, cudaStream_t st, bool accumulate, int groups) {
    if (out == nullptr) return cudaErrorInvalidValue;
    return launch_colreduce(t, out_t, mode, x, pre, gamma, gout, M, N, 0, out, accumulate, st, nullptr, false, groups);
}

cudaError_t launch_scale_bias_bwd(DType t, DType out_t, const void* gy, const void* pre, const void* gamma, void* gpre,
                                  int64_t M, int N, void* ggamma, bool acc_gamma, void* gbias, bool acc_bias,
                                  cudaStream_t st) {
    return launch_colreduce(t, out_t, 3, gy, pre, gamma, gpre, M, N, 0, ggamma, acc_gamma, st, gbias, acc_bias);
}

cudaError_t launch_act_bwd_bias(DType t, DType out_t, const void* gy, const void* pre, void* gx, int64_t M, int N,
                                int act, void* gb, bool accumulate, cudaStream_t st) {
    return launch_colreduce(t, out_t, 2, gy, pre, nullptr, gx, M, N, act, gb, accumulate, st);
}

cudaError_t launch_colacc_finalize(float* acc, DType out_t, void* out, int N, bool accumulate, cudaStream_t st) {
    return MMLTK_DISPATCH_DT(out_t, [&] {
        colacc_finalize_kernel<scalar_t><<<(N + 255) / 256, 256, 0, st>>>(acc, static_cast<scalar_t*>(out), N,
                                                                          accumulate ? 1 : 0);
        return cudaGetLastError();
    });
}


cudaError_t launch_patch_unfold(DType t, const void* img, void* out, int B, int Cin, int H, int W, int p,
                                cudaStream_t st) {
    if (p % 8 != 0 || H % p != 0 || W % p != 0 || W % 8 != 0) return cudaErrorInvalidValue;
    const int64_t total = static_cast<int64_t>(B) * (H / p) * (W / p) * Cin * p * (p / 8);
    if (total == 0) return cudaSuccess;
    const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, static_cast<int64_t>(num_sms()) * 16));
    // the kernel indexes its work items in 32 bits, grid-stride step included
    if (total + static_cast<int64_t>(blocks) * 256 >= (int64_t(1) << 31) ||
        static_cast<int64_t>(Cin) * p * p >= (int64_t(1) << 31))
        return cudaErrorInvalidValue;
    return MMLTK_DISPATCH_DT(t, [&] {
        using T = scalar_t;
        patch_unfold_kernel<T><<<blocks, 256, 0, st>>>(static_cast<const T*>(img), static_cast<T*>(out), B, Cin, H, W,
                                                        p);
        return cudaGetLastError();
    });
}

cudaError_t launch_index_add_rows(const void* src, const int64_t* rows, void* out, int64_t n, int C, cudaStream_t st) {
    if (C % 8 != 0) return cudaErrorInvalidValue;
    if (n == 0) return cudaSuccess;
    const int64_t work = n * (C / 8);
    const int blocks = static_cast<int>(std::min<int64_t>((work + 255) / 256, static_cast<int64_t>(num_sms()) * 16));
    index_add_rows_kernel<<<blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(src), rows,
                                                  static_cast<__nv_bfloat16*>(out), n, C);
    return cudaGetLastError();
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

cudaError_t launch_gelu_fwd(DType t, const void* x, void* y, int64_t n, cudaStream_t st, void* deriv) {
    if (n % 8 != 0) return cudaErrorInvalidValue;
    const int64_t n8 = n / 8;
    if (n8 == 0) return cudaSuccess;
    const int blocks = static_cast<int>(std::min<int64_t>((n8 + 1023) / 1024, static_cast<int64_t>(num_sms()) * 8));
    return MMLTK_DISPATCH_DT(t, [&] {
        using T = scalar_t;
        gelu_fwd_kernel<T><<<std::max(blocks, 1), 256, 0, st>>>(static_cast<const T*>(x), static_cast<T*>(y),
                                                                static_cast<T*>(deriv), n8);
        return cudaGetLastError();
    });
}

}  // namespace mmltk
