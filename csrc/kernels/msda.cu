// Fused multi-scale deformable attention (forward and backward), bf16 in,
// fp32 accumulation.
//
// Reference semantics: `MSDeformAttnImpl::forward` (softmax over levels x
// points, loc = ref_xy + off / P * ref_wh * 0.5; `src/rfdetr/layers/model.cpp:829-871`)
// followed by the fp32 im2col/col2im kernels
// (`src/rfdetr/cuda/ms_deform_im2col_cuda.cuh:481-753`), i.e. bilinear
// sampling with align_corners=false and zero padding.
//
// Mapping: one "item" = (batch, query, head); D/8 threads per item, each
// owning 8 channels moved as one 16-byte vector per bilinear corner.  The
// softmax and the location arithmetic are recomputed per item inside the
// kernel, so the op consumes the raw sampling_offsets / attention_weights
// linear outputs and the (cx, cy, w, h) reference boxes directly.
//
// Backward: grad_value is accumulated with 16-byte fp32 vector atomics into a
// scratch accumulator [B, S, H, D] (then cast to the value dtype); the
// per-point dot products for the weight / location gradients are reduced
// across the D/8 threads of an item with shuffles; softmax, offset and
// reference-box gradients are produced in the same pass.
#include "common.cuh"

namespace mmltk {

namespace {

constexpr int kMaxLP = 32;
constexpr int kMaxLevels = 8;

template <int TPI>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int o = TPI / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o, TPI);
    return v;
}

template <typename T, int D>
__global__ void __launch_bounds__(256) msda_fwd_kernel(const T* __restrict__ value, const int* __restrict__ shapes,
                                                       const int* __restrict__ starts, const T* __restrict__ ref,
                                                       const T* __restrict__ off, const T* __restrict__ logits,
                                                       T* __restrict__ out, MsdaDims d) {
    constexpr int TPI = D / 8;
    __shared__ int s_h[kMaxLevels], s_w[kMaxLevels], s_st[kMaxLevels];
    if (threadIdx.x < d.L) {
        s_h[threadIdx.x] = shapes[2 * threadIdx.x];
        s_w[threadIdx.x] = shapes[2 * threadIdx.x + 1];
        s_st[threadIdx.x] = starts[threadIdx.x];
    }
    __syncthreads();
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t items = static_cast<int64_t>(d.B) * d.Lq * d.H;
    const int64_t item = tid / TPI;
    const int sub = static_cast<int>(tid % TPI);
    if (item >= items) return;
    const int h = static_cast<int>(item % d.H);
    const int64_t bq = item / d.H;
    const int b = static_cast<int>(bq / d.Lq);
    const int LP = d.L * d.P;

    // softmax over levels x points
    const T* lg = logits + item * LP;
    float wts[kMaxLP];
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < kMaxLP; ++k)
        if (k < LP) {
            wts[k] = to_f(lg[k]);
            mx = fmaxf(mx, wts[k]);
        }
    float den = 0.f;
#pragma unroll
    for (int k = 0; k < kMaxLP; ++k)
        if (k < LP) {
            wts[k] = __expf(wts[k] - mx);
            den += wts[k];
        }
    const float inv = 1.f / den;

    float acc[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] = 0.f;
    const T* rp = ref + bq * d.L * 4;
    const T* op = off + item * LP * 2;
    const float invP = 1.f / d.P;
    const int64_t vstride = static_cast<int64_t>(d.H) * D;
    const T* vb = value + static_cast<int64_t>(b) * d.S * vstride + h * D + sub * 8;
    for (int l = 0; l < d.L; ++l) {
        const float rx = to_f(rp[4 * l]), ry = to_f(rp[4 * l + 1]);
        const float rw = to_f(rp[4 * l + 2]) * 0.5f * invP, rh = to_f(rp[4 * l + 3]) * 0.5f * invP;
        const int Hl = s_h[l], Wl = s_w[l];
        const T* vl = vb + static_cast<int64_t>(s_st[l]) * vstride;
        for (int p = 0; p < d.P; ++p) {
            const int k = l * d.P + p;
            const float lx = rx + to_f(op[2 * k]) * rw;
            const float ly = ry + to_f(op[2 * k + 1]) * rh;
            const float x = lx * Wl - 0.5f, y = ly * Hl - 0.5f;
            if (!(x > -1.f && y > -1.f && x < Wl && y < Hl)) continue;
            const float a = wts[k] * inv;
            const int x0 = static_cast<int>(floorf(x)), y0 = static_cast<int>(floorf(y));
            const float fx = x - x0, fy = y - y0, hx = 1.f - fx, hy = 1.f - fy;
            const float cw[4] = {hy * hx, hy * fx, fy * hx, fy * fx};
#pragma unroll
            for (int corner = 0; corner < 4; ++corner) {
                const int xx = x0 + (corner & 1), yy = y0 + (corner >> 1);
                if (xx < 0 || yy < 0 || xx >= Wl || yy >= Hl) continue;
                float v[8];
                load8(vl + (static_cast<int64_t>(yy) * Wl + xx) * vstride, v);
                const float s = a * cw[corner];
#pragma unroll
                for (int c = 0; c < 8; ++c) acc[c] += s * v[c];
            }
        }
    }
    store8(out + item * D + sub * 8, acc);
}

template <typename T, int D>
__global__ void __launch_bounds__(256, 3) msda_bwd_kernel(const T* __restrict__ gout, const T* __restrict__ value,
                                                       const int* __restrict__ shapes, const int* __restrict__ starts,
                                                       const T* __restrict__ ref, const T* __restrict__ off,
                                                       const T* __restrict__ logits, float* __restrict__ gvalue,
                                                       float* __restrict__ gref, T* __restrict__ goff,
                                                       T* __restrict__ glogits, MsdaDims d) {
    constexpr int TPI = D / 8;
    __shared__ int s_h[kMaxLevels], s_w[kMaxLevels], s_st[kMaxLevels];
    if (threadIdx.x < d.L) {
        s_h[threadIdx.x] = shapes[2 * threadIdx.x];
        s_w[threadIdx.x] = shapes[2 * threadIdx.x + 1];
        s_st[threadIdx.x] = starts[threadIdx.x];
    }
    __syncthreads();
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t items = static_cast<int64_t>(d.B) * d.Lq * d.H;
    // whole item groups stay together in a warp (TPI divides 32); tail threads
    // of the last warp take part in the shuffles with zero contributions
    const int64_t item_raw = tid / TPI;
    const bool active = item_raw < items;
    const int64_t item = active ? item_raw : items - 1;
    const int sub = static_cast<int>(tid % TPI);
    const int h = static_cast<int>(item % d.H);
    const int64_t bq = item / d.H;
    const int b = static_cast<int>(bq / d.Lq);
    const int LP = d.L * d.P;

    const T* lg = logits + item * LP;
    float wts[kMaxLP];
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < kMaxLP; ++k)
        if (k < LP) {
            wts[k] = to_f(lg[k]);
            mx = fmaxf(mx, wts[k]);
        }
    float den = 0.f;
#pragma unroll
    for (int k = 0; k < kMaxLP; ++k)
        if (k < LP) {
            wts[k] = __expf(wts[k] - mx);
            den += wts[k];
        }
    const float inv = 1.f / den;
#pragma unroll
    for (int k = 0; k < kMaxLP; ++k)
        if (k < LP) wts[k] *= inv;

    float g[8];
    load8(gout + item * D + sub * 8, g);
    if (!active) {
#pragma unroll
        for (int c = 0; c < 8; ++c) g[c] = 0.f;
    }

    const T* rp = ref + bq * d.L * 4;
    const T* op = off + item * LP * 2;
    const float invP = 1.f / d.P;
    const int64_t vstride = static_cast<int64_t>(d.H) * D;
    const int64_t vbase = static_cast<int64_t>(b) * d.S * vstride + h * D + sub * 8;

    float gw[kMaxLP];
    float gsum = 0.f;
    float gref_acc[kMaxLevels][4];
    for (int l = 0; l < d.L; ++l) {
        const float rx = to_f(rp[4 * l]), ry = to_f(rp[4 * l + 1]);
        const float rwh = to_f(rp[4 * l + 2]), rhh = to_f(rp[4 * l + 3]);
        const float rw = rwh * 0.5f * invP, rh = rhh * 0.5f * invP;
        const int Hl = s_h[l], Wl = s_w[l];
        const int64_t lbase = vbase + static_cast<int64_t>(s_st[l]) * vstride;
        float g_rx = 0.f, g_ry = 0.f, g_rw = 0.f, g_rh = 0.f;
        for (int p = 0; p < d.P; ++p) {
            const int k = l * d.P + p;
            const float ox = to_f(op[2 * k]), oy = to_f(op[2 * k + 1]);
            const float lx = rx + ox * rw, ly = ry + oy * rh;
            const float x = lx * Wl - 0.5f, y = ly * Hl - 0.5f;
            float dot = 0.f, dx = 0.f, dy = 0.f;
            if (x > -1.f && y > -1.f && x < Wl && y < Hl) {
                const int x0 = static_cast<int>(floorf(x)), y0 = static_cast<int>(floorf(y));
                const float fx = x - x0, fy = y - y0, hx = 1.f - fx, hy = 1.f - fy;
                const float cw[4] = {hy * hx, hy * fx, fy * hx, fy * fx};
                const float cdx[4] = {-hy, hy, -fy, fy};
                const float cdy[4] = {-hx, -fx, hx, fx};
                const float a = wts[k];
#pragma unroll
                for (int corner = 0; corner < 4; ++corner) {
                    const int xx = x0 + (corner & 1), yy = y0 + (corner >> 1);
                    if (xx < 0 || yy < 0 || xx >= Wl || yy >= Hl) continue;
                    const int64_t off_v = lbase + (static_cast<int64_t>(yy) * Wl + xx) * vstride;
                    float v[8];
                    load8(value + off_v, v);
                    float gv = 0.f;
#pragma unroll
                    for (int c = 0; c < 8; ++c) gv += g[c] * v[c];
                    dot += cw[corner] * gv;
                    dx += cdx[corner] * gv;
                    dy += cdy[corner] * gv;
                    if (active) {
                        const float s = a * cw[corner];
                        float4* dst = reinterpret_cast<float4*>(gvalue + off_v);
                        atomicAdd(dst, make_float4(s * g[0], s * g[1], s * g[2], s * g[3]));
                        atomicAdd(dst + 1, make_float4(s * g[4], s * g[5], s * g[6], s * g[7]));
                    }
                }
            }
            dot = group_sum<TPI>(dot);
            dx = group_sum<TPI>(dx);
            dy = group_sum<TPI>(dy);
            gw[k] = dot;
            gsum += wts[k] * dot;
            const float glx = wts[k] * dx * Wl, gly = wts[k] * dy * Hl;
            if (sub == 0 && active) {
                goff[(item * LP + k) * 2] = from_f<T>(glx * rw);
                goff[(item * LP + k) * 2 + 1] = from_f<T>(gly * rh);
            }
            g_rx += glx;
            g_ry += gly;
            g_rw += glx * ox * 0.5f * invP;
            g_rh += gly * oy * 0.5f * invP;
        }
        gref_acc[l][0] = g_rx;
        gref_acc[l][1] = g_ry;
        gref_acc[l][2] = g_rw;
        gref_acc[l][3] = g_rh;
    }
    if (sub == 0 && active) {
#pragma unroll
        for (int k = 0; k < kMaxLP; ++k)
            if (k < LP) glogits[item * LP + k] = from_f<T>(wts[k] * (gw[k] - gsum));
        for (int l = 0; l < d.L; ++l)
#pragma unroll
            for (int c = 0; c < 4; ++c) atomicAdd(gref + (bq * d.L + l) * 4 + c, gref_acc[l][c]);
    }
}

template <typename T>
__global__ void f32_to_kernel(const float* __restrict__ src, T* __restrict__ dst, int64_t n) {
    const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
    if (i + 3 < n) {
        store4(dst + i, *reinterpret_cast<const float4*>(src + i));
    } else {
        for (int64_t j = i; j < n; ++j) dst[j] = from_f<T>(src[j]);
    }
}

template <typename F>
cudaError_t dispatch_head_dim(int D, F&& f) {
    switch (D) {
        case 8: return f(std::integral_constant<int, 8>{});
        case 16: return f(std::integral_constant<int, 16>{});
        case 32: return f(std::integral_constant<int, 32>{});
        case 64: return f(std::integral_constant<int, 64>{});
        case 128: return f(std::integral_constant<int, 128>{});
        default: return cudaErrorInvalidValue;
    }
}

bool dims_ok(const MsdaDims& d) {
    return d.L >= 1 && d.L <= kMaxLevels && d.P >= 1 && d.L * d.P <= kMaxLP;
}

}  // namespace

cudaError_t launch_msda_fwd(DType t, const void* value, const int* shapes, const int* starts, const void* ref,
                            const void* off, const void* logits, void* out, MsdaDims d, cudaStream_t st) {
    if (!dims_ok(d)) return cudaErrorInvalidValue;
    const int64_t threads_total = static_cast<int64_t>(d.B) * d.Lq * d.H * (d.D / 8);
    if (threads_total == 0) return cudaSuccess;
    const int threads = 256;
    const int64_t blocks = (threads_total + threads - 1) / threads;
    return MMLTK_DISPATCH_DT(t, [&] {
        using T = scalar_t;
        return dispatch_head_dim(d.D, [&](auto dd) {
            msda_fwd_kernel<T, decltype(dd)::value><<<blocks, threads, 0, st>>>(
                static_cast<const T*>(value), shapes, starts, static_cast<const T*>(ref), static_cast<const T*>(off),
                static_cast<const T*>(logits), static_cast<T*>(out), d);
            return cudaGetLastError();
        });
    });
}

template <typename T>
cudaError_t cast_f32_impl(const float* src, T* dst, int64_t n, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    f32_to_kernel<T><<<(n / 4 + 255) / 256 + 1, 256, 0, st>>>(src, dst, n);
    return cudaGetLastError();
}

cudaError_t launch_cast_f32(DType dst_t, const float* src, void* dst, int64_t n, cudaStream_t st) {
    if (dst_t == DType::kBF16) return cast_f32_impl(src, static_cast<__nv_bfloat16*>(dst), n, st);
    return cast_f32_impl(src, static_cast<float*>(dst), n, st);
}

cudaError_t launch_msda_bwd(DType t, const void* gout, const void* value, const int* shapes, const int* starts,
                            const void* ref, const void* off, const void* logits, float* gvalue_acc, float* gref_acc,
                            void* gvalue, void* gref, void* goff, void* glogits, MsdaDims d, cudaStream_t st) {
    if (!dims_ok(d)) return cudaErrorInvalidValue;
    const int64_t nv = static_cast<int64_t>(d.B) * d.S * d.H * d.D;
    const int64_t nr = static_cast<int64_t>(d.B) * d.Lq * d.L * 4;
    cudaError_t e = cudaMemsetAsync(gvalue_acc, 0, nv * sizeof(float), st);
    if (e != cudaSuccess) return e;
    e = cudaMemsetAsync(gref_acc, 0, nr * sizeof(float), st);
    if (e != cudaSuccess) return e;
    const int64_t threads_total = static_cast<int64_t>(d.B) * d.Lq * d.H * (d.D / 8);
    const int threads = 256;
    if (threads_total > 0) {
        const int64_t blocks = (threads_total + threads - 1) / threads;
        e = MMLTK_DISPATCH_DT(t, [&] {
            using T = scalar_t;
            return dispatch_head_dim(d.D, [&](auto dd) {
                msda_bwd_kernel<T, decltype(dd)::value><<<blocks, threads, 0, st>>>(
                    static_cast<const T*>(gout), static_cast<const T*>(value), shapes, starts,
                    static_cast<const T*>(ref), static_cast<const T*>(off), static_cast<const T*>(logits), gvalue_acc,
                    gref_acc, static_cast<T*>(goff), static_cast<T*>(glogits), d);
                return cudaGetLastError();
            });
        });
        if (e != cudaSuccess) return e;
    }
    e = launch_cast_f32(t, gvalue_acc, gvalue, nv, st);
    if (e != cudaSuccess) return e;
    return launch_cast_f32(t, gref_acc, gref, nr, st);
}

}  // namespace mmltk
