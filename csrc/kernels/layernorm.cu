// LayerNorm over the last dimension, one warp per row.
//
// Forward: y = (x - mean) * rstd * w + b, statistics in fp32 (two passes over
// registers, no E[x^2]-E[x]^2 cancellation).  Saves mean/rstd for backward.
// Backward: dx per row; dgamma/dbeta accumulated per lane over the rows its
// warp visits (each lane owns fixed columns), reduced across the CTA's warps
// in shared memory, added into per-device fp32 accumulators with vector
// atomics; the last CTA to arrive writes (or accumulates into) dgamma/dbeta.
// One launch; float atomics make the last bits run dependent.
#include <algorithm>

#include "common.cuh"

namespace mmltk {

namespace {

// Optional fusions of the forward: res -> normalise x + res (+ rbias, a bias row vector of the
// residual branch) and store the sum -- or, with rscale, res + rscale * (x + rbias), a LayerScale
// residual; pos -> also store y + pos.
template <typename T, typename W>
struct LnFwdExtra {
    const T* res;
    T* sum;
    const T* pos;
    T* y2;
    const W* rbias;
    const W* rscale;   // with res: normalise res + rscale * (x + rbias) (a LayerScale residual)
    const int* ymap;   // y row of input row r (negative: not stored); null: row r
    int64_t yld;       // y row pitch with ymap
    int64_t wgroup_rows;   // > 0: rows come in groups of this many, group g normalised with w / b row g
    int act;               // 1: y = SiLU(normalised row), the channels-last ConvX's norm + activation
};

__device__ __forceinline__ float silu_f(float o) { return o / (1.f + __expf(-o)); }
// d SiLU / d o = s (1 + o (1 - s)), s = sigmoid(o)
__device__ __forceinline__ float silu_grad_f(float o) {
    const float s = 1.f / (1.f + __expf(-o));
    return s * (1.f + o * (1.f - s));
}

template <typename T, typename W, int kMaxVec>
__global__ void __launch_bounds__(256) ln_fwd_kernel(const T* __restrict__ x, const W* __restrict__ w,
                                                     const W* __restrict__ b, T* __restrict__ y,
                                                     float* __restrict__ mean_out, float* __restrict__ rstd_out,
                                                     int64_t rows, int C, float eps, LnFwdExtra<T, W> ex) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const int nv = C >> 2;
    for (int64_t r = warp; r < rows; r += nwarps) {
        const T* xr = x + r * C;
        float4 v[kMaxVec];
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < kMaxVec; ++k) {
            const int i = lane + 32 * k;
            if (i < nv) {
                v[k] = load4(xr + 4 * i);
                if (ex.res != nullptr) {   // fused residual add: the norm's input is x + res (+ rbias)
                    const float4 r4 = load4(ex.res + r * C + 4 * i);
                    const int c0 = 4 * i;
                    if (ex.rscale != nullptr) {   // res + gamma * (x + rbias)
                        if (ex.rbias != nullptr) {
                            v[k].x += to_f(ex.rbias[c0]); v[k].y += to_f(ex.rbias[c0 + 1]);
                            v[k].z += to_f(ex.rbias[c0 + 2]); v[k].w += to_f(ex.rbias[c0 + 3]);
                        }
                        v[k].x = r4.x + to_f(ex.rscale[c0]) * v[k].x;
                        v[k].y = r4.y + to_f(ex.rscale[c0 + 1]) * v[k].y;
                        v[k].z = r4.z + to_f(ex.rscale[c0 + 2]) * v[k].z;
                        v[k].w = r4.w + to_f(ex.rscale[c0 + 3]) * v[k].w;
                    } else {
                        v[k].x += r4.x; v[k].y += r4.y; v[k].z += r4.z; v[k].w += r4.w;
                        if (ex.rbias != nullptr) {
                            v[k].x += to_f(ex.rbias[c0]); v[k].y += to_f(ex.rbias[c0 + 1]);
                            v[k].z += to_f(ex.rbias[c0 + 2]); v[k].w += to_f(ex.rbias[c0 + 3]);
                        }
                    }
                    store4(ex.sum + r * C + 4 * i, v[k]);
                }
                s += v[k].x + v[k].y + v[k].z + v[k].w;
            }
        }
        const float mean = warp_sum(s) / C;
        float q = 0.f;
#pragma unroll
        for (int k = 0; k < kMaxVec; ++k) {
            const int i = lane + 32 * k;
            if (i < nv) {
                const float a = v[k].x - mean, bb = v[k].y - mean, c = v[k].z - mean, d = v[k].w - mean;
                q += a * a + bb * bb + c * c + d * d;
            }
        }
        const float rstd = rsqrtf(warp_sum(q) / C + eps);
        const int64_t orow = ex.ymap != nullptr ? ex.ymap[r] : r;
        T* yr = y + orow * (ex.ymap != nullptr ? ex.yld : C);
        const int64_t woff = ex.wgroup_rows > 0 ? (r / ex.wgroup_rows) * C : 0;
        const W* __restrict__ wr = w + woff;
        const W* __restrict__ br = b + woff;
#pragma unroll
        for (int k = 0; k < kMaxVec; ++k) {
            const int i = lane + 32 * k;
            if (i < nv && orow >= 0) {
                const int c0 = 4 * i;
                float4 o;
                o.x = (v[k].x - mean) * rstd * to_f(wr[c0]) + to_f(br[c0]);
                o.y = (v[k].y - mean) * rstd * to_f(wr[c0 + 1]) + to_f(br[c0 + 1]);
                o.z = (v[k].z - mean) * rstd * to_f(wr[c0 + 2]) + to_f(br[c0 + 2]);
                o.w = (v[k].w - mean) * rstd * to_f(wr[c0 + 3]) + to_f(br[c0 + 3]);
                if (ex.act == 1) o = make_float4(silu_f(o.x), silu_f(o.y), silu_f(o.z), silu_f(o.w));
                store4(yr + c0, o);
                if (ex.pos != nullptr) {   // second output y + pos (e.g. a query with its position embedding)
                    const float4 p4 = load4(ex.pos + r * C + c0);
                    store4(ex.y2 + r * C + c0, make_float4(o.x + p4.x, o.y + p4.y, o.z + p4.z, o.w + p4.w));
                }
            }
        }
        if (lane == 0) {
            mean_out[r] = mean;
            rstd_out[r] = rstd;
        }
    }
}

// 4 elements as loaded, widened only when used (keeps the next row's loads in few registers)
template <typename T>
struct Raw4;
template <>
struct Raw4<__nv_bfloat16> {
    uint2 v;
    __device__ __forceinline__ void load(const __nv_bfloat16* p) { v = *reinterpret_cast<const uint2*>(p); }
    __device__ __forceinline__ void zero() { v = make_uint2(0u, 0u); }
    __device__ __forceinline__ float4 widen() const {
        const float2 a = unpack_bf16x2(v.x), b = unpack_bf16x2(v.y);
        return make_float4(a.x, a.y, b.x, b.y);
    }
};
template <>
struct Raw4<float> {
    float4 v;
    __device__ __forceinline__ void load(const float* p) { v = *reinterpret_cast<const float4*>(p); }
    __device__ __forceinline__ void zero() { v = make_float4(0.f, 0.f, 0.f, 0.f); }
    __device__ __forceinline__ float4 widen() const { return v; }
};

// one row of the backward pass: xv / gv hold this lane's x and gy columns (fp32)
template <typename T, typename W, int kMaxVec, bool kBias2>
__device__ __forceinline__ void ln_bwd_row(float4 (&xh)[kMaxVec], float4 (&g)[kMaxVec], float mean, float rstd,
                                           const W* __restrict__ w, float4 (&aw)[kMaxVec], float4 (&ab)[kMaxVec],
                                           float4 (&ad)[kMaxVec], T* __restrict__ gxr, int lane,
                                           int nv, int C, const T* __restrict__ gresr, const W* __restrict__ bvec,
                                           int act) {
    // the residual gradient is loaded first so its latency hides behind the reductions below
    Raw4<T> gr[kMaxVec];
    if (gresr != nullptr) {
#pragma unroll
        for (int k = 0; k < kMaxVec; ++k)
            if (lane + 32 * k < nv) gr[k].load(gresr + 4 * (lane + 32 * k));
    }
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int k = 0; k < kMaxVec; ++k) {
        const int i = lane + 32 * k;
        if (i < nv) {
            const int c0 = 4 * i;
            const float4 xv = xh[k];
            float4 gv = g[k];
            xh[k] = make_float4((xv.x - mean) * rstd, (xv.y - mean) * rstd, (xv.z - mean) * rstd,
                                (xv.w - mean) * rstd);
            if (act == 1) {   // the forward applied SiLU to the affine output: recompute it, chain its slope
                gv.x *= silu_grad_f(xh[k].x * to_f(w[c0]) + to_f(bvec[c0]));
                gv.y *= silu_grad_f(xh[k].y * to_f(w[c0 + 1]) + to_f(bvec[c0 + 1]));
                gv.z *= silu_grad_f(xh[k].z * to_f(w[c0 + 2]) + to_f(bvec[c0 + 2]));
                gv.w *= silu_grad_f(xh[k].w * to_f(w[c0 + 3]) + to_f(bvec[c0 + 3]));
            }
            aw[k].x += gv.x * xh[k].x; aw[k].y += gv.y * xh[k].y;
            aw[k].z += gv.z * xh[k].z; aw[k].w += gv.w * xh[k].w;
            ab[k].x += gv.x; ab[k].y += gv.y; ab[k].z += gv.z; ab[k].w += gv.w;
            g[k] = make_float4(gv.x * to_f(w[c0]), gv.y * to_f(w[c0 + 1]), gv.z * to_f(w[c0 + 2]),
                               gv.w * to_f(w[c0 + 3]));
            s1 += g[k].x + g[k].y + g[k].z + g[k].w;
            s2 += g[k].x * xh[k].x + g[k].y * xh[k].y + g[k].z * xh[k].z + g[k].w * xh[k].w;
        }
    }
    s1 = warp_sum(s1) / C;
    s2 = warp_sum(s2) / C;
#pragma unroll
    for (int k = 0; k < kMaxVec; ++k) {
        const int i = lane + 32 * k;
        if (i < nv) {
            float4 o;
            o.x = (g[k].x - s1 - xh[k].x * s2) * rstd;
            o.y = (g[k].y - s1 - xh[k].y * s2) * rstd;
            o.z = (g[k].z - s1 - xh[k].z * s2) * rstd;
            o.w = (g[k].w - s1 - xh[k].w * s2) * rstd;
            if constexpr (kBias2) {   // column sums of the input gradient: the fused residual branch's bias gradient
                ad[k].x += o.x; ad[k].y += o.y; ad[k].z += o.z; ad[k].w += o.w;
            }
            if (gresr != nullptr) {   // gradient reaching x through a residual branch, added here
                const float4 r4 = gr[k].widen();
                o.x += r4.x; o.y += r4.y; o.z += r4.z; o.w += r4.w;
            }
            store4(gxr + 4 * i, o);
        }
    }
}

template <typename T, typename W, int kMaxVec, bool kBias2>
__global__ void __launch_bounds__(256) ln_bwd_kernel(const T* __restrict__ gy, const T* __restrict__ x,
                                                     const W* __restrict__ w, const float* __restrict__ mean_in,
                                                     const float* __restrict__ rstd_in, T* __restrict__ gx,
                                                     float* acc_w, float* acc_b, unsigned* counter,
                                                     W* __restrict__ gw, W* __restrict__ gb, int accumulate,
                                                     int64_t rows, int C, const T* __restrict__ gy2,
                                                     const T* __restrict__ gres, W* __restrict__ gbias2,
                                                     int accumulate2, const int* __restrict__ gmap, int64_t gld,
                                                     int64_t group_rows, const W* __restrict__ bvec, int act) {
    extern __shared__ float smem[];  // [warps][2][C]
    // groups (group_rows > 0): blockIdx.y = group g, rows [g * group_rows, +group_rows), weight / bias
    // row g, gradient accumulators, arrival counter and gw / gb row of that group
    int64_t row_begin = 0;
    if (group_rows > 0) {
        const int g = blockIdx.y;
        row_begin = g * group_rows;
        rows = min(rows, row_begin + group_rows);
        w += static_cast<int64_t>(g) * C;
        if (bvec != nullptr) bvec += static_cast<int64_t>(g) * C;
        gw += static_cast<int64_t>(g) * C;
        gb += static_cast<int64_t>(g) * C;
        acc_w += static_cast<int64_t>(g) * (kBias2 ? 3 : 2) * C;
        acc_b += static_cast<int64_t>(g) * (kBias2 ? 3 : 2) * C;
        counter += g;
    }
    // this row's output gradient: row gmap[r] of gy (pitch gld; none = zero) or row r
    auto gy_row = [&](int64_t r) -> const T* {
        if (gmap == nullptr) return gy + r * C;
        const int g = gmap[r];
        return g >= 0 ? gy + static_cast<int64_t>(g) * gld : nullptr;
    };
    const int lane = threadIdx.x & 31;
    const int wib = threadIdx.x >> 5;
    const int nwib = blockDim.x >> 5;
    const int64_t warp = row_begin + static_cast<int64_t>(blockIdx.x) * nwib + wib;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * nwib;
    const int nv = C >> 2;
    float4 aw[kMaxVec], ab[kMaxVec], ad[kMaxVec];
#pragma unroll
    for (int k = 0; k < kMaxVec; ++k) {
        aw[k] = make_float4(0, 0, 0, 0);
        ab[k] = make_float4(0, 0, 0, 0);
        ad[k] = make_float4(0, 0, 0, 0);
    }
    if constexpr (kMaxVec <= 6) {
        // the next row's x / gy / statistics are loaded while the current row is reduced and
        // written, so each warp keeps two rows of loads in flight
        Raw4<T> nx[kMaxVec], ng[kMaxVec];
        float nmean = 0.f, nrstd = 0.f;
        int64_t r = warp;
        if (r < rows) {
            nmean = mean_in[r];
            nrstd = rstd_in[r];
            const T* gr0 = gy_row(r);
#pragma unroll
            for (int k = 0; k < kMaxVec; ++k) {
                const int i = lane + 32 * k;
                if (i < nv) {
                    nx[k].load(x + r * C + 4 * i);
                    if (gr0 != nullptr) ng[k].load(gr0 + 4 * i);
                    else ng[k].zero();
                }
            }
        }
        for (; r < rows; r += nwarps) {
            const float mean = nmean, rstd = nrstd;
            float4 xv[kMaxVec], gv[kMaxVec];
#pragma unroll
            for (int k = 0; k < kMaxVec; ++k) {
                xv[k] = nx[k].widen();
                gv[k] = ng[k].widen();
                if (gy2 != nullptr && lane + 32 * k < nv) {   // gradient of the fused y + pos output
                    const float4 g2 = load4(gy2 + r * C + 4 * (lane + 32 * k));
                    gv[k].x += g2.x; gv[k].y += g2.y; gv[k].z += g2.z; gv[k].w += g2.w;
                }
            }
            const int64_t rn = r + nwarps;
            if (rn < rows) {
                nmean = mean_in[rn];
                nrstd = rstd_in[rn];
                const T* grn = gy_row(rn);
#pragma unroll
                for (int k = 0; k < kMaxVec; ++k) {
                    const int i = lane + 32 * k;
                    if (i < nv) {
                        nx[k].load(x + rn * C + 4 * i);
                        if (grn != nullptr) ng[k].load(grn + 4 * i);
                        else ng[k].zero();
                    }
                }
            }
            ln_bwd_row<T, W, kMaxVec, kBias2>(xv, gv, mean, rstd, w, aw, ab, ad, gx + r * C, lane, nv, C,
                                      gres != nullptr ? gres + r * C : nullptr, bvec, act);
        }
    } else {
        // wide rows have no registers to spare for a second row
        for (int64_t r = warp; r < rows; r += nwarps) {
            float4 xv[kMaxVec], gv[kMaxVec];
            const T* grr = gy_row(r);
#pragma unroll
            for (int k = 0; k < kMaxVec; ++k) {
                const int i = lane + 32 * k;
                if (i < nv) {
                    xv[k] = load4(x + r * C + 4 * i);
                    gv[k] = grr != nullptr ? load4(grr + 4 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
                    if (gy2 != nullptr) {
                        const float4 g2 = load4(gy2 + r * C + 4 * i);
                        gv[k].x += g2.x; gv[k].y += g2.y; gv[k].z += g2.z; gv[k].w += g2.w;
                    }
                }
            }
            ln_bwd_row<T, W, kMaxVec, kBias2>(xv, gv, mean_in[r], rstd_in[r], w, aw, ab, ad, gx + r * C, lane, nv,
                                              C,
                                      gres != nullptr ? gres + r * C : nullptr, bvec, act);
        }
    }
    // CTA reduction of the per-lane column partials ([warps][nacc][C]: gamma, beta[, input])
    constexpr int nacc = kBias2 ? 3 : 2;
    float* sw = smem + wib * nacc * C;
    float* sb = sw + C;
#pragma unroll
    for (int k = 0; k < kMaxVec; ++k) {
        const int i = lane + 32 * k;
        if (i < nv) {
            store4(sw + 4 * i, aw[k]);
            store4(sb + 4 * i, ab[k]);
            if constexpr (kBias2) store4(sb + C + 4 * i, ad[k]);
        }
    }
    __syncthreads();
    // CTA partials go to the fp32 accumulators with 16-byte atomics (resolved in L2); the last
    // CTA to arrive writes (or adds into) gw / gb and clears the scratch for the next launch
    for (int c4 = threadIdx.x; c4 < nv; c4 += blockDim.x) {
        float4 a = make_float4(0, 0, 0, 0), bb = make_float4(0, 0, 0, 0), dd = make_float4(0, 0, 0, 0);
        for (int q = 0; q < nwib; ++q) {
            const float4 pa = *reinterpret_cast<const float4*>(smem + q * nacc * C + 4 * c4);
            const float4 pb = *reinterpret_cast<const float4*>(smem + q * nacc * C + C + 4 * c4);
            a.x += pa.x; a.y += pa.y; a.z += pa.z; a.w += pa.w;
            bb.x += pb.x; bb.y += pb.y; bb.z += pb.z; bb.w += pb.w;
            if constexpr (kBias2) {
                const float4 pd = *reinterpret_cast<const float4*>(smem + q * nacc * C + 2 * C + 4 * c4);
                dd.x += pd.x; dd.y += pd.y; dd.z += pd.z; dd.w += pd.w;
            }
        }
        atomicAdd(reinterpret_cast<float4*>(acc_w + 4 * c4), a);
        atomicAdd(reinterpret_cast<float4*>(acc_b + 4 * c4), bb);
        if constexpr (kBias2) atomicAdd(reinterpret_cast<float4*>(acc_b + C + 4 * c4), dd);
    }
    // arrival (one thread fences after the barrier, as in a grid sync)
    __shared__ unsigned s_last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        s_last = atomicAdd(counter, 1u) == gridDim.x - 1;
        if (s_last) __threadfence();
    }
    __syncthreads();
    if (!s_last) return;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        const float a = __ldcg(acc_w + c), bb = __ldcg(acc_b + c);
        gw[c] = from_f<W>((accumulate ? to_f(gw[c]) : 0.f) + a);
        gb[c] = from_f<W>((accumulate ? to_f(gb[c]) : 0.f) + bb);
        acc_w[c] = 0.f;
        acc_b[c] = 0.f;
        if constexpr (kBias2) {
            const float d = __ldcg(acc_b + C + c);
            gbias2[c] = from_f<W>((accumulate2 ? to_f(gbias2[c]) : 0.f) + d);
            acc_b[C + c] = 0.f;
        }
    }
    if (threadIdx.x == 0) *counter = 0u;
}

template <typename F>
void dispatch_vec(int C, F&& f) {
    const int nvl = (C / 4 + 31) / 32;
    switch (nvl) {
        case 1: return f(std::integral_constant<int, 1>{});
        case 2: return f(std::integral_constant<int, 2>{});
        case 3: return f(std::integral_constant<int, 3>{});
        case 4: return f(std::integral_constant<int, 4>{});
        case 5: case 6: return f(std::integral_constant<int, 6>{});
        case 7: case 8: return f(std::integral_constant<int, 8>{});
        default: return f(std::integral_constant<int, 12>{});
    }
}

}  // namespace

cudaError_t launch_layernorm_fwd(DType xt, DType wt, const void* x, const void* w, const void* b, void* y, float* mean,
                                 float* rstd, int64_t rows, int C, float eps, cudaStream_t st, const void* res,
                                 void* sum, const void* pos, void* y2, const void* rbias, const void* rscale,
                                 const int* ymap, int64_t yld, int64_t wgroup_rows, int act) {
    if ((rbias != nullptr || rscale != nullptr) && res == nullptr) return cudaErrorInvalidValue;
    if ((res == nullptr) != (sum == nullptr) || (pos == nullptr) != (y2 == nullptr)) return cudaErrorInvalidValue;
    if (ymap != nullptr && (pos != nullptr || yld < C || yld % 4 != 0)) return cudaErrorInvalidValue;
    if (rows == 0) return cudaSuccess;
    if (C % 4 != 0 || C > 4 * 32 * 12) return cudaErrorInvalidValue;
    const int threads = 256;
    const int64_t blocks = std::min<int64_t>((rows + 7) / 8, static_cast<int64_t>(num_sms()) * 16);
    return MMLTK_DISPATCH_DT(xt, [&] {
        using T = scalar_t;
        return MMLTK_DISPATCH_DT(wt, [&] {
            using Wt = scalar_t;
            dispatch_vec(C, [&](auto nvl) {
                ln_fwd_kernel<T, Wt, decltype(nvl)::value><<<blocks, threads, 0, st>>>(
                    static_cast<const T*>(x), static_cast<const Wt*>(w), static_cast<const Wt*>(b),
                    static_cast<T*>(y), mean, rstd, rows, C, eps,
                    LnFwdExtra<T, Wt>{static_cast<const T*>(res), static_cast<T*>(sum), static_cast<const T*>(pos),
                                      static_cast<T*>(y2), static_cast<const Wt*>(rbias),
                                      static_cast<const Wt*>(rscale), ymap, yld, wgroup_rows, act});
            });
            return cudaGetLastError();
        });
    });
}

namespace {
// one resident wave: as many CTAs as fit on every SM (registers / shared memory of this
// instantiation), each warp then strides over rows
template <typename K>
int ln_bwd_blocks(K kern, int threads, size_t smem, int64_t rows) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem) != cudaSuccess || per_sm < 1)
        per_sm = 1;
    const int64_t want = static_cast<int64_t>(num_sms()) * per_sm;
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, (rows + threads / 32 - 1) / (threads / 32))));
}
}  // namespace

cudaError_t launch_layernorm_bwd(DType xt, DType wt, const void* gy, const void* x, const void* w, const float* mean,
                                 const float* rstd, void* gx, void* gw, void* gb, int64_t rows, int C,
                                 bool accumulate, cudaStream_t st, const void* gy2, const void* gres, void* gbias2,
                                 bool accumulate2, const int* gmap, int64_t gld, int64_t group_rows, const void* bvec,
                                 int act) {
    if (act != 0 && bvec == nullptr) return cudaErrorInvalidValue;
    if (gmap != nullptr && (gy2 != nullptr || gld < C || gld % 4 != 0)) return cudaErrorInvalidValue;
    const int64_t groups = group_rows > 0 ? (rows + group_rows - 1) / group_rows : 1;
    if (group_rows > 0 && (rows % group_rows != 0 || groups > kMaxCounters || groups > 65535 ||
                           groups * (gbias2 != nullptr ? 3 : 2) * C > kReduceAccFloats))
        return cudaErrorInvalidValue;
    if (C % 4 != 0 || C > 4 * 32 * 12 || 3 * C > kReduceAccFloats) return cudaErrorInvalidValue;
    const ReduceScratch rs = reduce_scratch();
    if (rs.counters == nullptr) return cudaErrorMemoryAllocation;
    const int threads = 256;
    const int nwib = threads / 32;
    const size_t smem = static_cast<size_t>(nwib) * (gbias2 != nullptr ? 3 : 2) * C * sizeof(float);
    return MMLTK_DISPATCH_DT(xt, [&] {
        using T = scalar_t;
        return MMLTK_DISPATCH_DT(wt, [&] {
            using Wt = scalar_t;
            cudaError_t e = cudaSuccess;
            auto run = [&](auto nvl, auto b2) {
                auto kern = ln_bwd_kernel<T, Wt, decltype(nvl)::value, decltype(b2)::value>;
                // the kernel also has a few bytes of static shared memory, so opt in at 48 KB already
                if (smem >= 40 * 1024)
                    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
                if (e != cudaSuccess) return;
                // one resident wave over all groups
                const int blocks = static_cast<int>(std::max<int64_t>(
                    1, std::min<int64_t>(ln_bwd_blocks(kern, threads, smem, rows) / groups, (group_rows > 0 ? group_rows : rows) / 8 + 1)));
                kern<<<dim3(blocks, static_cast<unsigned>(groups)), threads, smem, st>>>(static_cast<const T*>(gy), static_cast<const T*>(x),
                                                    static_cast<const Wt*>(w), mean, rstd, static_cast<T*>(gx), rs.acc,
                                                    rs.acc + C, rs.counters, static_cast<Wt*>(gw),
                                                    static_cast<Wt*>(gb), accumulate ? 1 : 0, rows, C,
                                                    static_cast<const T*>(gy2), static_cast<const T*>(gres),
                                                    static_cast<Wt*>(gbias2), accumulate2 ? 1 : 0, gmap, gld,
                                                    group_rows, static_cast<const Wt*>(bvec), act);
            };
            dispatch_vec(C, [&](auto nvl) {
                if (gbias2 != nullptr) run(nvl, std::true_type{});
                else run(nvl, std::false_type{});
            });
            if (e != cudaSuccess) return e;
            return cudaGetLastError();
        });
    });
}

}  // namespace mmltk
