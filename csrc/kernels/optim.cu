// Fused optimizer step over the flat parameter / gradient buffers:
//   kernel 1  per-CTA partial sum of squares of the bf16 gradients + non-finite flag
//   kernel 2  every CTA reduces the partials (global L2 norm, clip coefficient
//             min(1, max_norm / (norm + 1e-6))), then applies decoupled-weight-decay
//             AdamW to the fp32 master weights, writes the bf16 working copy and
//             updates the fp32 EMA shadow -- one pass over memory.
//
// Reference: `clip_grad_norm_(0.1)` + `at::_fused_adamw_` + ModelEma
// `_foreach_mul_/_foreach_add_` (`src/rfdetr/training/train.cpp:2287-2344`,
// `src/rfdetr/training/native_optimizer.cpp:374-419`,
// `include/mmltk/rfdetr/training_ops.h:177-229`).
//
// Per-step scalars (lr scale, bias corrections, EMA decay) come from a device
// struct that the host refreshes with one async copy, so the whole step can be
// replayed from a CUDA graph.  A non-finite gradient norm skips the update and
// raises a device flag the host checks at its once-per-step sync.
#include <algorithm>

#include "common.cuh"
#include "optim.cuh"

namespace mmltk {

namespace {

__global__ void __launch_bounds__(256) grad_sumsq_kernel(const __nv_bfloat16* __restrict__ g, int64_t n,
                                                         float* __restrict__ partials) {
    __shared__ float red[8];
    float s = 0.f;
    const int64_t n8 = n / 8;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float v[8];
        load8(g + 8 * i, v);
#pragma unroll
        for (int c = 0; c < 8; ++c) s += v[c] * v[c];
    }
    if (blockIdx.x == 0)
        for (int64_t i = n8 * 8 + threadIdx.x; i < n; i += blockDim.x) {
            const float v = __bfloat162float(g[i]);
            s += v * v;
        }
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) partials[blockIdx.x] = t;  // inf/nan propagate
    }
}

__device__ float reduce_partials(const float* partials, int nparts, float* red) {
    float s = 0.f;
    for (int i = threadIdx.x; i < nparts; i += blockDim.x) s += partials[i];
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float total = red[0];
    __syncthreads();
    return total;
}

__global__ void __launch_bounds__(256) adamw_ema_kernel(const ChunkDesc* __restrict__ chunks, int nchunks,
                                                        const __nv_bfloat16* __restrict__ grad,
                                                        float* __restrict__ master, float* __restrict__ m,
                                                        float* __restrict__ v, float* __restrict__ ema,
                                                        __nv_bfloat16* __restrict__ param,
                                                        const GroupHyper* __restrict__ groups,
                                                        const StepScalars* __restrict__ sc,
                                                        const float* __restrict__ partials, int nparts,
                                                        int* __restrict__ flags) {
    __shared__ float red[8];
    const float sumsq = reduce_partials(partials, nparts, red);
    // gradients arrive summed over ranks: the norm of the average is sqrt(sumsq) / world
    const float inv_world = sc->inv_world > 0.f ? sc->inv_world : 1.f;
    const float norm = sqrtf(sumsq) * inv_world;
    if (!isfinite(norm)) {
        if (blockIdx.x == 0 && threadIdx.x == 0) flags[0] = 1;
        return;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) reinterpret_cast<float*>(flags)[1] = norm;
    float clip = 1.f;
    if (sc->max_norm > 0.f) clip = fminf(1.f, sc->max_norm / (norm + 1e-6f));
    const float b1 = sc->beta1, b2 = sc->beta2, eps = sc->eps;
    const float inv_bc1 = 1.f / sc->bias_corr1, inv_sqrt_bc2 = rsqrtf(sc->bias_corr2);
    const float ema_d = sc->ema_decay;
    const bool do_ema = ema != nullptr && sc->ema_enabled;
    for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
        const ChunkDesc cd = chunks[c];
        const GroupHyper gh = groups[cd.group];
        const float lr = gh.lr * sc->lr_scale;
        const float decay = 1.f - lr * gh.weight_decay;
        for (int64_t i = cd.offset + 4 * threadIdx.x; i < cd.offset + cd.length; i += 4 * blockDim.x) {
            // every operand of this element group is loaded before any is used (one memory
            // round trip per iteration, the EMA included)
            const float4 gg = load4(grad + i);
            float4 p = *reinterpret_cast<float4*>(master + i);
            float4 mm = *reinterpret_cast<float4*>(m + i);
            float4 vv = *reinterpret_cast<float4*>(v + i);
            float4 e = do_ema ? *reinterpret_cast<const float4*>(ema + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            const float gs = clip * inv_world;
            float gv[4] = {gg.x * gs, gg.y * gs, gg.z * gs, gg.w * gs};
            float* pp = &p.x;
            float* mp = &mm.x;
            float* vp = &vv.x;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                mp[k] = b1 * mp[k] + (1.f - b1) * gv[k];
                vp[k] = b2 * vp[k] + (1.f - b2) * gv[k] * gv[k];
                const float denom = sqrtf(vp[k]) * inv_sqrt_bc2 + eps;
                pp[k] = pp[k] * decay - lr * inv_bc1 * mp[k] / denom;
            }
            *reinterpret_cast<float4*>(master + i) = p;
            *reinterpret_cast<float4*>(m + i) = mm;
            *reinterpret_cast<float4*>(v + i) = vv;
            store4(param + i, p);
            if (do_ema) {
                e.x = ema_d * e.x + (1.f - ema_d) * p.x;
                e.y = ema_d * e.y + (1.f - ema_d) * p.y;
                e.z = ema_d * e.z + (1.f - ema_d) * p.z;
                e.w = ema_d * e.w + (1.f - ema_d) * p.w;
                *reinterpret_cast<float4*>(ema + i) = e;
            }
        }
    }
}

}  // namespace

int optim_num_partials() { return num_sms() * 2; }

void launch_grad_sumsq(const __nv_bfloat16* grad, int64_t n, float* partials, int nparts, cudaStream_t st) {
    grad_sumsq_kernel<<<nparts, 256, 0, st>>>(grad, n, partials);
}

void launch_adamw_ema(const ChunkDesc* chunks, int nchunks, const __nv_bfloat16* grad, float* master, float* m,
                      float* v, float* ema, __nv_bfloat16* param, const GroupHyper* groups, const StepScalars* sc,
                      const float* partials, int nparts, int* flags, cudaStream_t st) {
    // one resident wave; blocks stride over the (small) chunks, which balances the work
    static int per_sm = 0;
    if (per_sm == 0 && (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, adamw_ema_kernel, 256, 0) !=
                            cudaSuccess || per_sm < 1))
        per_sm = 2;
    const int blocks = std::min(nchunks, num_sms() * per_sm);
    if (blocks <= 0) return;
    adamw_ema_kernel<<<blocks, 256, 0, st>>>(chunks, nchunks, grad, master, m, v, ema, param, groups, sc, partials,
                                             nparts, flags);
}

}  // namespace mmltk
