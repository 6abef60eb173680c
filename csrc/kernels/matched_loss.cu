// Fused matched-pair losses of every supervised layer: one launch forward,
// one launch backward, reading the layers' logits / boxes in place.
//
// For each (layer, image, group, target slot) with a match (query q): the L1
// and GIoU box losses between prediction q and the target box (cxcywh), and the
// classification correction of the matched logit x = logits[b, q, label] --
// IA-BCE (target t = clamp(sigmoid(x)^alpha * IoU^(1-alpha), 0.01), no gradient
// through t) or sigmoid focal -- relative to the dense "every logit is a
// negative" term computed over all logits by the dense loss kernel.  Per-layer
// sums: out[l] = (correction, L1, 1 - GIoU).  The backward kernel adds the
// matched logit gradients into the dense-term gradient tensors and writes the
// box gradients (the box-gradient tensors arrive zeroed); a query is matched at
// most once per layer, so the scattered updates never collide.  Reference
// formulas: `src/rfdetr/detection_ops.cpp:1303-1392`.  The per-element torch
// statement of the same terms launches ~60 small kernels per layer each way.
#include "common.cuh"

namespace mmltk {

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + __expf(-x)); }
__device__ __forceinline__ float softplusf_(float x) { return fmaxf(x, 0.f) + log1pf(__expf(-fabsf(x))); }

struct BoxTerms {
    float l1, giou_loss, iou;
    float g[4];   // d(1 - giou)/d(cx, cy, w, h)
};

// s, t: cxcywh
__device__ __forceinline__ BoxTerms box_terms(const float* s, const float* t, bool want_grad) {
    BoxTerms r;
    const float x0 = s[0] - 0.5f * s[2], x1 = s[0] + 0.5f * s[2];
    const float y0 = s[1] - 0.5f * s[3], y1 = s[1] + 0.5f * s[3];
    const float a0 = t[0] - 0.5f * t[2], a1 = t[0] + 0.5f * t[2];
    const float b0 = t[1] - 0.5f * t[3], b1 = t[1] + 0.5f * t[3];
    r.l1 = fabsf(s[0] - t[0]) + fabsf(s[1] - t[1]) + fabsf(s[2] - t[2]) + fabsf(s[3] - t[3]);
    const float sw = x1 - x0, sh = y1 - y0;
    const float area_s = fmaxf(sw, 0.f) * fmaxf(sh, 0.f);
    const float area_t = fmaxf(a1 - a0, 0.f) * fmaxf(b1 - b0, 0.f);
    const float ix0 = fmaxf(x0, a0), ix1 = fminf(x1, a1), iy0 = fmaxf(y0, b0), iy1 = fminf(y1, b1);
    const float iw = fmaxf(ix1 - ix0, 0.f), ih = fmaxf(iy1 - iy0, 0.f);
    const float inter = iw * ih;
    const float uni = area_s + area_t - inter;
    const float iou = inter / uni;
    const float ex0 = fminf(x0, a0), ex1 = fmaxf(x1, a1), ey0 = fminf(y0, b0), ey1 = fmaxf(y1, b1);
    const float cw = fmaxf(ex1 - ex0, 0.f), ch = fmaxf(ey1 - ey0, 0.f);
    const float area_c = cw * ch;
    r.iou = iou;
    r.giou_loss = 1.f - (iou - (area_c - uni) / area_c);
    if (!want_grad) return r;
    // partials w.r.t. (x0, x1, y0, y1)
    const bool on = ix1 - ix0 > 0.f && iy1 - iy0 > 0.f;
    const float d_inter[4] = {(on && x0 > a0) ? -ih : 0.f, (on && x1 < a1) ? ih : 0.f, (on && y0 > b0) ? -iw : 0.f,
                              (on && y1 < b1) ? iw : 0.f};
    const float hs = fmaxf(sh, 0.f), ws = fmaxf(sw, 0.f);
    const float d_area_s[4] = {sw > 0.f ? -hs : 0.f, sw > 0.f ? hs : 0.f, sh > 0.f ? -ws : 0.f,
                               sh > 0.f ? ws : 0.f};
    const bool cw_on = ex1 - ex0 > 0.f, ch_on = ey1 - ey0 > 0.f;
    const float d_area_c[4] = {(cw_on && x0 < a0) ? -ch : 0.f, (cw_on && x1 > a1) ? ch : 0.f,
                               (ch_on && y0 < b0) ? -cw : 0.f, (ch_on && y1 > b1) ? cw : 0.f};
    float dl[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float d_uni = d_area_s[k] - d_inter[k];
        const float d_iou = (d_inter[k] * uni - inter * d_uni) / (uni * uni);
        const float d_ratio = (d_uni * area_c - uni * d_area_c[k]) / (area_c * area_c);  // d(union / area_c)
        dl[k] = -(d_iou + d_ratio);                                                       // giou = iou - 1 + union/area_c
    }
    r.g[0] = dl[0] + dl[1];
    r.g[1] = dl[2] + dl[3];
    r.g[2] = 0.5f * (dl[1] - dl[0]);
    r.g[3] = 0.5f * (dl[3] - dl[2]);
    return r;
}

__device__ __forceinline__ float sgn(float v) { return v > 0.f ? 1.f : (v < 0.f ? -1.f : 0.f); }

// mode 0: IA-BCE correction; 1: sigmoid focal (pos - neg).  dx: derivative w.r.t. x.
__device__ __forceinline__ float ce_term(float x, float iou, int mode, float alpha, float* dx) {
    const float p = sigmoidf_(x);
    const float spx = softplusf_(x), spn = softplusf_(-x);
    if (mode == 0) {
        const float t = fmaxf(powf(p, alpha) * powf(fmaxf(iou, 0.f), 1.f - alpha), 0.01f);
        if (dx) *dx = p - t - 2.f * p * p * (1.f - p) * spx - p * p * p;
        return (1.f - t) * x + spn - p * p * spx;
    }
    const float q = 1.f - p;
    if (dx) *dx = alpha * (-q * q * q - 2.f * p * q * q * spn) - (1.f - alpha) * (2.f * p * p * q * spx + p * p * p);
    return alpha * spn * q * q - (1.f - alpha) * p * p * spx;
}

struct Elem {
    bool valid;
    int64_t logit_off, box_off;
    float s[4], t[4];
};

template <typename LT, typename BT>
__device__ __forceinline__ Elem load_elem(const MatchedLayers& L, int l, int i, const int32_t* match,
                                          const float* tgt, const int64_t* labels, int per_layer, int GT, int T,
                                          int Q, int C) {
    Elem e;
    const int32_t q = match[static_cast<int64_t>(l) * per_layer + i];
    e.valid = q >= 0;
    if (!e.valid) return e;
    const int b = i / GT, t = i % T;
    int64_t lab = labels[static_cast<int64_t>(b) * T + t];
    MMLTK_DEBUG_CHECK(lab >= 0 && lab < C, kDbgLossLabel);
#if defined(MMLTK_DEBUG_BOUNDS) && MMLTK_DEBUG_BOUNDS
    if (q >= Q) {   // the debug build skips a matched query index past the predictions
        debug_flag(kDbgLossQuery);
        e.valid = false;
        return e;
    }
#endif
    lab = lab < 0 ? 0 : (lab >= C ? C - 1 : lab);
    e.logit_off = (static_cast<int64_t>(b) * Q + q) * C + lab;
    e.box_off = (static_cast<int64_t>(b) * Q + q) * 4;
    const BT* bx = static_cast<const BT*>(L.boxes[l]) + e.box_off;
    const float* tb = tgt + 4 * (static_cast<int64_t>(b) * T + t);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        e.s[k] = to_f(bx[k]);
        e.t[k] = tb[k];
    }
    return e;
}

template <typename LT, typename BT>
__global__ void __launch_bounds__(kThreads) matched_fwd_kernel(MatchedLayers L, const int32_t* __restrict__ match,
                                                               const float* __restrict__ tgt,
                                                               const int64_t* __restrict__ labels, int per_layer,
                                                               int GT, int T, int Q, int C, int mode, float alpha,
                                                               float* __restrict__ out) {
    const int l = blockIdx.y;
    const int i = blockIdx.x * kThreads + threadIdx.x;
    float ce = 0.f, l1 = 0.f, gl = 0.f;
    if (i < per_layer) {
        const Elem e = load_elem<LT, BT>(L, l, i, match, tgt, labels, per_layer, GT, T, Q, C);
        if (e.valid) {
            const BoxTerms bt = box_terms(e.s, e.t, false);
            l1 = bt.l1;
            gl = bt.giou_loss;
            ce = ce_term(to_f(static_cast<const LT*>(L.logits[l])[e.logit_off]), bt.iou, mode, alpha, nullptr);
        }
    }
    ce = warp_sum(ce);
    l1 = warp_sum(l1);
    gl = warp_sum(gl);
    __shared__ float red[3][kThreads / 32];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        red[0][w] = ce;
        red[1][w] = l1;
        red[2][w] = gl;
    }
    __syncthreads();
    if (threadIdx.x < 3) {
        float s = 0.f;
        for (int q = 0; q < kThreads / 32; ++q) s += red[threadIdx.x][q];
        atomicAdd(out + 3 * l + threadIdx.x, s);
    }
}

template <typename LT, typename BT>
__global__ void __launch_bounds__(kThreads) matched_bwd_kernel(MatchedLayers L, const int32_t* __restrict__ match,
                                                               const float* __restrict__ tgt,
                                                               const int64_t* __restrict__ labels,
                                                               const float* __restrict__ gout, int per_layer, int GT,
                                                               int T, int Q, int C, int mode, float alpha) {
    const int l = blockIdx.y;
    const int i = blockIdx.x * kThreads + threadIdx.x;
    if (i >= per_layer) return;
    const Elem e = load_elem<LT, BT>(L, l, i, match, tgt, labels, per_layer, GT, T, Q, C);
    if (!e.valid) return;
    const BoxTerms bt = box_terms(e.s, e.t, true);
    float dx = 0.f;
    ce_term(to_f(static_cast<const LT*>(L.logits[l])[e.logit_off]), bt.iou, mode, alpha, &dx);
    const float g_ce = gout[3 * l], g_l1 = gout[3 * l + 1], g_gi = gout[3 * l + 2];
    LT* gl = static_cast<LT*>(L.glogits[l]) + e.logit_off;
    *gl = from_f<LT>(to_f(*gl) + g_ce * dx);                 // unique (b, q) per layer: no collision
    BT* gb = static_cast<BT*>(L.gboxes[l]) + e.box_off;
#pragma unroll
    for (int k = 0; k < 4; ++k) gb[k] = from_f<BT>(to_f(gb[k]) + g_l1 * sgn(e.s[k] - e.t[k]) + g_gi * bt.g[k]);
}

}  // namespace

cudaError_t launch_matched_loss(bool backward, DType lt, DType bt, const MatchedLayers& L, int NL, int B, int Q,
                                int C, int G, int T, const int32_t* match, const float* tgt, const int64_t* labels,
                                int mode, float alpha, float* out_or_gout, cudaStream_t st) {
    const int per_layer = B * G * T;
    if (per_layer == 0 || NL == 0) return cudaSuccess;
    if (NL > kMatchedMaxLayers) return cudaErrorInvalidValue;
    const dim3 grid((per_layer + kThreads - 1) / kThreads, NL);
#define MMLTK_ML(LT_, BT_)                                                                                       \
    do {                                                                                                         \
        if (backward)                                                                                            \
            matched_bwd_kernel<LT_, BT_><<<grid, kThreads, 0, st>>>(L, match, tgt, labels, out_or_gout,         \
                                                                    per_layer, G * T, T, Q, C, mode, alpha);     \
        else                                                                                                     \
            matched_fwd_kernel<LT_, BT_><<<grid, kThreads, 0, st>>>(L, match, tgt, labels, per_layer, G * T, T, \
                                                                    Q, C, mode, alpha, out_or_gout);             \
    } while (0)
    if (lt == DType::kBF16 && bt == DType::kBF16) MMLTK_ML(__nv_bfloat16, __nv_bfloat16);
    else if (lt == DType::kBF16) MMLTK_ML(__nv_bfloat16, float);
    else if (bt == DType::kBF16) MMLTK_ML(float, __nv_bfloat16);
    else MMLTK_ML(float, float);
#undef MMLTK_ML
    return cudaGetLastError();
}

MMLTK_DEBUG_STATUS_TU(matched_loss)

}  // namespace mmltk
