// Hungarian matcher on the device: cost matrix for every supervised layer in
// one launch, then a batched shortest-augmenting-path LSAP solver with one
// warp per (layer, image, Group-DETR group) problem.
//
// Reference: `matcher_cost_kernel` (`src/rfdetr/cuda/detr_ops_cuda.cu:117-152`)
// builds one layer's [B,Q,maxT] cost; the costs are then copied to the host
// and solved per (layer, image, group) on a CPU thread pool
// (`src/rfdetr/detection_ops.cpp:1138-1279`).  Here nothing leaves the GPU:
// the solver writes a [NL, B, G, T] int32 table of matched query indices that
// the loss kernels consume directly, so the training step has no host sync
// and can be captured in a CUDA graph.
//
// The solver runs the same algorithm as the CPU oracle (csrc/host/lsap.cpp)
// in fp64, including the column scan order and the tie rule, so both return
// identical assignments.
#include "common.cuh"

namespace mmltk {

namespace {

__device__ __forceinline__ float softplus_f(float x) {
    // log(1 + exp(x)) without overflow
    return fmaxf(x, 0.f) + log1pf(__expf(-fabsf(x)));
}

__device__ __forceinline__ float giou_cxcywh(const float* a, const float* b) {
    const float ax1 = a[0] - 0.5f * a[2], ay1 = a[1] - 0.5f * a[3], ax2 = a[0] + 0.5f * a[2],
                ay2 = a[1] + 0.5f * a[3];
    const float bx1 = b[0] - 0.5f * b[2], by1 = b[1] - 0.5f * b[3], bx2 = b[0] + 0.5f * b[2],
                by2 = b[1] + 0.5f * b[3];
    const float iw = fmaxf(0.f, fminf(ax2, bx2) - fmaxf(ax1, bx1));
    const float ih = fmaxf(0.f, fminf(ay2, by2) - fmaxf(ay1, by1));
    const float inter = iw * ih;
    const float area_a = fmaxf(0.f, ax2 - ax1) * fmaxf(0.f, ay2 - ay1);
    const float area_b = fmaxf(0.f, bx2 - bx1) * fmaxf(0.f, by2 - by1);
    const float uni = area_a + area_b - inter;
    const float ew = fmaxf(ax2, bx2) - fminf(ax1, bx1), eh = fmaxf(ay2, by2) - fminf(ay1, by1);
    const float encl = fmaxf(0.f, ew) * fmaxf(0.f, eh);
    return inter / uni - (encl - uni) / encl;
}

// One CTA per (layer, image, query tile of 128); targets of the image in shared memory.
template <typename TL, typename TB>
__global__ void __launch_bounds__(128) matcher_cost_kernel(MatcherLayers lp, const int64_t* __restrict__ labels,
                                                          const float* __restrict__ tboxes,
                                                          const int32_t* __restrict__ counts, float* __restrict__ cost,
                                                          int B, int Q, int C, int T, float w_class, float w_bbox,
                                                          float w_giou, float alpha) {
    extern __shared__ float sm[];
    float* sbox = sm;                                         // [T,4]
    int* slab = reinterpret_cast<int*>(sm + 4 * T);           // [T]
    const int qtiles = (Q + blockDim.x - 1) / blockDim.x;
    const int tile = blockIdx.x % qtiles;
    const int b = (blockIdx.x / qtiles) % B;
    const int l = blockIdx.x / (qtiles * B);
    MMLTK_DEBUG_CHECK(counts[b] <= T, kDbgMatcherCount);
    const int nt = min(counts[b], T);
    for (int i = threadIdx.x; i < nt * 4; i += blockDim.x) sbox[i] = tboxes[static_cast<int64_t>(b) * T * 4 + i];
    for (int i = threadIdx.x; i < nt; i += blockDim.x) {
        const int64_t lab = labels[static_cast<int64_t>(b) * T + i];
        MMLTK_DEBUG_CHECK(lab >= 0 && lab < C, kDbgMatcherLabel);
        slab[i] = static_cast<int>(lab < 0 ? 0 : (lab >= C ? C - 1 : lab));  // labels are validated on the host
    }
    __syncthreads();
    const int q = tile * blockDim.x + threadIdx.x;
    if (q >= Q) return;
    const TL* lg = reinterpret_cast<const TL*>(lp.logits[l]) + (static_cast<int64_t>(b) * Q + q) * C;
    const TB* bx = reinterpret_cast<const TB*>(lp.boxes[l]) + (static_cast<int64_t>(b) * Q + q) * 4;
    const float pb[4] = {to_f(bx[0]), to_f(bx[1]), to_f(bx[2]), to_f(bx[3])};
    float* out = cost + ((static_cast<int64_t>(l) * B + b) * Q + q) * T;
    for (int t = 0; t < T; ++t) {
        if (t >= nt) {
            out[t] = 0.f;
            continue;
        }
        const float x = to_f(lg[slab[t]]);
        const float p = 1.f / (1.f + __expf(-x));
        const float pos = alpha * (1.f - p) * (1.f - p) * softplus_f(-x);
        const float neg = (1.f - alpha) * p * p * softplus_f(x);
        const float* tb = sbox + 4 * t;
        const float l1 = fabsf(pb[0] - tb[0]) + fabsf(pb[1] - tb[1]) + fabsf(pb[2] - tb[2]) + fabsf(pb[3] - tb[3]);
        out[t] = w_class * (pos - neg) + w_bbox * l1 - w_giou * giou_cxcywh(pb, tb);
    }
}

// ---------------------------------------------------------------- LSAP
// Problem (l, b, g) over the nt targets of image b and the Qg queries of group g, cost
// cost[l, b, g*Qg + q, t].  Rows are the shorter side: the targets when nt <= Qg, the queries
// otherwise (scipy's rectangular_lsap transposes the same way).  All state lives in shared
// memory; the kernel carves every array with max(Qg, T) entries.
struct LsapSmem {
    double* u;     // [rows]
    double* v;     // [cols]
    double* spc;   // [cols]
    int* path;     // [cols]
    int* row4col;  // [cols]
    int* rem;      // [cols]
    int* col4row;  // [rows]
    unsigned char* sr;  // [rows]
    unsigned char* sc;  // [cols]
};

__host__ __device__ inline size_t lsap_smem_bytes(int Qg, int T) {
    size_t b = 0;
    b += sizeof(double) * (T + 2 * static_cast<size_t>(Qg));
    b += sizeof(int) * (3 * static_cast<size_t>(Qg) + T);
    b += T + Qg;
    return (b + 15) & ~static_cast<size_t>(15);
}

__device__ inline LsapSmem lsap_carve(char* base, int Qg, int T) {
    LsapSmem s;
    s.u = reinterpret_cast<double*>(base);
    s.v = s.u + T;
    s.spc = s.v + Qg;
    s.path = reinterpret_cast<int*>(s.spc + Qg);
    s.row4col = s.path + Qg;
    s.rem = s.row4col + Qg;
    s.col4row = s.rem + Qg;
    s.sr = reinterpret_cast<unsigned char*>(s.col4row + T);
    s.sc = s.sr + T;
    return s;
}

// Key for the warp arg-min that reproduces the sequential scan: the minimum
// value wins; among equal values an unassigned column wins, the last such in
// scan order; among equal assigned columns the first in scan order.
__device__ __forceinline__ bool better(double va, int ua, int ia, double vb, int ub, int ib) {
    if (va != vb) return va < vb;
    if (ua != ub) return ua > ub;
    if (ua) return ia > ib;
    return ia < ib;
}

__global__ void __launch_bounds__(128) lsap_kernel(const float* __restrict__ cost, const int32_t* __restrict__ counts,
                                                  int32_t* __restrict__ match, int NL, int B, int G, int Qg, int T,
                                                  int* __restrict__ status) {
    extern __shared__ __align__(16) char lsm[];
    const int lane = threadIdx.x & 31;
    const int wib = threadIdx.x >> 5;
    const int wpb = blockDim.x >> 5;
    const int prob = blockIdx.x * wpb + wib;
    if (prob >= NL * B * G) return;
    const int g = prob % G;
    const int b = (prob / G) % B;
    const int l = prob / (G * B);
    const int Q = Qg * G;
    const int M = Qg > T ? Qg : T;   // every per-row / per-column array holds max(Qg, T) entries
    LsapSmem s = lsap_carve(lsm + static_cast<size_t>(wib) * lsap_smem_bytes(M, M), M, M);
    int32_t* out = match + ((static_cast<int64_t>(l) * B + b) * G + g) * T;
    for (int t = lane; t < T; t += 32) out[t] = -1;
    const int nt = min(counts[b], T);
    if (nt <= 0) return;
    // rows are the shorter side (scipy's rectangular LSAP): targets when nt <= Qg (each target gets a
    // query), queries otherwise (each query gets a target, nt - Qg targets stay unmatched)
    const bool tr = nt > Qg;
    const int nr = tr ? Qg : nt, nc = tr ? nt : Qg;
    const float* cbase = cost + ((static_cast<int64_t>(l) * B + b) * Q + static_cast<int64_t>(g) * Qg) * T;
    // sanitize: non-finite -> max finite + max |finite| + 1 (as the host solver)
    double fmax = -INFINITY, amax = 0.0;
    int bad = 0;
    for (int idx = lane; idx < nt * Qg; idx += 32) {
        const int q = idx / nt, t = idx % nt;
        const double c = cbase[static_cast<int64_t>(q) * T + t];
        if (isfinite(c)) {
            fmax = fmax > c ? fmax : c;
            amax = amax > fabs(c) ? amax : fabs(c);
        } else {
            bad = 1;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        // every lane executes every shuffle exactly once (a shuffle inside a
        // conditional expression would desynchronise the warp)
        const double of = __shfl_xor_sync(0xffffffffu, fmax, o);
        const double oa = __shfl_xor_sync(0xffffffffu, amax, o);
        const int ob = __shfl_xor_sync(0xffffffffu, bad, o);
        fmax = fmax > of ? fmax : of;
        amax = amax > oa ? amax : oa;
        bad |= ob;
    }
    const double flt_max = 3.4028234663852886e38;
    double rep = flt_max;
    if (fmax > -INFINITY) {
        const double cand = fmax + amax + 1.0;
        if (isfinite(cand)) rep = cand < rep ? cand : rep;
    }
    auto C = [&](int r, int col) -> double {
        const int q = tr ? r : col, t = tr ? col : r;
        const double c = cbase[static_cast<int64_t>(q) * T + t];
        return (bad && !isfinite(c)) ? rep : c;
    };

    for (int r = lane; r < nr; r += 32) {
        s.u[r] = 0.0;
        s.col4row[r] = -1;
    }
    for (int c = lane; c < nc; c += 32) {
        s.v[c] = 0.0;
        s.row4col[c] = -1;
        s.path[c] = -1;
    }
    __syncwarp();
    constexpr int kMaxSteps = 1 << 20;  // bound on the inner search (never reached by a valid problem)
    for (int cur = 0; cur < nr; ++cur) {
        for (int r = lane; r < nr; r += 32) s.sr[r] = 0;
        for (int c = lane; c < nc; c += 32) {
            s.sc[c] = 0;
            s.spc[c] = INFINITY;
            s.rem[c] = nc - 1 - c;
        }
        __syncwarp();
        int n_rem = nc;
        double min_val = 0.0;
        int i = cur;
        int sink = -1;
        int steps = 0;
        while (sink < 0) {
            if (++steps > kMaxSteps) {
                if (lane == 0) atomicExch(status, 1);
                return;
            }
            if (lane == 0) s.sr[i] = 1;
            const double ui = s.u[i];
            double best_v = INFINITY;
            int best_u = 0, best_it = 0x7fffffff;
            bool have = false;
            for (int it = lane; it < n_rem; it += 32) {
                const int j = s.rem[it];
                const double r = min_val + C(i, j) - ui - s.v[j];
                if (r < s.spc[j]) {
                    s.path[j] = i;
                    s.spc[j] = r;
                }
                const double sv = s.spc[j];
                const int un = s.row4col[j] < 0 ? 1 : 0;
                if (!have || better(sv, un, it, best_v, best_u, best_it)) {
                    best_v = sv;
                    best_u = un;
                    best_it = it;
                    have = true;
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const double ov = __shfl_xor_sync(0xffffffffu, best_v, o);
                const int ou = __shfl_xor_sync(0xffffffffu, best_u, o);
                const int oi = __shfl_xor_sync(0xffffffffu, best_it, o);
                const int oh = __shfl_xor_sync(0xffffffffu, have ? 1 : 0, o);
                if (oh && (!have || better(ov, ou, oi, best_v, best_u, best_it))) {
                    best_v = ov;
                    best_u = ou;
                    best_it = oi;
                    have = true;
                }
            }
            __syncwarp();
            min_val = best_v;
            if (!(min_val < INFINITY)) {
                if (lane == 0) atomicExch(status, 2);
                return;
            }
            if (best_it < 0 || best_it >= n_rem) {  // self-check: record and stop, never touch memory
                if (lane == 0) atomicExch(status, 3);
                return;
            }
            const int j = s.rem[best_it];
            if (j < 0 || j >= nc) {
                if (lane == 0) atomicExch(status, 4);
                return;
            }
            if (s.row4col[j] < 0) {
                sink = j;
            } else {
                i = s.row4col[j];
                if (i < 0 || i >= nr) {
                    if (lane == 0) atomicExch(status, 5);
                    return;
                }
            }
            __syncwarp();
            if (lane == 0) {
                s.sc[j] = 1;
                s.rem[best_it] = s.rem[n_rem - 1];
            }
            --n_rem;
            __syncwarp();
        }
        // dual updates
        if (lane == 0) s.u[cur] += min_val;
        for (int r = lane; r < nr; r += 32)
            if (s.sr[r] && r != cur) {
                const int c4 = s.col4row[r];
                if (c4 < 0 || c4 >= nc) {
                    atomicExch(status, 8);
                    continue;
                }
                s.u[r] += min_val - s.spc[c4];
            }
        for (int c = lane; c < nc; c += 32)
            if (s.sc[c]) s.v[c] -= min_val - s.spc[c];
        __syncwarp();
        if (lane == 0) {
            int j = sink;
            for (int guard = 0; guard <= nr; ++guard) {
                if (j < 0 || j >= nc) {
                    atomicExch(status, 6);
                    break;
                }
                const int r = s.path[j];
                if (r < 0 || r >= nr) {
                    atomicExch(status, 7);
                    break;
                }
                s.row4col[j] = r;
                const int prev = s.col4row[r];
                s.col4row[r] = j;
                j = prev;
                if (r == cur) break;
            }
        }
        __syncwarp();
    }
    if (!tr) {
        for (int t = lane; t < nt; t += 32) {
            const int q = s.col4row[t];
            out[t] = q >= 0 ? g * Qg + q : -1;
        }
    } else {
        for (int q = lane; q < nr; q += 32) {
            const int t = s.col4row[q];
            if (t >= 0 && t < nt) out[t] = g * Qg + q;
        }
    }
}

}  // namespace

cudaError_t launch_matcher_cost(DType lt, DType bt, MatcherLayers lp, int NL, const int64_t* labels,
                                const float* tboxes, const int32_t* counts, float* cost, int B, int Q, int C, int T,
                                float w_class, float w_bbox, float w_giou, float alpha, cudaStream_t st) {
    if (NL < 1 || NL > kMatcherMaxLayers) return cudaErrorInvalidValue;
    if (T == 0 || Q == 0 || B == 0) return cudaSuccess;
    const int threads = 128;
    const int qtiles = (Q + threads - 1) / threads;
    const size_t smem = static_cast<size_t>(T) * 5 * sizeof(float);
    return MMLTK_DISPATCH_DT(lt, [&] {
        using TL = scalar_t;
        return MMLTK_DISPATCH_DT(bt, [&] {
            using TB = scalar_t;
            matcher_cost_kernel<TL, TB><<<NL * B * qtiles, threads, smem, st>>>(
                lp, labels, tboxes, counts, cost, B, Q, C, T, w_class, w_bbox, w_giou, alpha);
            return cudaGetLastError();
        });
    });
}

// every array of a problem is sized max(Qg, T): rows and columns swap when T > Qg
size_t lsap_shared_bytes(int Qg, int T, int warps_per_block) {
    const int M = std::max(Qg, T);
    return lsap_smem_bytes(M, M) * warps_per_block;
}

int lsap_warps_per_block(int Qg, int T) {
    const int M = std::max(Qg, T);
    int wpb = 4;
    while (wpb > 1 && lsap_smem_bytes(M, M) * wpb > 200 * 1024) wpb >>= 1;
    return wpb;
}

cudaError_t launch_lsap(const float* cost, const int32_t* counts, int32_t* match, int NL, int B, int G, int Qg, int T,
                        int* status, cudaStream_t st) {
    const int problems = NL * B * G;
    if (problems == 0 || T == 0) return cudaSuccess;
    const int wpb = lsap_warps_per_block(Qg, T);
    const size_t smem = lsap_shared_bytes(Qg, T, wpb);
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(lsap_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    lsap_kernel<<<(problems + wpb - 1) / wpb, 32 * wpb, smem, st>>>(cost, counts, match, NL, B, G, Qg, T, status);
    return cudaGetLastError();
}

MMLTK_DEBUG_STATUS_TU(matcher)

}  // namespace mmltk
