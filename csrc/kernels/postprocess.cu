// Fused detection post-process (sm_100a): per image, top-k over the flattened
// [Q * C] class logits, then labels / query indices, sigmoid scores and the
// selected boxes converted cxcywh -> xyxy (w, h clamped at 0) and scaled to
// pixels -- one launch instead of the reference's sigmoid, topk, two integer
// ops, box conversion, gather and scale (`src/rfdetr/inference/postprocess.cpp:19-238`).
//
// One CTA (1024 threads) per image:
//  1. radix select of the k-th largest logit on order-preserving uint32 keys,
//     four 8-bit digit passes with a 256-bin shared histogram (the logits of one
//     image are a few hundred KB at most and stay in L1/L2 between passes);
//  2. compaction: keys above the threshold through a shared counter, keys equal
//     to it in flat-index order (block scan over per-thread contiguous chunks)
//     until k are taken -- deterministic ties, lowest flat index first;
//  3. bitonic sort of the k candidates on (key desc, index asc) in shared memory;
//  4. epilogue.  Since sigmoid is monotone the selection runs on raw logits.
#include "common.cuh"

namespace mmltk {

namespace {

constexpr int kThreads = 1024;
constexpr int kMaxK = 1024;

__device__ __forceinline__ uint32_t order_key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <typename T>
__device__ __forceinline__ float ld(const T* p, int64_t i) { return to_f(p[i]); }

// The K largest of x[0, N) into cand[0, K), sorted (value descending, index ascending), each entry the
// order-preserving key in the high word and ~index in the low word; one CTA of kThreads threads.
template <typename LT>
__device__ void block_topk(const LT* __restrict__ x, int64_t N, int K, unsigned long long* cand) {
    __shared__ uint32_t hist[256];
    __shared__ uint32_t s_prefix, s_mask, s_need, s_count;
    __shared__ uint32_t scan[kThreads];
    const int tid = threadIdx.x;
    if (tid == 0) {
        s_prefix = 0;
        s_mask = 0;
        s_need = uint32_t(K);
        s_count = 0;
    }
    // 1. radix select, most significant digit first
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += kThreads) hist[i] = 0;
        __syncthreads();
        const uint32_t prefix = s_prefix, mask = s_mask;
        // warp-aggregated counting: the logits of one image share a few leading digits, so most lanes
        // of a warp hit the same bin; one shared atomic per distinct bin instead of one per lane
        const int64_t span = (N + 31) / 32 * 32;    // every lane of a warp takes part in each round
        for (int64_t i = tid; i < span; i += kThreads) {
            uint32_t bin = 0xffffffffu;
            if (i < N) {
                const uint32_t k = order_key(ld(x, i));
                if ((k & mask) == prefix) bin = (k >> shift) & 0xffu;
            }
            const uint32_t same = __match_any_sync(0xffffffffu, bin);
            if (bin != 0xffffffffu && (threadIdx.x & 31) == __ffs(same) - 1) atomicAdd(&hist[bin], __popc(same));
        }
        __syncthreads();
        if (tid == 0) {
            uint32_t need = s_need, acc = 0;
            int d = 255;
            for (; d > 0; --d) {
                if (acc + hist[d] >= need) break;
                acc += hist[d];
            }
            s_need = need - acc;  // how many of the threshold-prefix keys still have to be taken
            s_prefix = prefix | (uint32_t(d) << shift);
            s_mask = mask | (0xffu << shift);
        }
        __syncthreads();
    }
    const uint32_t thr = s_prefix;      // the k-th largest key
    const uint32_t ties = s_need;       // keys == thr to take (>= 1)
    // 2a. strictly greater keys (there are K - ties of them)
    for (int64_t i = tid; i < N; i += kThreads) {
        const uint32_t k = order_key(ld(x, i));
        if (k > thr) {
            const uint32_t s = atomicAdd(&s_count, 1u);
            cand[s] = (static_cast<unsigned long long>(k) << 32) | (0xffffffffu - uint32_t(i));
        }
    }
    // 2b. equal keys in index order
    const int64_t chunk = (N + kThreads - 1) / kThreads;
    const int64_t lo = int64_t(tid) * chunk, hi = min(N, lo + chunk);
    uint32_t mine = 0;
    for (int64_t i = lo; i < hi; ++i) mine += order_key(ld(x, i)) == thr;
    scan[tid] = mine;
    __syncthreads();
    for (int off = 1; off < kThreads; off <<= 1) {  // inclusive Hillis-Steele scan
        const uint32_t v = tid >= off ? scan[tid - off] : 0u;
        __syncthreads();
        scan[tid] += v;
        __syncthreads();
    }
    uint32_t rank = scan[tid] - mine;
    const uint32_t base = uint32_t(K) - ties;
    for (int64_t i = lo; i < hi && rank < ties; ++i) {
        if (order_key(ld(x, i)) == thr) {
            cand[base + rank] = (static_cast<unsigned long long>(thr) << 32) | (0xffffffffu - uint32_t(i));
            ++rank;
        }
    }
    // 3. bitonic sort, descending, over the next power of two
    int P = 1;
    while (P < K) P <<= 1;
    for (int i = K + tid; i < P; i += kThreads) cand[i] = 0ull;
    __syncthreads();
    for (int size = 2; size <= P; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < P; i += kThreads) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool desc = (i & size) == 0;
                    const unsigned long long a = cand[i], c = cand[j];
                    if ((a < c) == desc) {
                        cand[i] = c;
                        cand[j] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
}

__device__ __forceinline__ uint32_t cand_index(unsigned long long c) {
    return 0xffffffffu - uint32_t(c & 0xffffffffull);
}

template <typename LT, typename BT>
__global__ void __launch_bounds__(kThreads) topk_post_kernel(const LT* __restrict__ logits, const BT* __restrict__ boxes,
                                                             const float* __restrict__ sizes, int Q, int C, int K,
                                                             float fixed_h, float fixed_w, float* __restrict__ scores,
                                                             int64_t* __restrict__ labels, float* __restrict__ out_boxes,
                                                             int32_t* __restrict__ queries) {
    __shared__ unsigned long long cand[kMaxK];
    const int b = blockIdx.x, tid = threadIdx.x;
    const int64_t N = int64_t(Q) * C;
    const LT* x = logits + int64_t(b) * N;
    block_topk(x, N, K, cand);
    // 4. epilogue
    const float H = sizes ? sizes[2 * b] : fixed_h, W = sizes ? sizes[2 * b + 1] : fixed_w;
    for (int r = tid; r < K; r += kThreads) {
        const uint32_t idx = cand_index(cand[r]);
        const int q = int(idx / uint32_t(C)), c = int(idx % uint32_t(C));
        const float v = ld(x, idx);
        const int64_t o = int64_t(b) * K + r;
        scores[o] = 1.f / (1.f + expf(-v));
        labels[o] = c;
        queries[o] = q;
        const BT* bx = boxes + (int64_t(b) * Q + q) * 4;
        const float cx = ld(bx, 0), cy = ld(bx, 1), w = fmaxf(ld(bx, 2), 0.f), h = fmaxf(ld(bx, 3), 0.f);
        out_boxes[4 * o + 0] = (cx - 0.5f * w) * W;
        out_boxes[4 * o + 1] = (cy - 0.5f * h) * H;
        out_boxes[4 * o + 2] = (cx + 0.5f * w) * W;
        out_boxes[4 * o + 3] = (cy + 0.5f * h) * H;
    }
}

// Indices of the K largest entries of every row of x [rows, N], sorted (value descending, index
// ascending on ties): one CTA per row -- the two-stage head's per-group proposal selection.
template <typename LT>
__global__ void __launch_bounds__(kThreads) row_topk_kernel(const LT* __restrict__ x, int64_t N, int K,
                                                            int64_t* __restrict__ idx) {
    __shared__ unsigned long long cand[kMaxK];
    block_topk(x + int64_t(blockIdx.x) * N, N, K, cand);
    for (int r = threadIdx.x; r < K; r += kThreads) idx[int64_t(blockIdx.x) * K + r] = cand_index(cand[r]);
}

}  // namespace

cudaError_t launch_row_topk(DType t, const void* x, int64_t rows, int64_t N, int K, int64_t* idx, cudaStream_t st) {
    if (rows == 0 || K == 0) return cudaSuccess;
    if (K > kMaxK || K > N || N >= (int64_t(1) << 31) || rows > 0x7fffffff) return cudaErrorInvalidValue;
    if (t == DType::kBF16)
        row_topk_kernel<__nv_bfloat16><<<static_cast<unsigned>(rows), kThreads, 0, st>>>(
            static_cast<const __nv_bfloat16*>(x), N, K, idx);
    else if (t == DType::kF32)
        row_topk_kernel<float><<<static_cast<unsigned>(rows), kThreads, 0, st>>>(static_cast<const float*>(x), N, K, idx);
    else
        return cudaErrorInvalidValue;
    return cudaGetLastError();
}

cudaError_t launch_topk_postprocess(DType lt, DType bt, const void* logits, const void* boxes, const float* sizes,
                                    int B, int Q, int C, int K, float fixed_h, float fixed_w, float* scores,
                                    int64_t* labels, float* out_boxes, int32_t* queries, cudaStream_t st) {
    if (B == 0 || K == 0) return cudaSuccess;
    if (K > kMaxK || int64_t(K) > int64_t(Q) * C || int64_t(Q) * C >= (int64_t(1) << 31)) return cudaErrorInvalidValue;
#define MMLTK_TK(L, BX)                                                                                   \
    topk_post_kernel<L, BX><<<B, kThreads, 0, st>>>(static_cast<const L*>(logits), static_cast<const BX*>(boxes), \
                                                    sizes, Q, C, K, fixed_h, fixed_w, scores, labels, out_boxes, queries)
    if (lt == DType::kBF16 && bt == DType::kBF16) MMLTK_TK(__nv_bfloat16, __nv_bfloat16);
    else if (lt == DType::kBF16) MMLTK_TK(__nv_bfloat16, float);
    else if (bt == DType::kBF16) MMLTK_TK(float, __nv_bfloat16);
    else MMLTK_TK(float, float);
#undef MMLTK_TK
    return cudaGetLastError();
}

}  // namespace mmltk
