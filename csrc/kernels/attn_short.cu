// Short-sequence scaled dot-product attention on the 5th-generation tensor cores (tcgen05), forward
// and backward, head dim 32 or 64, sequences of at most 384 tokens: the Group-DETR decoder's
// self-attention (300 queries per group, head dim 32; reference `nn::MultiheadAttention`,
// `src/rfdetr/layers/model.cpp:917,945`) and the windowed ViT layers (325 tokens per window, head
// dim 64; reference `at::scaled_dot_product_attention`, `model.cpp:498`).
//
// One CTA per (sequence, head).  Because a whole sequence fits on chip, every score row is
// complete before its softmax: S = Q.K^T for a 128-query tile spans all keys in tensor memory
// (<= 384 fp32 columns), so the softmax is exact in two passes over the row (maximum, then
// exponentials) with no running-maximum rescaling, and the backward pass accumulates dV, dK and
// dQ on chip without atomics.
//
// Operands are read by TMA as 128-row x 64-column bf16 boxes with the 128-byte swizzle, straight
// out of the projection outputs (each of q / k / v / dO has its own tensor map and first column,
// head h at column col + h * D).  With D = 32 a box also carries the neighbouring head's columns;
// the MMAs read only the first D.  Rows past the sequence are the next sequence's (or TMA's zero
// fill) and are masked by index.
//
// Forward, warps 0-7 = softmax / epilogue (warp w: TMEM lane quadrant w % 4, so thread = query row,
// and half w / 4 of the row's score columns; partial maxima and sums meet in shared memory),
// warp 8 = TMA producer + TMEM owner, warp 9 = MMA issuer.  Per 128-query tile t:
//   S_t = Q_t.K^T  (M=128, N=keys, K=D)              TMEM columns [0, 384)
//   P_t = exp2(S_t * scale * log2e - m)  -> bf16, K-major swizzled in shared memory
//   O_t = P_t.V    (M=128, N=D, K=keys, V MN-major)  TMEM columns [384, 384 + D)
// S_{t+1} is issued as soon as the softmax has read S_t, so it overlaps O_t and its epilogue.
//
// Backward, same roles; thread = key row for the transposed products, the two halves taking the
// block's two 64-query column tiles.  For every (key tile kt, query tile qt) block:
//   S^T  = K_kt.Q_qt^T, dP^T = V_kt.dO_qt^T            TMEM [0, 128), [128, 256)
//   P^T  = exp2(S^T * scale * log2e - lse2[q]),  dS^T = P^T * (dP^T - delta[q])  -> bf16 smem
//   dV_kt += P^T.dO_qt,  dK_kt += dS^T.Q_qt            (dS^T K-major: rows = keys)
//   dQ_qt += dS.K_kt                                   (the same dS^T tile read MN-major)
// with delta[q] = sum_d dO[q, d] O[q, d] from a small pre-pass.  D = 32 keeps all three dQ tiles
// in tensor memory; D = 64 (whose dQ tiles do not fit next to the rest) takes each block's dQ
// part out of tensor memory and adds it into an fp32 row owned by the same thread (no atomics:
// query row q is always thread q % 128).
//
// Every mbarrier wait is bounded; on timeout the kernel records a code in the status word, every
// role leaves, and tensor memory is released.
#include <cudaTypedefs.h>

#include <cstdio>

#include "common.cuh"
#include "launch_api.h"
#include "tcgen05.cuh"

namespace mmltk {

namespace {

using namespace tc;

constexpr int kRows = 128;
constexpr int kBox = kRows * 64 * 2;    // 16 KB: one 128-row x 64-column bf16 box
constexpr int kMaxL = 384;
constexpr int kSoftWarps = 8;           // two per TMEM lane quadrant; each takes half of a row's columns
constexpr int kSoftThreads = 32 * kSoftWarps;
constexpr int kProdWarp = kSoftWarps, kMmaWarp = kSoftWarps + 1;
constexpr int kThreads = 32 * (kSoftWarps + 2);
constexpr int kTmemCols = 512;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// named barrier of the softmax warps that also ANDs a flag across them, so that when one warp's
// bounded wait gives up every softmax warp learns it at the same barrier and they leave together
__device__ __forceinline__ bool soft_sync_and(bool ok) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(ok ? 1u : 0u), "n"(kSoftThreads)
        : "memory");
    return r != 0;
}

// 16-byte chunk j (8 bf16) of row r of a K-major 128-byte-swizzled tile
__device__ __forceinline__ void put16(unsigned char* tile, int r, int j, uint4 v) {
    *reinterpret_cast<uint4*>(tile + r * 128 + ((j ^ (r & 7)) << 4)) = v;
}
// 8 consecutive keys / queries starting at column k (a multiple of 8) of a P-style smem matrix made of
// 64-column K-major tiles
__device__ __forceinline__ void put8(unsigned char* mat, int r, int k, const uint32_t* w) {
    put16(mat + (k >> 6) * kBox, r, (k & 63) >> 3, make_uint4(w[0], w[1], w[2], w[3]));
}

struct __align__(8) FwdCtl {
    uint64_t kv_full, q_full, q_empty, s_full, p_full, o_full, o_free;
    uint32_t tmem_base;
    int abort;
};

struct FwdArgs {
    __nv_bfloat16* o;
    int64_t ldo;
    float* lse;        // [N, H, L] natural log, or null
    int* status;
    int L, H, qcol, kcol, vcol, ocol;
    float scale_log2;
};

// score columns computed per row: a multiple of 64, so that each half is whole 32-column loads
__host__ __device__ __forceinline__ int fwd_score_cols(int L) { return (L + 63) / 64 * 64; }

__host__ __device__ size_t fwd_smem_bytes(int L) {
    const int T = (L + kRows - 1) / kRows;
    const int NP = fwd_score_cols(L) / 64;
    return 1024 + static_cast<size_t>(kBox) * (1 + 2 * T + NP) + 4 * kRows * sizeof(float);
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attn_short_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                          const __grid_constant__ CUtensorMap tv, FwdArgs a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    FwdCtl* ctl = reinterpret_cast<FwdCtl*>(smem_raw);
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + sizeof(FwdCtl) + 1023) & ~uintptr_t(1023));
    const int L = a.L;
    const int T = (L + kRows - 1) / kRows;     // 128-row tiles of queries (and keys)
    const int SN = fwd_score_cols(L);          // score columns computed / read
    const int NP = SN / 64;                    // 64-key P tiles
    const int KO = (L + 15) / 16 * 16;         // keys reduced by P.V
    unsigned char* sQ = smem;
    unsigned char* sK = sQ + kBox;
    unsigned char* sV = sK + T * kBox;
    unsigned char* sP = sV + T * kBox;
    float* s_max = reinterpret_cast<float*>(sP + NP * kBox);   // [2][128] partial row maxima
    float* s_sum = s_max + 2 * kRows;                          // [2][128] partial row sums
    if (L > kMaxL ||
        reinterpret_cast<unsigned char*>(s_sum + 2 * kRows) - smem_raw > static_cast<ptrdiff_t>(fwd_smem_bytes(L))) {
        if (threadIdx.x == 0) atomicCAS(a.status, 0, 8);
        return;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = blockIdx.x / a.H, h = blockIdx.x % a.H;
    const int row0 = n * L;

    if (threadIdx.x == 0) {
        mbar_init(&ctl->kv_full, 1);
        mbar_init(&ctl->q_full, 1);
        mbar_init(&ctl->q_empty, 1);
        mbar_init(&ctl->s_full, 1);
        mbar_init(&ctl->p_full, kSoftWarps);
        mbar_init(&ctl->o_full, 1);
        mbar_init(&ctl->o_free, kSoftWarps);
        ctl->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == kProdWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&ctl->tmem_base)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;
    const uint32_t tS = tmem, tO = tmem + kMaxL;

    if (warp == kProdWarp) {
        if (lane == 0) {
            mbar_expect_tx(&ctl->kv_full, 2 * T * kBox);
            for (int t = 0; t < T; ++t) {
                tma_load_2d(&tk, &ctl->kv_full, sK + t * kBox, a.kcol + h * D, row0 + t * kRows);
                tma_load_2d(&tv, &ctl->kv_full, sV + t * kBox, a.vcol + h * D, row0 + t * kRows);
            }
            for (int t = 0; t < T; ++t) {
                if (t > 0 && !mbar_wait(&ctl->q_empty, (t - 1) & 1, &ctl->abort)) {
                    ctl->abort = 1;
                    atomicCAS(a.status, 0, 1);
                    break;
                }
                mbar_expect_tx(&ctl->q_full, kBox);
                tma_load_2d(&tq, &ctl->q_full, sQ, a.qcol + h * D, row0 + t * kRows);
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            constexpr uint32_t idesc_o = instr_desc(false, true, D);
            const uint32_t q = smem_u32(sQ), k = smem_u32(sK), v = smem_u32(sV), p = smem_u32(sP);
            auto issue_s = [&]() {
                for (int c0 = 0; c0 < SN; c0 += 256) {
                    const int nc = min(256, SN - c0);
                    const uint32_t idesc_s = instr_desc(false, false, nc);
#pragma unroll
                    for (int kk = 0; kk < D / 16; ++kk)
                        tc_mma(tS + c0, operand_desc<false>(q, kk), smem_desc(k + c0 * 128 + kk * 32, 16, 1024),
                               idesc_s, kk > 0);
                }
                tc_commit(&ctl->q_empty);
                tc_commit(&ctl->s_full);
            };
            bool ok = mbar_wait(&ctl->kv_full, 0, &ctl->abort) && mbar_wait(&ctl->q_full, 0, &ctl->abort);
            if (ok) {
                tc_fence_after();
                issue_s();
            }
            for (int t = 0; ok && t < T; ++t) {
                ok = mbar_wait(&ctl->p_full, t & 1, &ctl->abort);   // P_t written, S_t read
                if (!ok) break;
                tc_fence_after();
                if (t + 1 < T) {
                    ok = mbar_wait(&ctl->q_full, (t + 1) & 1, &ctl->abort);
                    if (!ok) break;
                    tc_fence_after();
                    issue_s();
                }
                if (t > 0) {
                    ok = mbar_wait(&ctl->o_free, (t - 1) & 1, &ctl->abort);   // O_{t-1} read out
                    if (!ok) break;
                    tc_fence_after();
                }
                for (int j = 0; j < KO / 16; ++j)
                    tc_mma(tO, smem_desc(p + (j >> 2) * kBox + (j & 3) * 32, 16, 1024),
                           smem_desc(v + j * 2048, 8192, 1024), idesc_o, j > 0);
                tc_commit(&ctl->o_full);
            }
            if (!ok) {
                ctl->abort = 1;
                atomicCAS(a.status, 0, 2);
            }
        }
    } else {
        // softmax / epilogue: warp w reads TMEM lane quadrant w % 4 (thread = query row r of the
        // tile) and the half w / 4 of the row's score columns; partial maxima / sums meet in shared
        // memory
        const int quad = warp & 3, half = warp >> 2;
        const int r = 32 * quad + lane;
        const uint32_t lane_off = static_cast<uint32_t>(32 * quad) << 16;
        const int cn = SN / 2, c0 = half * cn;
        bool ok = true;
        for (int t = 0; t < T; ++t) {
            ok = ok && mbar_wait(&ctl->s_full, t & 1, &ctl->abort);
            float mx = -1e30f;
            if (ok) {
                tc_fence_after();
                int c = c0;
                for (; c + 64 <= c0 + cn; c += 64) {
                    float sv[64];
                    tmem_ld64(tS + lane_off + c, sv);
#pragma unroll
                    for (int i = 0; i < 64; ++i)
                        if (c + i < L) mx = fmaxf(mx, sv[i]);
                }
                if (c < c0 + cn) {
                    float sv[32];
                    tmem_ld32(tS + lane_off + c, sv);
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (c + i < L) mx = fmaxf(mx, sv[i]);
                }
            }
            s_max[half * kRows + r] = mx;
            ok = soft_sync_and(ok);
            if (!ok) break;
            const float m = fmaxf(s_max[r], s_max[kRows + r]) * a.scale_log2;
            float sum = 0.f;
            for (int c = c0; c < c0 + cn; c += 32) {
                float sv[32];
                tmem_ld32(tS + lane_off + c, sv);
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    uint32_t w[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int k0 = c + 8 * g + 2 * i;
                        const float p0 = k0 < L ? ex2(sv[8 * g + 2 * i] * a.scale_log2 - m) : 0.f;
                        const float p1 = k0 + 1 < L ? ex2(sv[8 * g + 2 * i + 1] * a.scale_log2 - m) : 0.f;
                        sum += p0 + p1;
                        w[i] = pack_bf16x2(p0, p1);
                    }
                    put8(sP, r, c + 8 * g, w);
                }
            }
            s_sum[half * kRows + r] = sum;
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc_fence_before();
            soft_sync_and(true);
            const float total = s_sum[r] + s_sum[kRows + r];
            __syncwarp();
            if (lane == 0) mbar_arrive(&ctl->p_full);
            ok = mbar_wait(&ctl->o_full, t & 1, &ctl->abort);
            if (ok) {
                tc_fence_after();
                // this half's D / 2 output columns
                float o[D / 2];
                if (D == 32) tmem_ld16(tO + lane_off + half * 16, o);
                else tmem_ld32(tO + lane_off + half * 32, o);
                const int qrow = t * kRows + r;
                if (qrow < L) {
                    const float inv = 1.f / total;
                    uint4* dst = reinterpret_cast<uint4*>(a.o + static_cast<int64_t>(row0 + qrow) * a.ldo + a.ocol +
                                                          h * D + half * (D / 2));
#pragma unroll
                    for (int j = 0; j < D / 16; ++j)
                        dst[j] = make_uint4(pack_bf16x2(o[8 * j] * inv, o[8 * j + 1] * inv),
                                            pack_bf16x2(o[8 * j + 2] * inv, o[8 * j + 3] * inv),
                                            pack_bf16x2(o[8 * j + 4] * inv, o[8 * j + 5] * inv),
                                            pack_bf16x2(o[8 * j + 6] * inv, o[8 * j + 7] * inv));
                    if (a.lse && half == 0)
                        a.lse[(static_cast<int64_t>(n) * a.H + h) * L + qrow] = (m + __log2f(total)) * 0.69314718055994531f;
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ctl->o_free);
        }
        if (!ok) {
            ctl->abort = 1;
            if (lane == 0) atomicCAS(a.status, 0, 3);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kProdWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// ------------------------------------------------------------------------ forward, ping-pong form
//
// Two softmax warpgroups (warps 0-3, 4-7; thread = query row) each own a region of tensor memory
// (S chunk: 128 columns, O: 64 columns) and a P buffer in shared memory, and work through the keys in
// 128-key chunks with an online softmax: while one warpgroup exponentiates its chunk, the tensor core
// computes the other's.  The running maximum is only moved (and O rescaled in tensor memory) when a
// chunk's maximum exceeds it by more than 2^8, so rescaling is rare.  Head dim 32: one CTA takes two
// heads of a sequence (the 64-column boxes of q / k / v hold both), warpgroup w head 2j + w, every
// query tile; P.V runs with N = 64 (both heads' v columns) and each warpgroup keeps its half.  Head
// dim 64: one CTA per (sequence, head), warpgroup w takes query tiles w, w + 2, ...
namespace pp {
constexpr int kWarps = 10;                  // 8 softmax (2 warpgroups), producer, MMA issuer
constexpr int kThreadsPP = 32 * kWarps;
constexpr int kProd = 8, kMma = 9;
constexpr int kRegion = 256;                // tensor-memory columns per warpgroup: S [0, 128), O [128, 192)
constexpr float kRescale = 8.f;             // log2 slack before the running maximum is moved
}  // namespace pp

struct __align__(8) Fwd2Ctl {
    uint64_t kv_full, q_full[2], q_empty[2], s_full[2], p_full[2], o_full[2], o_free[2];
    uint32_t tmem_base;
    int abort;
};

__host__ __device__ constexpr size_t fwd2_smem_bytes() {
    // K, V (3 boxes each), Q (2 buffers), P (2 warpgroups x 2 boxes of 64 keys), control block
    return 1024 + static_cast<size_t>(kBox) * (3 + 3 + 2 + 4) + 256;
}

template <int D>
__global__ void __launch_bounds__(pp::kThreadsPP, 1)
    attn_short_fwd2_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                           const __grid_constant__ CUtensorMap tv, FwdArgs a) {
    using namespace pp;
    constexpr bool kPair = D == 32;           // two heads per CTA
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    Fwd2Ctl* ctl = reinterpret_cast<Fwd2Ctl*>(smem_raw);
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + sizeof(Fwd2Ctl) + 1023) & ~uintptr_t(1023));
    const int L = a.L;
    const int T = (L + kRows - 1) / kRows;    // query tiles = key chunks
    unsigned char* sK = smem;
    unsigned char* sV = sK + 3 * kBox;
    unsigned char* sQ = sV + 3 * kBox;        // 2 buffers
    unsigned char* sP = sQ + 2 * kBox;        // 2 warpgroups x 2 boxes
    if (L > kMaxL || sP + 4 * kBox - smem_raw > static_cast<ptrdiff_t>(fwd2_smem_bytes())) {
        if (threadIdx.x == 0) atomicCAS(a.status, 0, 8);
        return;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int groups = kPair ? (a.H + 1) / 2 : a.H;     // CTAs per sequence
    const int n = blockIdx.x / groups, g = blockIdx.x % groups;
    const int row0 = n * L;
    const int hcol = g * 64;                  // first column of this CTA's boxes within each source
    // jobs (query tiles) of warpgroup w: pair form every tile, else tiles w, w + 2, ...
    auto jobs = [&](int w) { return kPair ? (2 * g + w < a.H ? T : 0) : (T - w + 1) / 2; };
    auto tile_of = [&](int w, int j) { return kPair ? j : w + 2 * j; };

    if (threadIdx.x == 0) {
        mbar_init(&ctl->kv_full, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&ctl->q_full[i], 1);
            mbar_init(&ctl->q_empty[i], 1);
            mbar_init(&ctl->s_full[i], 1);
            mbar_init(&ctl->p_full[i], 4);
            mbar_init(&ctl->o_full[i], 1);
            mbar_init(&ctl->o_free[i], 4);
        }
        ctl->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == kProd) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&ctl->tmem_base)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;

    if (warp == kProd) {
        if (lane == 0) {
            mbar_expect_tx(&ctl->kv_full, 2 * T * kBox);
            for (int t = 0; t < T; ++t) {
                tma_load_2d(&tk, &ctl->kv_full, sK + t * kBox, a.kcol + hcol, row0 + t * kRows);
                tma_load_2d(&tv, &ctl->kv_full, sV + t * kBox, a.vcol + hcol, row0 + t * kRows);
            }
            bool ok = true;
            if (kPair) {
                for (int t = 0; ok && t < T; ++t) {
                    const int b = t & 1;
                    if (t >= 2 && !mbar_wait(&ctl->q_empty[b], ((t >> 1) - 1) & 1, &ctl->abort)) ok = false;
                    if (!ok) break;
                    mbar_expect_tx(&ctl->q_full[b], kBox);
                    tma_load_2d(&tq, &ctl->q_full[b], sQ + b * kBox, a.qcol + hcol, row0 + t * kRows);
                }
            } else {
                for (int j = 0; ok && 2 * j < T; ++j) {
                    for (int w = 0; w < 2; ++w) {
                        const int t = w + 2 * j;
                        if (t >= T) break;
                        if (j >= 1 && !mbar_wait(&ctl->q_empty[w], (j - 1) & 1, &ctl->abort)) {
                            ok = false;
                            break;
                        }
                        mbar_expect_tx(&ctl->q_full[w], kBox);
                        tma_load_2d(&tq, &ctl->q_full[w], sQ + w * kBox, a.qcol + hcol, row0 + t * kRows);
                    }
                }
            }
            if (!ok) {
                ctl->abort = 1;
                atomicCAS(a.status, 0, 1);
            }
        }
    } else if (warp == kMma) {
        if (lane == 0) {
            constexpr uint32_t idesc_s = instr_desc(false, false, kRows);   // S chunk: N = 128 keys
            constexpr uint32_t idesc_o = instr_desc(false, true, 64);       // O: N = 64 (a whole v box)
            const uint32_t qb = smem_u32(sQ), kb = smem_u32(sK), vb = smem_u32(sV), pb = smem_u32(sP);
            const int steps[2] = {jobs(0) * T, jobs(1) * T};
            bool ok = mbar_wait(&ctl->kv_full, 0, &ctl->abort);
            // S chunk of warpgroup w at step k (job k / T, key chunk k % T)
            auto issue_s = [&](int w, int k) -> bool {
                const int j = k / T, c = k % T;
                const int qbuf = kPair ? (j & 1) : w;
                if (c == 0) {
                    const uint32_t qph = kPair ? ((j >> 1) & 1) : (j & 1);
                    if (!mbar_wait(&ctl->q_full[qbuf], qph, &ctl->abort)) return false;
                    tc_fence_after();
                }
                const int kk0 = kPair ? 2 * w : 0;   // head 2g + w: columns [32 w, 32 w + 32) of the box
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    tc_mma(tmem + w * kRegion, operand_desc<false>(qb + qbuf * kBox, kk0 + kk),
                           operand_desc<false>(kb + c * kBox, kk0 + kk), idesc_s, kk > 0);
                tc_commit(&ctl->s_full[w]);
                if (c == T - 1 && (!kPair || w == 1 || jobs(1) == 0)) tc_commit(&ctl->q_empty[qbuf]);
                return true;
            };
            for (int w = 0; ok && w < 2; ++w)
                if (steps[w] > 0) ok = issue_s(w, 0);
            for (int k = 0; ok; ++k) {
                bool any = false;
                for (int w = 0; ok && w < 2; ++w) {
                    if (k >= steps[w]) continue;
                    any = true;
                    const int j = k / T, c = k % T;
                    if (!mbar_wait(&ctl->p_full[w], k & 1, &ctl->abort)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (c == 0 && j > 0) {
                        if (!mbar_wait(&ctl->o_free[w], (j - 1) & 1, &ctl->abort)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                    }
                    const uint32_t p = pb + w * 2 * kBox;
                    // K slices of 16 keys that hold a key of the sequence (the last chunk's P is only
                    // written that far)
                    const int nks = min(kRows / 16, (L - c * kRows + 15) / 16);
                    for (int s16 = 0; s16 < nks; ++s16)
                        tc_mma(tmem + w * kRegion + 128, smem_desc(p + (s16 >> 2) * kBox + (s16 & 3) * 32, 16, 1024),
                               smem_desc(vb + c * kBox + s16 * 2048, 8192, 1024), idesc_o, (c > 0 || s16 > 0));
                    if (c == T - 1) tc_commit(&ctl->o_full[w]);
                    if (k + 1 < steps[w]) ok = issue_s(w, k + 1);
                }
                if (!any) break;
            }
            if (!ok) {
                ctl->abort = 1;
                atomicCAS(a.status, 0, 2);
            }
        }
    } else {
        // softmax warpgroup w = warp / 4: thread = query row r of the current tile (TMEM lane r)
        const int w = warp >> 2, quad = warp & 3;
        const int r = 32 * quad + lane;
        const uint32_t lane_off = static_cast<uint32_t>(32 * quad) << 16;
        const uint32_t tS = tmem + w * kRegion + lane_off, tO = tS + 128;
        const int h = kPair ? 2 * g + w : g;
        const int ocol_t = kPair ? 32 * w : 0;   // this head's columns of the O accumulator
        unsigned char* myP = sP + w * 2 * kBox;
        const int J = jobs(w);
        bool ok = true;
        int k = 0;
        for (int j = 0; ok && j < J; ++j) {
            const int t = tile_of(w, j);
            const bool live = t * kRows + 32 * quad < L;   // warp-uniform: any valid query row here
            float m_used = -1e30f, l = 0.f;
            for (int c = 0; c < T; ++c, ++k) {
                if (!mbar_wait(&ctl->s_full[w], k & 1, &ctl->abort)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (live) {
                    // the row maximum over the chunk: 64 columns per tensor-memory round trip, four
                    // independent running maxima; columns past the sequence only in the last chunk
                    const int kbase = c * kRows;
                    const bool full = kbase + kRows <= L;   // warp-uniform
                    float mx[4] = {-1e30f, -1e30f, -1e30f, -1e30f};
#pragma unroll
                    for (int h2 = 0; h2 < 2; ++h2) {
                        if (kbase + 64 * h2 >= L) break;   // no key of this half (warp-uniform)
                        float sv[64];
                        tmem_ld64(tS + 64 * h2, sv);
                        if (!full) {
#pragma unroll
                            for (int i = 0; i < 64; ++i)
                                if (kbase + 64 * h2 + i >= L) sv[i] = -1e30f;
                        }
#pragma unroll
                        for (int i = 0; i < 64; ++i) mx[i & 3] = fmaxf(mx[i & 3], sv[i]);
                        asm volatile("" : "+f"(mx[0]), "+f"(mx[1]), "+f"(mx[2]), "+f"(mx[3]));
                    }
                    const float mc = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
                    const float m_new = mc * a.scale_log2;
                    bool need = false;
                    float alpha = 1.f;
                    if (c == 0) {
                        m_used = m_new;
                    } else if (m_new > m_used + kRescale) {
                        need = true;
                        alpha = ex2(m_used - m_new);
                        m_used = m_new;
                        l *= alpha;
                    }
                    if (__any_sync(0xffffffffu, need)) {
                        // O holds the chunks so far (their P.V are complete: S of this chunk was issued
                        // after them); bring it to the new maximum before this chunk's P.V adds to it
#pragma unroll
                        for (int part = 0; part < D / 32; ++part) {
                            float o[32];
                            const uint32_t at = tO + ocol_t + 32 * part;
                            tmem_ld32(at, o);
#pragma unroll
                            for (int i = 0; i < 32; ++i) o[i] *= alpha;
                            tmem_st16(at, o);
                            tmem_st16(at + 16, o + 16);
                            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                        }
                    }
                    // exponentials: 2^(s * scale * log2 e - m) with the columns past the sequence at
                    // -inf (2^-inf = 0), four independent partial sums, bf16 P into shared memory
                    float sm4[4] = {0.f, 0.f, 0.f, 0.f};
                    const float sl = a.scale_log2, mneg = -m_used;
#pragma unroll
                    for (int h2 = 0; h2 < 2; ++h2) {
                        // a half with no key is neither exponentiated nor read by P.V (its K slices
                        // are not issued)
                        if (kbase + 64 * h2 >= L) break;
                        float sv[64];
                        tmem_ld64(tS + 64 * h2, sv);
                        if (!full) {
#pragma unroll
                            for (int i = 0; i < 64; ++i)
                                if (kbase + 64 * h2 + i >= L) sv[i] = -__int_as_float(0x7f800000);
                        }
#pragma unroll
                        for (int g8 = 0; g8 < 8; ++g8) {
                            uint32_t wv[4];
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const float p0 = ex2(fmaf(sv[8 * g8 + 2 * i], sl, mneg));
                                const float p1 = ex2(fmaf(sv[8 * g8 + 2 * i + 1], sl, mneg));
                                sm4[i] += p0 + p1;
                                wv[i] = pack_bf16x2(p0, p1);
                            }
                            put8(myP, r, 64 * h2 + 8 * g8, wv);
                        }
                        asm volatile("" : "+f"(sm4[0]), "+f"(sm4[1]), "+f"(sm4[2]), "+f"(sm4[3])::"memory");
                    }
                    const float sum = (sm4[0] + sm4[1]) + (sm4[2] + sm4[3]);
                    l += sum;
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&ctl->p_full[w]);
            }
            if (!ok) break;
            if (!mbar_wait(&ctl->o_full[w], j & 1, &ctl->abort)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float o[32];
            if (D == 32) {
                tmem_ld32(tO + ocol_t, o);
            } else {
                tmem_ld32(tO, o);
            }
            float o2[32];
            if (D == 64) tmem_ld32(tO + 32, o2);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ctl->o_free[w]);
            const int qrow = t * kRows + r;
            if (qrow < L) {
                const float inv = 1.f / l;
                uint4* dst = reinterpret_cast<uint4*>(a.o + static_cast<int64_t>(row0 + qrow) * a.ldo + a.ocol + h * D);
#pragma unroll
                for (int q8 = 0; q8 < 4; ++q8)
                    dst[q8] = make_uint4(pack_bf16x2(o[8 * q8] * inv, o[8 * q8 + 1] * inv),
                                         pack_bf16x2(o[8 * q8 + 2] * inv, o[8 * q8 + 3] * inv),
                                         pack_bf16x2(o[8 * q8 + 4] * inv, o[8 * q8 + 5] * inv),
                                         pack_bf16x2(o[8 * q8 + 6] * inv, o[8 * q8 + 7] * inv));
                if (D == 64) {
#pragma unroll
                    for (int q8 = 0; q8 < 4; ++q8)
                        dst[4 + q8] = make_uint4(pack_bf16x2(o2[8 * q8] * inv, o2[8 * q8 + 1] * inv),
                                                 pack_bf16x2(o2[8 * q8 + 2] * inv, o2[8 * q8 + 3] * inv),
                                                 pack_bf16x2(o2[8 * q8 + 4] * inv, o2[8 * q8 + 5] * inv),
                                                 pack_bf16x2(o2[8 * q8 + 6] * inv, o2[8 * q8 + 7] * inv));
                }
                if (a.lse) a.lse[(static_cast<int64_t>(n) * a.H + h) * L + qrow] = (m_used + __log2f(l)) * 0.69314718055994531f;
            }
        }
        if (!ok) {
            ctl->abort = 1;
            if (lane == 0) atomicCAS(a.status, 0, 3);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kProd) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// ------------------------------------------------------------------------------------ backward

struct __align__(8) BwdCtl {
    uint64_t qdo_full, kv_full, kv_empty, sdp_full, pds_full, mma_done, dkv_full, dkv_free, dq_free;
    uint32_t tmem_base;
    int abort;
};

struct BwdArgs {
    const float* lse;     // [N, H, L] natural log
    const float* delta;   // [N, H, L]: sum_d dO * O
    float* dq_acc;        // D = 64: fp32 [N * H, L, 64] scratch
    __nv_bfloat16 *dq, *dk, *dv;
    int64_t lddq, lddk, lddv;
    int dqcol, dkcol, dvcol;
    int* status;
    int L, H, qcol, kcol, vcol, docol;
    float scale_log2, scale;
};

__host__ __device__ size_t bwd_smem_bytes(int L) {
    const int T = (L + kRows - 1) / kRows;
    // Q and dO (all tiles), K and V (one tile), P^T and dS^T (two 64-query tiles each), lse / delta
    return 1024 + static_cast<size_t>(kBox) * (2 * T + 2 + 4) + 2 * kMaxL * sizeof(float);
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attn_short_bwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                          const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                          BwdArgs a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    BwdCtl* ctl = reinterpret_cast<BwdCtl*>(smem_raw);
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + sizeof(BwdCtl) + 1023) & ~uintptr_t(1023));
    const int L = a.L;
    const int T = (L + kRows - 1) / kRows;
    unsigned char* sQ = smem;
    unsigned char* sDO = sQ + T * kBox;
    unsigned char* sK = sDO + T * kBox;
    unsigned char* sV = sK + kBox;
    unsigned char* sPt = sV + kBox;          // [128 keys x 128 queries] as two 64-query tiles
    unsigned char* sDSt = sPt + 2 * kBox;
    float* s_lse2 = reinterpret_cast<float*>(sDSt + 2 * kBox);
    float* s_delta = s_lse2 + kMaxL;
    if (L > kMaxL ||
        reinterpret_cast<unsigned char*>(s_delta + kMaxL) - smem_raw > static_cast<ptrdiff_t>(bwd_smem_bytes(L))) {
        if (threadIdx.x == 0) atomicCAS(a.status, 0, 8);
        return;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = blockIdx.x / a.H, h = blockIdx.x % a.H;
    const int row0 = n * L;
    const int nblk = T * T;

    // tensor memory: S^T, dP^T, dV, dK, then dQ (D = 32: one D-wide slot per query tile,
    // accumulated over key tiles; D = 64: one slot reused by every block)
    constexpr uint32_t cS = 0, cDP = 128, cDV = 256, cDK = 256 + D, cDQ = 256 + 2 * D;

    if (threadIdx.x == 0) {
        mbar_init(&ctl->qdo_full, 1);
        mbar_init(&ctl->kv_full, 1);
        mbar_init(&ctl->kv_empty, 1);
        mbar_init(&ctl->sdp_full, 1);
        mbar_init(&ctl->pds_full, kSoftWarps);
        mbar_init(&ctl->mma_done, 1);
        mbar_init(&ctl->dkv_full, 1);
        mbar_init(&ctl->dkv_free, kSoftWarps);
        mbar_init(&ctl->dq_free, kSoftWarps);
        ctl->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == kProdWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&ctl->tmem_base)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;

    if (warp == kProdWarp) {
        if (lane == 0) {
            mbar_expect_tx(&ctl->qdo_full, 2 * T * kBox);
            for (int t = 0; t < T; ++t) {
                tma_load_2d(&tq, &ctl->qdo_full, sQ + t * kBox, a.qcol + h * D, row0 + t * kRows);
                tma_load_2d(&tdo, &ctl->qdo_full, sDO + t * kBox, a.docol + h * D, row0 + t * kRows);
            }
            for (int kt = 0; kt < T; ++kt) {
                if (kt > 0 && !mbar_wait(&ctl->kv_empty, (kt - 1) & 1, &ctl->abort)) {
                    ctl->abort = 1;
                    atomicCAS(a.status, 0, 1);
                    break;
                }
                mbar_expect_tx(&ctl->kv_full, 2 * kBox);
                tma_load_2d(&tk, &ctl->kv_full, sK, a.kcol + h * D, row0 + kt * kRows);
                tma_load_2d(&tv, &ctl->kv_full, sV, a.vcol + h * D, row0 + kt * kRows);
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            constexpr uint32_t idesc_t = instr_desc(false, false, kRows);   // S^T / dP^T
            constexpr uint32_t idesc_kv = instr_desc(false, true, D);        // dV / dK
            constexpr uint32_t idesc_q = instr_desc(true, true, D);          // dQ (dS read MN-major)
            const uint32_t q = smem_u32(sQ), dob = smem_u32(sDO), k = smem_u32(sK), v = smem_u32(sV);
            const uint32_t pt = smem_u32(sPt), dst = smem_u32(sDSt);
            bool ok = mbar_wait(&ctl->qdo_full, 0, &ctl->abort);
            for (int kt = 0; ok && kt < T; ++kt) {
                ok = mbar_wait(&ctl->kv_full, kt & 1, &ctl->abort);
                if (!ok) break;
                tc_fence_after();
                for (int qt = 0; qt < T; ++qt) {
                    const int blk = kt * T + qt;
                    const uint32_t qb = q + qt * kBox, db = dob + qt * kBox;
#pragma unroll
                    for (int kk = 0; kk < D / 16; ++kk)
                        tc_mma(tmem + cS, operand_desc<false>(k, kk), operand_desc<false>(qb, kk), idesc_t, kk > 0);
#pragma unroll
                    for (int kk = 0; kk < D / 16; ++kk)
                        tc_mma(tmem + cDP, operand_desc<false>(v, kk), operand_desc<false>(db, kk), idesc_t, kk > 0);
                    tc_commit(&ctl->sdp_full);
                    ok = mbar_wait(&ctl->pds_full, blk & 1, &ctl->abort);   // P^T, dS^T in smem; S^T, dP^T read
                    if (!ok) break;
                    if (qt == 0 && kt > 0) {
                        ok = mbar_wait(&ctl->dkv_free, (kt - 1) & 1, &ctl->abort);   // dV / dK of kt-1 read out
                        if (!ok) break;
                    }
                    if (D == 64 && blk > 0) {
                        ok = mbar_wait(&ctl->dq_free, (blk - 1) & 1, &ctl->abort);   // previous dQ part read out
                        if (!ok) break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int j = 0; j < kRows / 16; ++j) {
                        const uint64_t ap = smem_desc(pt + (j >> 2) * kBox + (j & 3) * 32, 16, 1024);
                        const uint64_t ad = smem_desc(dst + (j >> 2) * kBox + (j & 3) * 32, 16, 1024);
                        tc_mma(tmem + cDV, ap, smem_desc(db + j * 2048, 8192, 1024), idesc_kv, (qt > 0 || j > 0));
                        tc_mma(tmem + cDK, ad, smem_desc(qb + j * 2048, 8192, 1024), idesc_kv, (qt > 0 || j > 0));
                    }
                    const uint32_t dq_col = D == 32 ? cDQ + 32 * qt : cDQ;
#pragma unroll
                    for (int j = 0; j < kRows / 16; ++j)
                        tc_mma(tmem + dq_col, smem_desc(dst + j * 2048, kBox, 1024),
                               smem_desc(k + j * 2048, 8192, 1024), idesc_q, (D == 32 ? (kt > 0 || j > 0) : j > 0));
                    tc_commit(&ctl->mma_done);
                    if (qt == T - 1) {
                        tc_commit(&ctl->dkv_full);
                        tc_commit(&ctl->kv_empty);
                    }
                }
            }
            if (!ok) {
                ctl->abort = 1;
                atomicCAS(a.status, 0, 2);
            }
        }
    } else {
        // warp w: TMEM lane quadrant w % 4 (thread = key row r for the transposed products, query
        // row r for dQ) and half w / 4: query columns [64 * half, +64) of each block, output columns
        // [half * D / 2, +D / 2) of dV / dK / dQ
        const int quad = warp & 3, half = warp >> 2;
        const int r = 32 * quad + lane;
        const uint32_t lane_off = static_cast<uint32_t>(32 * quad) << 16;
        const float* lse = a.lse + (static_cast<int64_t>(n) * a.H + h) * L;
        const float* delta = a.delta + (static_cast<int64_t>(n) * a.H + h) * L;
        for (int i = threadIdx.x; i < kMaxL; i += kSoftThreads) {
            s_lse2[i] = i < L ? lse[i] * kLog2e : __int_as_float(0x7f800000);   // +inf: P = 0 past the sequence
            s_delta[i] = i < L ? delta[i] : 0.f;
        }
        soft_sync_and(true);
        float* dq_acc = a.dq_acc + (static_cast<int64_t>(n) * a.H + h) * L * 64;
        bool ok = true;
        for (int kt = 0; ok && kt < T; ++kt) {
            const bool kvalid = kt * kRows + r < L;
            for (int qt = 0; qt < T; ++qt) {
                const int blk = kt * T + qt;
                if (!mbar_wait(&ctl->sdp_full, blk & 1, &ctl->abort) ||
                    (blk > 0 && !mbar_wait(&ctl->mma_done, (blk - 1) & 1, &ctl->abort))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const int qc = 64 * half;                       // this half's query columns in the block
                // 16-byte broadcast reads of the per-query log-sum-exp / delta; 32 columns of S^T and
                // dP^T per tensor-memory round trip; the exponential is computed for every key row and
                // zeroed after (no predicated MUFU work)
                const float4* l2v = reinterpret_cast<const float4*>(s_lse2 + qt * kRows + qc);
                const float4* dlv = reinterpret_cast<const float4*>(s_delta + qt * kRows + qc);
                const float sl = a.scale_log2;
                const float keep = kvalid ? 1.f : 0.f;
#pragma unroll
                for (int piece = 0; piece < 2; ++piece) {
                    float sv[32], dp[32];
                    tmem_ld32x2(tmem + cS + lane_off + qc + 32 * piece, tmem + cDP + lane_off + qc + 32 * piece, sv, dp);
#pragma unroll
                    for (int g = 0; g < 4; ++g) {
                        uint32_t wp[4], wd[4];
                        const float4 la = l2v[8 * piece + 2 * g], lb = l2v[8 * piece + 2 * g + 1];
                        const float4 da = dlv[8 * piece + 2 * g], db = dlv[8 * piece + 2 * g + 1];
                        const float lv[8] = {la.x, la.y, la.z, la.w, lb.x, lb.y, lb.z, lb.w};
                        const float dv[8] = {da.x, da.y, da.z, da.w, db.x, db.y, db.z, db.w};
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int c = 8 * g + 2 * i;
                            const float p0 = keep * ex2(fmaf(sv[c], sl, -lv[2 * i]));
                            const float p1 = keep * ex2(fmaf(sv[c + 1], sl, -lv[2 * i + 1]));
                            wp[i] = pack_bf16x2(p0, p1);
                            wd[i] = pack_bf16x2(p0 * (dp[c] - dv[2 * i]), p1 * (dp[c + 1] - dv[2 * i + 1]));
                        }
                        put16(sPt + half * kBox, r, 4 * piece + g, make_uint4(wp[0], wp[1], wp[2], wp[3]));
                        put16(sDSt + half * kBox, r, 4 * piece + g, make_uint4(wd[0], wd[1], wd[2], wd[3]));
                    }
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&ctl->pds_full);
                if (D == 64) {
                    // this block's dQ part: thread = query row qt*128 + r, columns [32 * half, +32)
                    if (!mbar_wait(&ctl->mma_done, blk & 1, &ctl->abort)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    float part[32];
                    tmem_ld32(tmem + cDQ + lane_off + 32 * half, part);
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&ctl->dq_free);
                    const int qrow = qt * kRows + r;
                    if (qrow < L) {
                        float4* acc = reinterpret_cast<float4*>(dq_acc + static_cast<int64_t>(qrow) * 64 + 32 * half);
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            float4 x = make_float4(part[4 * j], part[4 * j + 1], part[4 * j + 2], part[4 * j + 3]);
                            if (kt > 0) {
                                const float4 y = acc[j];
                                x.x += y.x;
                                x.y += y.y;
                                x.z += y.z;
                                x.w += y.w;
                            }
                            acc[j] = x;
                        }
                    }
                }
            }
            if (!ok) break;
            // dV / dK of this key tile are complete: thread = key row, this half's output columns
            if (!mbar_wait(&ctl->dkv_full, kt & 1, &ctl->abort)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float dvr[D / 2], dkr[D / 2];
            if (D == 32) {
                tmem_ld16(tmem + cDV + lane_off + 16 * half, dvr);
                tmem_ld16(tmem + cDK + lane_off + 16 * half, dkr);
            } else {
                tmem_ld32(tmem + cDV + lane_off + 32 * half, dvr);
                tmem_ld32(tmem + cDK + lane_off + 32 * half, dkr);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ctl->dkv_free);
            if (kvalid) {
                const int64_t row = row0 + kt * kRows + r;
                uint4* ov = reinterpret_cast<uint4*>(a.dv + row * a.lddv + a.dvcol + h * D + half * (D / 2));
                uint4* ok_ = reinterpret_cast<uint4*>(a.dk + row * a.lddk + a.dkcol + h * D + half * (D / 2));
                const float s = a.scale;
#pragma unroll
                for (int j = 0; j < D / 16; ++j) {
                    ov[j] = make_uint4(pack_bf16x2(dvr[8 * j], dvr[8 * j + 1]), pack_bf16x2(dvr[8 * j + 2], dvr[8 * j + 3]),
                                       pack_bf16x2(dvr[8 * j + 4], dvr[8 * j + 5]),
                                       pack_bf16x2(dvr[8 * j + 6], dvr[8 * j + 7]));
                    ok_[j] = make_uint4(pack_bf16x2(dkr[8 * j] * s, dkr[8 * j + 1] * s),
                                        pack_bf16x2(dkr[8 * j + 2] * s, dkr[8 * j + 3] * s),
                                        pack_bf16x2(dkr[8 * j + 4] * s, dkr[8 * j + 5] * s),
                                        pack_bf16x2(dkr[8 * j + 6] * s, dkr[8 * j + 7] * s));
                }
            }
        }
        if (ok) {
            // dQ: thread = query row qt*128 + r, this half's output columns
            if (D == 32 && !mbar_wait(&ctl->mma_done, (nblk - 1) & 1, &ctl->abort)) ok = false;
            if (ok) {
                tc_fence_after();
                for (int qt = 0; qt < T; ++qt) {
                    float dqr[D / 2];
                    const int qrow = qt * kRows + r;
                    if (D == 32) {
                        tmem_ld16(tmem + cDQ + 32 * qt + lane_off + 16 * half, dqr);
                    } else if (qrow < L) {
                        const float4* acc =
                            reinterpret_cast<const float4*>(dq_acc + static_cast<int64_t>(qrow) * 64 + 32 * half);
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const float4 y = acc[j];
                            dqr[4 * j] = y.x;
                            dqr[4 * j + 1] = y.y;
                            dqr[4 * j + 2] = y.z;
                            dqr[4 * j + 3] = y.w;
                        }
                    }
                    if (qrow < L) {
                        uint4* oq = reinterpret_cast<uint4*>(a.dq + static_cast<int64_t>(row0 + qrow) * a.lddq +
                                                             a.dqcol + h * D + half * (D / 2));
                        const float s = a.scale;
#pragma unroll
                        for (int j = 0; j < D / 16; ++j)
                            oq[j] = make_uint4(pack_bf16x2(dqr[8 * j] * s, dqr[8 * j + 1] * s),
                                               pack_bf16x2(dqr[8 * j + 2] * s, dqr[8 * j + 3] * s),
                                               pack_bf16x2(dqr[8 * j + 4] * s, dqr[8 * j + 5] * s),
                                               pack_bf16x2(dqr[8 * j + 6] * s, dqr[8 * j + 7] * s));
                    }
                }
            }
        }
        if (!ok) {
            ctl->abort = 1;
            if (lane == 0) atomicCAS(a.status, 0, 3);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kProdWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// ---------------------------------------------------------------- backward, head dim 32, pipelined
//
// The head-dim-32 backward above runs each 128 x 128 block strictly in turn (S^T / dP^T products,
// then the exponentials, then the dV / dK / dQ products), so the tensor core idles while the
// softmax warps work and the other way round.  This kernel overlaps them:
//   * work is cut into half-blocks of 128 keys x 64 queries; S^T / dP^T of half-block j + 1 are
//     issued into the second of two tensor-memory buffers before the MMA warp waits for the
//     softmax of half-block j, so the exponentials of j + 1 run while dV / dK of j are multiplied;
//   * P^T half-tiles rotate through two shared-memory buffers and dS^T blocks (both halves, which
//     the dQ product reads MN-major) through two, so the softmax never waits for the products of
//     the half-block before;
//   * dV / dK accumulate in one of two tensor-memory buffers per key tile, so the next key tile's
//     products start before the previous one is read out;
//   * Q / dO / K / V are 32-column boxes with the 64-byte swizzle (64-byte rows: exactly one head),
//     half the bytes of the 64-column boxes the kernels above share with the neighbouring head;
//   * a half-block whose 64 queries all lie past the sequence is skipped.
// Tensor memory: S^T / dP^T buffers at [0, 256), dV / dK buffers at [256, 384), dQ of query tile
// qt at 384 + 32 qt.
namespace bw2 {
constexpr int kTile = kRows * 32 * 2;       // 8 KB: 128 rows x 32 columns, 64-byte rows
constexpr int kHalfQ = 64 * 64;             // byte offset of query row 64 in a kTile
constexpr uint32_t cDKV = 256, cDQ = 384;
}

struct __align__(8) Bwd2Ctl {
    uint64_t qdo_full, kv_full[2], kv_empty[2], sdp_full[2], soft_done[2], p_free[2], ds_free[2], dkv_full[2],
        dkv_free[2], dq_done;
    uint32_t tmem_base;
    int abort;
};

__host__ __device__ constexpr size_t bwd2_smem_bytes() {
    // control block, 1024 alignment, Q + dO (3 tiles each), K + V (two buffers each), P^T (two
    // half-tiles), dS^T (two blocks of two half-tiles), log-sum-exp and delta rows
    return 1024 + 1024 + static_cast<size_t>(bw2::kTile) * (6 + 4) + static_cast<size_t>(kBox) * (2 + 4) +
           2 * kMaxL * sizeof(float);
}

// Shared-memory matrix descriptor, 64-byte swizzle (sm_100 layout type 4).
__device__ __forceinline__ uint64_t smem_desc64(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr >> 4) & 0x3fff);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3fff) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3fff) << 32;
    d |= 1ull << 46;
    d |= 4ull << 61;
    return d;
}
// 16-wide K slice kk of a K-major 64-byte-row tile (rows x 32 columns): 8-row groups 512 B apart
__device__ __forceinline__ uint64_t kmajor64(uint32_t tile, int kk) { return smem_desc64(tile + kk * 32, 16, 512); }
// 16-row K slice j of the same tile read MN-major (the 32 columns are the N side)
__device__ __forceinline__ uint64_t mnmajor64(uint32_t tile, int j) { return smem_desc64(tile + j * 1024, 8192, 512); }

// the number of 64-query halves of query tile qt that hold a query of the sequence
__device__ __forceinline__ int bw2_halves(int qt, int T, int L) { return (qt == T - 1 && L - qt * kRows <= 64) ? 1 : 2; }

__global__ void __launch_bounds__(kThreads, 1)
    attn_short_bwd2_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                           const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo, BwdArgs a) {
    using namespace bw2;
    constexpr int D = 32;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    Bwd2Ctl* ctl = reinterpret_cast<Bwd2Ctl*>(smem_raw);
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + sizeof(Bwd2Ctl) + 1023) & ~uintptr_t(1023));
    const int L = a.L;
    const int T = (L + kRows - 1) / kRows;
    unsigned char* sQ = smem;
    unsigned char* sDO = sQ + 3 * kTile;
    unsigned char* sK = sDO + 3 * kTile;       // two buffers
    unsigned char* sV = sK + 2 * kTile;        // two buffers
    unsigned char* sP = sV + 2 * kTile;        // two 16 KB half-tiles [128 keys x 64 queries]
    unsigned char* sDS = sP + 2 * kBox;        // two blocks of two half-tiles
    float* s_lse2 = reinterpret_cast<float*>(sDS + 4 * kBox);
    float* s_delta = s_lse2 + kMaxL;
    if (L > kMaxL ||
        reinterpret_cast<unsigned char*>(s_delta + kMaxL) - smem_raw > static_cast<ptrdiff_t>(bwd2_smem_bytes())) {
        if (threadIdx.x == 0) atomicCAS(a.status, 0, 8);
        return;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = blockIdx.x / a.H, h = blockIdx.x % a.H;
    const int row0 = n * L;
    int J = 0;   // half-blocks: T key tiles x the valid halves of the T query tiles
    for (int qt = 0; qt < T; ++qt) J += bw2_halves(qt, T, L);
    J *= T;

    if (threadIdx.x == 0) {
        mbar_init(&ctl->qdo_full, 1);
        for (int x = 0; x < 2; ++x) {
            mbar_init(&ctl->kv_full[x], 1);
            mbar_init(&ctl->kv_empty[x], 1);
            mbar_init(&ctl->sdp_full[x], 1);
            mbar_init(&ctl->soft_done[x], kSoftWarps);
            mbar_init(&ctl->p_free[x], 1);
            mbar_init(&ctl->ds_free[x], 1);
            mbar_init(&ctl->dkv_full[x], 1);
            mbar_init(&ctl->dkv_free[x], kSoftWarps);
        }
        mbar_init(&ctl->dq_done, 1);
        ctl->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == kProdWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&ctl->tmem_base)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;

    if (warp == kProdWarp) {
        if (lane == 0) {
            mbar_expect_tx(&ctl->qdo_full, 2 * T * kTile);
            for (int t = 0; t < T; ++t) {
                tma_load_2d(&tq, &ctl->qdo_full, sQ + t * kTile, a.qcol + h * D, row0 + t * kRows);
                tma_load_2d(&tdo, &ctl->qdo_full, sDO + t * kTile, a.docol + h * D, row0 + t * kRows);
            }
            for (int kt = 0; kt < T; ++kt) {
                const int x = kt & 1;
                if (kt >= 2 && !mbar_wait(&ctl->kv_empty[x], ((kt >> 1) - 1) & 1, &ctl->abort)) {
                    ctl->abort = 1;
                    atomicCAS(a.status, 0, 1);
                    break;
                }
                mbar_expect_tx(&ctl->kv_full[x], 2 * kTile);
                tma_load_2d(&tk, &ctl->kv_full[x], sK + x * kTile, a.kcol + h * D, row0 + kt * kRows);
                tma_load_2d(&tv, &ctl->kv_full[x], sV + x * kTile, a.vcol + h * D, row0 + kt * kRows);
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            constexpr uint32_t idesc_sdp = instr_desc(false, false, 64);   // S^T / dP^T: 128 keys x 64 queries
            constexpr uint32_t idesc_kv = instr_desc(false, true, D);      // dV / dK
            constexpr uint32_t idesc_q = instr_desc(true, true, D);        // dQ (dS read MN-major)
            const uint32_t q = smem_u32(sQ), dob = smem_u32(sDO), k = smem_u32(sK), v = smem_u32(sV);
            const uint32_t pt = smem_u32(sP), dst = smem_u32(sDS);
            auto issue_sdp = [&](int x, int kt, int qt, int hb) {
                const uint32_t kb = k + (kt & 1) * kTile, vb = v + (kt & 1) * kTile;
                const uint32_t qb = q + qt * kTile + hb * kHalfQ, db = dob + qt * kTile + hb * kHalfQ;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    tc_mma(tmem + 128 * x, kmajor64(kb, kk), kmajor64(qb, kk), idesc_sdp, kk > 0);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    tc_mma(tmem + 128 * x + 64, kmajor64(vb, kk), kmajor64(db, kk), idesc_sdp, kk > 0);
                tc_commit(&ctl->sdp_full[x]);
            };
            bool ok = mbar_wait(&ctl->qdo_full, 0, &ctl->abort) && mbar_wait(&ctl->kv_full[0], 0, &ctl->abort);
            if (ok) {
                tc_fence_after();
                issue_sdp(0, 0, 0, 0);
            }
            int kt = 0, qt = 0, hb = 0, blk = 0;
            for (int j = 0; ok && j < J; ++j) {
                int nkt = kt, nqt = qt, nhb = hb + 1;
                if (nhb == bw2_halves(qt, T, L)) {
                    nhb = 0;
                    if (++nqt == T) {
                        nqt = 0;
                        ++nkt;
                    }
                }
                if (j + 1 < J) {
                    // the softmax of half-block j - 1 has read buffer (j + 1) & 1 (awaited last iteration)
                    if (nkt != kt && !(ok = mbar_wait(&ctl->kv_full[nkt & 1], (nkt >> 1) & 1, &ctl->abort))) break;
                    tc_fence_after();
                    issue_sdp((j + 1) & 1, nkt, nqt, nhb);
                }
                if (!(ok = mbar_wait(&ctl->soft_done[j & 1], (j >> 1) & 1, &ctl->abort))) break;
                tc_fence_after();
                const bool first = qt == 0 && hb == 0;     // first half-block of this key tile
                if (first && kt >= 2) {
                    if (!(ok = mbar_wait(&ctl->dkv_free[kt & 1], ((kt >> 1) - 1) & 1, &ctl->abort))) break;
                    tc_fence_after();
                }
                const uint32_t dv = tmem + cDKV + 64 * (kt & 1), dk = dv + 32;
                const uint32_t pb = pt + (j & 1) * kBox, dsb = dst + (blk & 1) * 2 * kBox;
                const uint32_t qb = q + qt * kTile + hb * kHalfQ, db = dob + qt * kTile + hb * kHalfQ;
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint32_t acc = (first && kk == 0) ? 0u : 1u;
                    tc_mma(dv, smem_desc(pb + kk * 32, 16, 1024), mnmajor64(db, kk), idesc_kv, acc);
                    tc_mma(dk, smem_desc(dsb + hb * kBox + kk * 32, 16, 1024), mnmajor64(qb, kk), idesc_kv, acc);
                }
                tc_commit(&ctl->p_free[j & 1]);
                if (hb == bw2_halves(qt, T, L) - 1) {
                    // dQ_qt += dS K_kt over the block's 128 keys (a skipped half only feeds query rows past
                    // the sequence, which are never stored)
                    const uint32_t kb = k + (kt & 1) * kTile;
#pragma unroll
                    for (int jj = 0; jj < kRows / 16; ++jj)
                        tc_mma(tmem + cDQ + 32 * qt, smem_desc(dsb + jj * 2048, kBox, 1024), mnmajor64(kb, jj), idesc_q,
                               (kt > 0 || jj > 0) ? 1u : 0u);
                    tc_commit(&ctl->ds_free[blk & 1]);
                    if (qt == T - 1) {
                        tc_commit(&ctl->dkv_full[kt & 1]);
                        tc_commit(&ctl->kv_empty[kt & 1]);
                    }
                    ++blk;
                }
                kt = nkt;
                qt = nqt;
                hb = nhb;
            }
            if (ok) tc_commit(&ctl->dq_done);
            if (!ok) {
                ctl->abort = 1;
                atomicCAS(a.status, 0, 2);
            }
        }
    } else {
        // warp w: TMEM lane quadrant w % 4 (thread = key row r of the transposed products, query row r
        // of dQ) and half w / 4: query columns [32 * half, +32) of each half-block, output columns
        // [16 * half, +16) of dV / dK / dQ
        const int quad = warp & 3, half = warp >> 2;
        const int r = 32 * quad + lane;
        const uint32_t lane_off = static_cast<uint32_t>(32 * quad) << 16;
        const float* lse = a.lse + (static_cast<int64_t>(n) * a.H + h) * L;
        const float* delta = a.delta + (static_cast<int64_t>(n) * a.H + h) * L;
        for (int i = threadIdx.x; i < kMaxL; i += kSoftThreads) {
            s_lse2[i] = i < L ? lse[i] * kLog2e : __int_as_float(0x7f800000);   // +inf: P = 0 past the sequence
            s_delta[i] = i < L ? delta[i] : 0.f;
        }
        soft_sync_and(true);
        bool ok = true;
        int kt = 0, qt = 0, hb = 0, blk = 0;
        const float sl = a.scale_log2;
        for (int j = 0; j < J; ++j) {
            if (!mbar_wait(&ctl->sdp_full[j & 1], (j >> 1) & 1, &ctl->abort) ||
                (j >= 2 && !mbar_wait(&ctl->p_free[j & 1], ((j >> 1) - 1) & 1, &ctl->abort)) ||
                (hb == 0 && blk >= 2 && !mbar_wait(&ctl->ds_free[blk & 1], ((blk >> 1) - 1) & 1, &ctl->abort))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const float keep = kt * kRows + r < L ? 1.f : 0.f;
            const int q0 = qt * kRows + hb * 64 + 32 * half;      // this thread's first query
            const float4* l2v = reinterpret_cast<const float4*>(s_lse2 + q0);
            const float4* dlv = reinterpret_cast<const float4*>(s_delta + q0);
            float sv[32], dp[32];
            tmem_ld32x2(tmem + 128 * (j & 1) + lane_off + 32 * half, tmem + 128 * (j & 1) + 64 + lane_off + 32 * half,
                        sv, dp);
            unsigned char* pbox = sP + (j & 1) * kBox;
            unsigned char* dbox = sDS + (blk & 1) * 2 * kBox + hb * kBox;
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                uint32_t wp[4], wd[4];
                const float4 la = l2v[2 * g], lb = l2v[2 * g + 1];
                const float4 da = dlv[2 * g], db = dlv[2 * g + 1];
                const float lv[8] = {la.x, la.y, la.z, la.w, lb.x, lb.y, lb.z, lb.w};
                const float dv[8] = {da.x, da.y, da.z, da.w, db.x, db.y, db.z, db.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int c = 8 * g + 2 * i;
                    const float p0 = keep * ex2(fmaf(sv[c], sl, -lv[2 * i]));
                    const float p1 = keep * ex2(fmaf(sv[c + 1], sl, -lv[2 * i + 1]));
                    wp[i] = pack_bf16x2(p0, p1);
                    wd[i] = pack_bf16x2(p0 * (dp[c] - dv[2 * i]), p1 * (dp[c + 1] - dv[2 * i + 1]));
                }
                put16(pbox, r, 4 * half + g, make_uint4(wp[0], wp[1], wp[2], wp[3]));
                put16(dbox, r, 4 * half + g, make_uint4(wd[0], wd[1], wd[2], wd[3]));
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ctl->soft_done[j & 1]);
            const bool block_end = hb == bw2_halves(qt, T, L) - 1;
            if (block_end && qt == T - 1) {
                // dV / dK of key tile kt complete: thread = key row, this half's 16 output columns
                if (!mbar_wait(&ctl->dkv_full[kt & 1], (kt >> 1) & 1, &ctl->abort)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                float dvr[16], dkr[16];
                tmem_ld16(tmem + cDKV + 64 * (kt & 1) + lane_off + 16 * half, dvr);
                tmem_ld16(tmem + cDKV + 64 * (kt & 1) + 32 + lane_off + 16 * half, dkr);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&ctl->dkv_free[kt & 1]);
                if (kt * kRows + r < L) {
                    const int64_t row = row0 + kt * kRows + r;
                    uint4* ov = reinterpret_cast<uint4*>(a.dv + row * a.lddv + a.dvcol + h * D + half * 16);
                    uint4* okp = reinterpret_cast<uint4*>(a.dk + row * a.lddk + a.dkcol + h * D + half * 16);
                    const float sc = a.scale;
#pragma unroll
                    for (int i = 0; i < 2; ++i) {
                        ov[i] = make_uint4(pack_bf16x2(dvr[8 * i], dvr[8 * i + 1]), pack_bf16x2(dvr[8 * i + 2], dvr[8 * i + 3]),
                                           pack_bf16x2(dvr[8 * i + 4], dvr[8 * i + 5]),
                                           pack_bf16x2(dvr[8 * i + 6], dvr[8 * i + 7]));
                        okp[i] = make_uint4(pack_bf16x2(dkr[8 * i] * sc, dkr[8 * i + 1] * sc),
                                            pack_bf16x2(dkr[8 * i + 2] * sc, dkr[8 * i + 3] * sc),
                                            pack_bf16x2(dkr[8 * i + 4] * sc, dkr[8 * i + 5] * sc),
                                            pack_bf16x2(dkr[8 * i + 6] * sc, dkr[8 * i + 7] * sc));
                    }
                }
            }
            if (block_end) ++blk;
            if (++hb == bw2_halves(qt, T, L)) {
                hb = 0;
                if (++qt == T) {
                    qt = 0;
                    ++kt;
                }
            }
        }
        if (ok && mbar_wait(&ctl->dq_done, 0, &ctl->abort)) {
            tc_fence_after();
            for (int t = 0; t < T; ++t) {
                float dqr[16];
                tmem_ld16(tmem + cDQ + 32 * t + lane_off + 16 * half, dqr);
                const int qrow = t * kRows + r;
                if (qrow < L) {
                    uint4* oq = reinterpret_cast<uint4*>(a.dq + static_cast<int64_t>(row0 + qrow) * a.lddq + a.dqcol +
                                                         h * D + half * 16);
                    const float sc = a.scale;
#pragma unroll
                    for (int i = 0; i < 2; ++i)
                        oq[i] = make_uint4(pack_bf16x2(dqr[8 * i] * sc, dqr[8 * i + 1] * sc),
                                           pack_bf16x2(dqr[8 * i + 2] * sc, dqr[8 * i + 3] * sc),
                                           pack_bf16x2(dqr[8 * i + 4] * sc, dqr[8 * i + 5] * sc),
                                           pack_bf16x2(dqr[8 * i + 6] * sc, dqr[8 * i + 7] * sc));
                }
            }
        } else {
            ok = false;
        }
        if (!ok) {
            ctl->abort = 1;
            if (lane == 0) atomicCAS(a.status, 0, 3);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kProdWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// delta[n, h, i] = sum_d dO[row, docol + h*D + d] * O[row, ocol + h*D + d], row = n*L + i
template <int D>
__global__ void attn_delta_kernel(const __nv_bfloat16* __restrict__ dout, int64_t lddo, int docol,
                                  const __nv_bfloat16* __restrict__ o, int64_t ldo, int ocol, float* __restrict__ delta,
                                  int N, int L, int H) {
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<int64_t>(N) * L * H) return;
    const int h = static_cast<int>(idx % H);
    const int64_t row = idx / H;
    const __nv_bfloat16* a = dout + row * lddo + docol + h * D;
    const __nv_bfloat16* b = o + row * ldo + ocol + h * D;
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < D; j += 8) {
        float x[8], y[8];
        load8(a + j, x);
        load8(b + j, y);
#pragma unroll
        for (int i = 0; i < 8; ++i) s += x[i] * y[i];
    }
    const int n = static_cast<int>(row / L), i = static_cast<int>(row % L);
    delta[(static_cast<int64_t>(n) * H + h) * L + i] = s;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (fn == nullptr) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 128-row x 64-column boxes of a row-major bf16 matrix [rows, cols] with row pitch ld (elements)
cudaError_t make_map(CUtensorMap* tm, const void* base, int64_t cols, int64_t rows, int64_t ld) {
    if (reinterpret_cast<uintptr_t>(base) % 16 != 0 || ld % 8 != 0 || cols > ld) return cudaErrorInvalidValue;
    auto fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
    cuuint32_t box[2] = {64, kRows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        std::fprintf(stderr, "attn_short: cuTensorMapEncodeTiled failed (%d)\n", static_cast<int>(r));
        return cudaErrorInvalidValue;
    }
    return cudaSuccess;
}

// 128-row x 32-column boxes (one head-dim-32 head: 64-byte rows) with the 64-byte swizzle
cudaError_t make_map32(CUtensorMap* tm, const void* base, int64_t cols, int64_t rows, int64_t ld) {
    if (reinterpret_cast<uintptr_t>(base) % 16 != 0 || ld % 8 != 0 || cols > ld) return cudaErrorInvalidValue;
    auto fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
    cuuint32_t box[2] = {32, kRows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        std::fprintf(stderr, "attn_short: cuTensorMapEncodeTiled (32-column boxes) failed (%d)\n", static_cast<int>(r));
        return cudaErrorInvalidValue;
    }
    return cudaSuccess;
}

// the shared-memory opt-in, once per (kernel, device): Tag makes every kernel its own instantiation
// (the D = 32 and D = 64 kernels have the same function-pointer type, so the flags cannot be keyed
// by that type alone)
template <typename Tag, typename K>
cudaError_t ensure_smem(K kern, size_t bytes, int dev) {
    static bool set[64] = {};
    if (set[dev & 63]) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e == cudaSuccess) set[dev & 63] = true;
    return e;
}
template <bool Bwd, int D>
struct KernelTag {};

// forward kernel: 1 = whole score row per (sequence, head), 2 = ping-pong warpgroups (default)
int g_fwd_variant = 2;
// head-dim-32 backward kernel: 1 = one block at a time, 2 = pipelined half-blocks (default)
int g_bwd_variant = 2;

}  // namespace

bool attn_short_supported(int L, int D) { return L >= 1 && L <= kMaxL && (D == 32 || D == 64); }

void attn_short_set_fwd_variant(int v) { g_fwd_variant = v == 1 ? 1 : 2; }
int attn_short_fwd_variant() { return g_fwd_variant; }
void attn_short_set_bwd_variant(int v) { g_bwd_variant = v == 1 ? 1 : 2; }
int attn_short_bwd_variant() { return g_bwd_variant; }

cudaError_t launch_attn_short_fwd(const AttnOperand& q, const AttnOperand& k, const AttnOperand& v, int nseq, int L,
                                  int H, int D, void* o, int64_t ldo, int ocol, float* lse, float scale, int* status,
                                  cudaStream_t st) {
    if (nseq == 0 || L == 0) return cudaSuccess;
    if (!attn_short_supported(L, D)) return cudaErrorInvalidValue;
    if (reinterpret_cast<uintptr_t>(o) % 16 != 0 || ldo % 8 != 0 || ocol % 8 != 0) return cudaErrorInvalidValue;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaSetDevice(dev);   // the driver-API encode needs a current context
    if (e != cudaSuccess) return e;
    const int64_t rows = static_cast<int64_t>(nseq) * L;
    CUtensorMap mq, mk, mv;
    if ((e = make_map(&mq, q.base, q.cols, rows, q.ld)) != cudaSuccess) return e;
    if ((e = make_map(&mk, k.base, k.cols, rows, k.ld)) != cudaSuccess) return e;
    if ((e = make_map(&mv, v.base, v.cols, rows, v.ld)) != cudaSuccess) return e;
    FwdArgs a{static_cast<__nv_bfloat16*>(o), ldo, lse, status, L, H, q.col, k.col, v.col, ocol, scale * kLog2e};
    if (g_fwd_variant == 2) {
        const size_t smem2 = fwd2_smem_bytes();
        if (D == 32) {
            if ((e = ensure_smem<KernelTag<false, 33>>(attn_short_fwd2_kernel<32>, smem2, dev)) != cudaSuccess) return e;
            attn_short_fwd2_kernel<32><<<nseq * ((H + 1) / 2), pp::kThreadsPP, smem2, st>>>(mq, mk, mv, a);
        } else {
            if ((e = ensure_smem<KernelTag<false, 65>>(attn_short_fwd2_kernel<64>, smem2, dev)) != cudaSuccess) return e;
            attn_short_fwd2_kernel<64><<<nseq * H, pp::kThreadsPP, smem2, st>>>(mq, mk, mv, a);
        }
        return cudaGetLastError();
    }
    const size_t smem = fwd_smem_bytes(kMaxL);   // one CTA per SM (the kernel takes all of tensor memory)
    if (D == 32) {
        if ((e = ensure_smem<KernelTag<false, 32>>(attn_short_fwd_kernel<32>, smem, dev)) != cudaSuccess) return e;
        attn_short_fwd_kernel<32><<<nseq * H, kThreads, smem, st>>>(mq, mk, mv, a);
    } else {
        if ((e = ensure_smem<KernelTag<false, 64>>(attn_short_fwd_kernel<64>, smem, dev)) != cudaSuccess) return e;
        attn_short_fwd_kernel<64><<<nseq * H, kThreads, smem, st>>>(mq, mk, mv, a);
    }
    return cudaGetLastError();
}

cudaError_t launch_attn_short_bwd(const AttnOperand& q, const AttnOperand& k, const AttnOperand& v,
                                  const AttnOperand& dout, const void* o, int64_t ldo, int ocol, const float* lse,
                                  float* delta, float* dq_acc, int nseq, int L, int H, int D, void* dq, int64_t lddq,
                                  int dqcol, void* dk, int64_t lddk, int dkcol, void* dv, int64_t lddv, int dvcol,
                                  float scale, int* status, cudaStream_t st) {
    if (nseq == 0 || L == 0) return cudaSuccess;
    if (!attn_short_supported(L, D)) return cudaErrorInvalidValue;
    for (auto* p : {dq, dk, dv})
        if (reinterpret_cast<uintptr_t>(p) % 16 != 0) return cudaErrorInvalidValue;
    if (lddq % 8 || lddk % 8 || lddv % 8 || dqcol % 8 || dkcol % 8 || dvcol % 8 || ldo % 8 || ocol % 8)
        return cudaErrorInvalidValue;
    if (D == 64 && dq_acc == nullptr) return cudaErrorInvalidValue;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaSetDevice(dev);
    if (e != cudaSuccess) return e;
    const int64_t rows = static_cast<int64_t>(nseq) * L;
    {
        const int64_t n = rows * H;
        const int threads = 256;
        const unsigned blocks = static_cast<unsigned>((n + threads - 1) / threads);
        if (D == 32)
            attn_delta_kernel<32><<<blocks, threads, 0, st>>>(static_cast<const __nv_bfloat16*>(dout.base), dout.ld,
                                                               dout.col, static_cast<const __nv_bfloat16*>(o), ldo, ocol,
                                                               delta, nseq, L, H);
        else
            attn_delta_kernel<64><<<blocks, threads, 0, st>>>(static_cast<const __nv_bfloat16*>(dout.base), dout.ld,
                                                               dout.col, static_cast<const __nv_bfloat16*>(o), ldo, ocol,
                                                               delta, nseq, L, H);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    BwdArgs a{lse,   delta, dq_acc, static_cast<__nv_bfloat16*>(dq), static_cast<__nv_bfloat16*>(dk),
              static_cast<__nv_bfloat16*>(dv), lddq, lddk, lddv, dqcol, dkcol, dvcol, status, L, H, q.col, k.col,
              v.col, dout.col, scale * kLog2e, scale};
    CUtensorMap mq, mk, mv, mdo;
    if (D == 32 && g_bwd_variant == 2) {
        if ((e = make_map32(&mq, q.base, q.cols, rows, q.ld)) != cudaSuccess) return e;
        if ((e = make_map32(&mk, k.base, k.cols, rows, k.ld)) != cudaSuccess) return e;
        if ((e = make_map32(&mv, v.base, v.cols, rows, v.ld)) != cudaSuccess) return e;
        if ((e = make_map32(&mdo, dout.base, dout.cols, rows, dout.ld)) != cudaSuccess) return e;
        constexpr size_t smem2 = bwd2_smem_bytes();
        if ((e = ensure_smem<KernelTag<true, 33>>(attn_short_bwd2_kernel, smem2, dev)) != cudaSuccess) return e;
        attn_short_bwd2_kernel<<<nseq * H, kThreads, smem2, st>>>(mq, mk, mv, mdo, a);
        return cudaGetLastError();
    }
    if ((e = make_map(&mq, q.base, q.cols, rows, q.ld)) != cudaSuccess) return e;
    if ((e = make_map(&mk, k.base, k.cols, rows, k.ld)) != cudaSuccess) return e;
    if ((e = make_map(&mv, v.base, v.cols, rows, v.ld)) != cudaSuccess) return e;
    if ((e = make_map(&mdo, dout.base, dout.cols, rows, dout.ld)) != cudaSuccess) return e;
    const size_t smem = bwd_smem_bytes(kMaxL);
    if (D == 32) {
        if ((e = ensure_smem<KernelTag<true, 32>>(attn_short_bwd_kernel<32>, smem, dev)) != cudaSuccess) return e;
        attn_short_bwd_kernel<32><<<nseq * H, kThreads, smem, st>>>(mq, mk, mv, mdo, a);
    } else {
        if ((e = ensure_smem<KernelTag<true, 64>>(attn_short_bwd_kernel<64>, smem, dev)) != cudaSuccess) return e;
        attn_short_bwd_kernel<64><<<nseq * H, kThreads, smem, st>>>(mq, mk, mv, mdo, a);
    }
    return cudaGetLastError();
}

size_t attn_short_smem_bytes(bool backward) { return backward ? bwd_smem_bytes(kMaxL) : fwd_smem_bytes(kMaxL); }

}  // namespace mmltk
