// Scaled dot-product attention forward on the 5th-generation tensor cores (tcgen05), head dim 64,
// reading q / k / v straight out of the packed ViT projection [N, L, 3, H, 64]
// (reference: `at::scaled_dot_product_attention`, `src/rfdetr/layers/model.cpp:498`).
//
// One CTA per (128-query tile, head, sequence), five warps:
//   warp 4   lane 0: TMA producer: the Q tile once, then 128-key K tiles into a two-stage
//            ring and V tiles into one stage, all 128-byte swizzled 64-wide boxes of the packed
//            projection (the column offset picks q / k / v and the head); also owns TMEM;
//   warp 4   lane 1: MMA issuer: S = Q.K^T (M=128, N=128, K=64) into TMEM columns 0-127,
//            then O += P.V (M=128, N=64, K=128; P from shared memory, V MN-major) into
//            columns 128-191;
//   warps 0-3 softmax: thread = query row = TMEM lane.  The S row (128 columns) is read from
//            TMEM into registers in one round; p = 2^(s*scale*log2e - m) is written as bf16
//            into the swizzled K-major P tile the next MMA reads.  O accumulates across key
//            tiles in TMEM; it is rescaled (tcgen05.ld / st) only when a row maximum grows by
//            more than 2^8 over the reference maximum in use (lazy rescaling), and normalised
//            by the row sum at the end.
// Keys past the sequence length are masked by index, so the 128-row boxes may run into the
// next sequence (or past the tensor, where TMA zero-fills).  Shared memory (Q 16 KB, K 2x16 KB,
// V 16 KB, P 32 KB) and TMEM (256 columns) are sized for two CTAs per SM.  Every mbarrier wait is
// bounded; on timeout the kernel records a code in the status word and leaves.
#include <cudaTypedefs.h>

#include <cstdio>

#include "common.cuh"
#include "launch_api.h"
#include "tcgen05.cuh"

namespace mmltk {

namespace {

using namespace tc;

constexpr int kRows = 128;                  // queries per CTA, keys per tile
constexpr int kHd = 64;                     // head dim (one 128-byte swizzle row)
constexpr int kTile = kRows * kHd * 2;      // 16 KB: one Q / K / V box
constexpr int kKStages = 2;
constexpr int kThreads = 160;
constexpr int kTmemCols = 256;
constexpr int kSCol = 0, kOCol = 128;
constexpr int kVStages = 1;   // two V stages (112 KB) measured slower: the SM then holds one CTA
// tiles + 1 KB: the control block sits in the alignment slack below the 1024-aligned tiles
constexpr size_t kSmemBytes = 1024 + kTile * (1 + kKStages + kVStages + 2);

struct __align__(8) AttnCtl {
    uint64_t q_full;
    uint64_t k_full[kKStages];
    uint64_t k_empty[kKStages];
    uint64_t v_full[kVStages], v_empty[kVStages];
    uint64_t s_full, pv_full;
    uint64_t p_full;               // 4 arrivals: one per softmax warp
    uint32_t tmem_base;
    int abort;
};

static_assert(sizeof(AttnCtl) <= 128, "control block must fit the alignment slack");

struct AttnArgs {
    __nv_bfloat16* o;     // [N*L, C] (row pitch ldo)
    float* lse;           // optional [N, H, L] natural-log row log-sum-exp
    int* status;
    int L, H, C;
    int64_t ldo;
    float scale_log2;     // softmax scale * log2(e)
};

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// kMinBlocks = 2 caps the kernel at 168 registers (each SM sub-partition holds 16384: three
// warps of two co-resident CTAs), with a few spilled; kMinBlocks = 1 uses 194 without spills,
// one CTA per SM.
template <int kMinBlocks>
__global__ void __launch_bounds__(kThreads, kMinBlocks) attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm, AttnArgs a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    AttnCtl* ctl = reinterpret_cast<AttnCtl*>(smem_raw);
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + sizeof(AttnCtl) + 1023) & ~uintptr_t(1023));
    unsigned char* sQ = smem;
    unsigned char* sK = sQ + kTile;
    unsigned char* sV = sK + kKStages * kTile;
    unsigned char* sP = sV + kVStages * kTile;      // two 64-key K-major tiles

    // the layout above fits kSmemBytes when the dynamic window is 128-byte aligned; anything
    // else is reported instead of overrunning (uniform across the CTA, before any barrier)
    if (smem - smem_raw + kTile * (1 + kKStages + kVStages + 2) > kSmemBytes) {
        if (threadIdx.x == 0) atomicCAS(a.status, 0, 4);
        return;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q0 = blockIdx.x * kRows, h = blockIdx.y, n = blockIdx.z;
    const int L = a.L;
    const int tiles = (L + kRows - 1) / kRows;
    const int row_base = n * L;

    if (threadIdx.x == 0) {
        mbar_init(&ctl->q_full, 1);
        for (int s = 0; s < kKStages; ++s) {
            mbar_init(&ctl->k_full[s], 1);
            mbar_init(&ctl->k_empty[s], 1);
        }
        for (int s = 0; s < kVStages; ++s) {
            mbar_init(&ctl->v_full[s], 1);
            mbar_init(&ctl->v_empty[s], 1);
        }
        mbar_init(&ctl->s_full, 1);
        mbar_init(&ctl->pv_full, 1);
        mbar_init(&ctl->p_full, 4);
        ctl->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 4) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&ctl->tmem_base)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;

    if (warp == 4 && lane == 0) {
        {
            const int cq = h * kHd, ck = a.C + h * kHd, cv = 2 * a.C + h * kHd;
            mbar_expect_tx(&ctl->q_full, kTile);
            tma_load_2d(&tm, &ctl->q_full, sQ, cq, row_base + q0);
            for (int j = 0; j < tiles; ++j) {
                const int s = j % kKStages;
                if (!mbar_wait(&ctl->k_empty[s], ((j / kKStages) & 1) ^ 1, &ctl->abort)) goto fail_producer;
                mbar_expect_tx(&ctl->k_full[s], kTile);
                tma_load_2d(&tm, &ctl->k_full[s], sK + s * kTile, ck, row_base + j * kRows);
                const int sv = j % kVStages;
                if (!mbar_wait(&ctl->v_empty[sv], ((j / kVStages) & 1) ^ 1, &ctl->abort)) goto fail_producer;
                mbar_expect_tx(&ctl->v_full[sv], kTile);
                tma_load_2d(&tm, &ctl->v_full[sv], sV + sv * kTile, cv, row_base + j * kRows);
            }
            goto done_producer;
        fail_producer:
            ctl->abort = 1;
            atomicCAS(a.status, 0, 1);
        done_producer:;
        }
    } else if (warp == 4 && lane == 1) {
        {
            constexpr uint32_t idesc_s = instr_desc(false, false, kRows);
            constexpr uint32_t idesc_o = instr_desc(false, true, kHd);
            const uint32_t q = smem_u32(sQ), p = smem_u32(sP);
            const uint32_t tS = tmem + kSCol, tO = tmem + kOCol;
            bool ok = mbar_wait(&ctl->q_full, 0, &ctl->abort) && mbar_wait(&ctl->k_full[0], 0, &ctl->abort);
            if (ok) {
                tc_fence_after();
                const uint32_t k = smem_u32(sK);
#pragma unroll
                for (int kk = 0; kk < kHd / 16; ++kk)
                    tc_mma(tS, operand_desc<false>(q, kk), operand_desc<false>(k, kk), idesc_s, kk > 0);
                tc_commit(&ctl->k_empty[0]);
                tc_commit(&ctl->s_full);
            }
            for (int j = 0; ok && j < tiles; ++j) {
                // P_j written and O rescaled (so S is free again), V_j landed
                ok = mbar_wait(&ctl->p_full, j & 1, &ctl->abort) &&
                     mbar_wait(&ctl->v_full[j % kVStages], (j / kVStages) & 1, &ctl->abort);
                if (!ok) break;
                tc_fence_after();
                const uint32_t v = smem_u32(sV + (j % kVStages) * kTile);
#pragma unroll
                for (int kk = 0; kk < kRows / 16; ++kk)
                    tc_mma(tO, operand_desc<false>(p + (kk >> 2) * kTile, kk & 3), operand_desc<true>(v, kk), idesc_o,
                           (j > 0 || kk > 0) ? 1u : 0u);
                tc_commit(&ctl->v_empty[j % kVStages]);
                tc_commit(&ctl->pv_full);
                if (j + 1 < tiles) {
                    const int s = (j + 1) % kKStages;
                    ok = mbar_wait(&ctl->k_full[s], ((j + 1) / kKStages) & 1, &ctl->abort);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t k = smem_u32(sK + s * kTile);
#pragma unroll
                    for (int kk = 0; kk < kHd / 16; ++kk)
                        tc_mma(tS, operand_desc<false>(q, kk), operand_desc<false>(k, kk), idesc_s, kk > 0);
                    tc_commit(&ctl->k_empty[s]);
                    tc_commit(&ctl->s_full);
                }
            }
            if (!ok) {
                ctl->abort = 1;
                atomicCAS(a.status, 0, 2);
            }
        }
    } else if (warp < 4) {
        // softmax warps: thread = query row r = TMEM lane r
        const int r = threadIdx.x;
        const uint32_t lane_off = static_cast<uint32_t>(32 * warp) << 16;
        const uint32_t tS = tmem + kSCol + lane_off, tO = tmem + kOCol + lane_off;
        float m = -1e30f, l = 0.f;   // reference maximum (log2 units) and row sum
        bool ok = true;
        unsigned char* prow = sP + r * 128;
        const int sw = r & 7;
        for (int j = 0; j < tiles; ++j) {
            // S_j landed; its commit also covers O_{j-1} = P_{j-1}.V_{j-1}, so P and O are free
            if (!mbar_wait(&ctl->s_full, j & 1, &ctl->abort)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int valid = min(kRows, L - j * kRows);   // keys of this tile inside the sequence
            float sv[kRows];
            tmem_ld128(tS, sv);
            float mx = -1e30f;
#pragma unroll
            for (int i = 0; i < kRows; ++i)
                if (i < valid) mx = fmaxf(mx, sv[i]);
            const float m_new = mx * a.scale_log2;
            // lazy rescale: keep the old reference maximum unless the row maximum grew by more than
            // 2^8 (p stays <= 256, exact enough in fp32 / bf16); the tensor-memory O is rescaled
            // only by warps with a row that moved
            float alpha = 1.f;
            if (m_new > m + 8.f) {
                alpha = ex2(m - m_new);
                m = m_new;
            }
            if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
                for (int c = 0; c < kHd / 16; ++c) {
                    float ov[16];
                    tmem_ld16(tO + 16 * c, ov);
#pragma unroll
                    for (int i = 0; i < 16; ++i) ov[i] *= alpha;
                    tmem_st16(tO + 16 * c, ov);
                }
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            }
            float sum = 0.f;
#pragma unroll
            for (int c = 0; c < kRows / 16; ++c) {
                uint32_t w[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int k0 = 16 * c + 2 * i;
                    const float p0 = k0 < valid ? ex2(sv[k0] * a.scale_log2 - m) : 0.f;
                    const float p1 = k0 + 1 < valid ? ex2(sv[k0 + 1] * a.scale_log2 - m) : 0.f;
                    sum += p0 + p1;
                    w[i] = pack_bf16x2(p0, p1);
                }
                // keys 16c..16c+15 -> tile c/4, 16-byte chunks 2*(c%4), +1 of this row (128B swizzle)
                unsigned char* base = prow + (c >> 2) * kTile;
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const int ch = 2 * (c & 3) + q;
                    *reinterpret_cast<uint4*>(base + ((ch ^ sw) << 4)) =
                        make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
                }
            }
            l = l * alpha + sum;
            // P visible to the tensor core; S and O may be overwritten / accumulated into
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ctl->p_full);
        }
        if (ok && !mbar_wait(&ctl->pv_full, (tiles - 1) & 1, &ctl->abort)) ok = false;
        if (!ok) {
            ctl->abort = 1;
            if (lane == 0) atomicCAS(a.status, 0, 3);
        } else {
            tc_fence_after();
            float o[kHd];
#pragma unroll
            for (int c = 0; c < kHd / 32; ++c) tmem_ld32(tO + 32 * c, o + 32 * c);
            if (q0 + r < L) {
                const float inv = 1.f / l;
                uint4* dst = reinterpret_cast<uint4*>(a.o + static_cast<int64_t>(row_base + q0 + r) * a.ldo + h * kHd);
#pragma unroll
                for (int q = 0; q < kHd / 8; ++q)
                    dst[q] = make_uint4(pack_bf16x2(o[8 * q] * inv, o[8 * q + 1] * inv),
                                        pack_bf16x2(o[8 * q + 2] * inv, o[8 * q + 3] * inv),
                                        pack_bf16x2(o[8 * q + 4] * inv, o[8 * q + 5] * inv),
                                        pack_bf16x2(o[8 * q + 6] * inv, o[8 * q + 7] * inv));
                if (a.lse)
                    a.lse[(static_cast<int64_t>(n) * a.H + h) * L + q0 + r] = (m + __log2f(l)) * 0.69314718055994531f;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 4) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

PFN_cuTensorMapEncodeTiled_v12000 attn_encode_fn() {
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

}  // namespace

size_t attn_fwd_tc_smem_bytes() { return kSmemBytes; }

namespace {
int g_attn_variant = 2;   // kMinBlocks of the launched instantiation

template <typename F>
auto attn_kernel_ptr(F&& f) {
    return g_attn_variant == 1 ? f(attn_fwd_tc_kernel<1>) : f(attn_fwd_tc_kernel<2>);
}
}  // namespace

void attn_fwd_tc_set_variant(int min_blocks) { g_attn_variant = min_blocks == 1 ? 1 : 2; }

int attn_fwd_tc_blocks_per_sm() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    return attn_kernel_ptr([](auto kern) {
        int n = 0;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytes)) !=
                cudaSuccess ||
            cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
            return 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kThreads, kSmemBytes) != cudaSuccess) return 0;
        return n;
    });
}

cudaError_t launch_attn_fwd_tc(const void* qkv, int64_t ld, int nseq, int L, int H, void* o, int64_t ldo, float* lse,
                               float scale, int* status, cudaStream_t st) {
    if (nseq == 0 || L == 0) return cudaSuccess;
    const int C = H * kHd;
    // TMA: 16-byte aligned base and row pitch; the q / k / v column offsets are multiples of 64 elements
    if (reinterpret_cast<uintptr_t>(qkv) % 16 != 0 || ld % 8 != 0 || ld < 3 * C) return cudaErrorInvalidValue;
    if (reinterpret_cast<uintptr_t>(o) % 16 != 0 || ldo % 8 != 0) return cudaErrorInvalidValue;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaSetDevice(dev);   // the driver-API encode needs a current context
    if (e != cudaSuccess) return e;
    auto fn = attn_encode_fn();
    if (!fn) return cudaErrorNotSupported;
    CUtensorMap tm;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(3 * C), static_cast<cuuint64_t>(static_cast<int64_t>(nseq) * L)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
    cuuint32_t box[2] = {kHd, kRows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(qkv), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        std::fprintf(stderr, "attn_fwd_tc: cuTensorMapEncodeTiled failed (%d)\n", static_cast<int>(r));
        return cudaErrorInvalidValue;
    }
    static bool attr_set[2][64] = {};
    AttnArgs a{static_cast<__nv_bfloat16*>(o), lse, status, L, H, C, ldo, scale * 1.4426950408889634f};
    dim3 grid((L + kRows - 1) / kRows, H, nseq);
    return attn_kernel_ptr([&](auto kern) {
        bool& set = attr_set[g_attn_variant - 1][dev & 63];
        if (!set) {
            cudaError_t ea = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  static_cast<int>(kSmemBytes));
            // all of the unified L1 / shared storage as shared memory (a property of this kernel)
            if (ea == cudaSuccess) ea = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
            if (ea != cudaSuccess) return ea;
            set = true;
        }
        kern<<<grid, kThreads, kSmemBytes, st>>>(tm, a);
        return cudaGetLastError();
    });
}

}  // namespace mmltk
