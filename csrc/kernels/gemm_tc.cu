// bf16 GEMM on the 5th-generation tensor cores (tcgen05) with the accumulator
// in tensor memory.
//
//   C[M,N] = opA(A) . opB(B)  (+ bias, + activation / LayerScale-residual epilogue)
//
// Persistent kernel, one CTA per SM, 128x256 output tiles, six warps:
//   warp 0    TMA producer: 128B-swizzled A (128x64) and B (256x64) tiles into a
//             4-stage ring (cp.async.bulk.tensor with mbarrier transaction
//             counts); also owns the TMEM allocation (all 512 columns);
//   warp 1    MMA issuer: one thread issues tcgen05.mma (M=128, N=256, K=16,
//             bf16 x bf16 -> fp32), 4 per K tile, into one of two TMEM
//             accumulators, and hands each smem stage back with tcgen05.commit;
//   warps 2-5 epilogue: tcgen05.ld (32 lanes x 16 columns per instruction),
//             fused bias / GELU / ReLU / LayerScale + residual, bf16 stores.
// The two accumulators let the epilogue of tile i run while tile i+1 is being
// multiplied.  Work units are (tile, K split); GEMMs with few output tiles and
// a long reduction (weight gradients reduce over all tokens) are split along K
// and the partial tiles are summed with 16-byte fp32 vector atomics into a
// workspace, then converted.  Operands may be K-major ([rows, K] row-major)
// or MN-major ([K, rows] row-major), so x.W^T, dY.W and dY^T.X all run without
// materialising a transpose.  M/N/K tails: TMA zero fill + masked stores.
//
// Pair variant (gemm_tc2_kernel): a cluster of two CTAs on two SMs computes one
// 256-row tile with tcgen05.mma.cta_group::2 (M = 256).  Each CTA loads its own
// 128 rows of A and its own half of the tile's B columns; the MMA issued by the
// even CTA reads both CTAs' shared memory, and each CTA's tensor memory receives
// its 128 accumulator rows.  Per SM that halves the B operand traffic through
// shared memory, which is what limits the single-CTA tiles.  Every CTA loads
// only its own tiles; the odd CTA's loads complete on the even CTA's mbarriers
// (the .cta_group::2 form of the tensor load), the MMA completion is committed
// to the stage / accumulator barriers of both CTAs, and both epilogues arrive
// on the even CTA's accumulator-free barrier.
//
// Every mbarrier wait is bounded; on timeout the kernel records an error code
// in a status word and leaves (after releasing its TMEM) instead of spinning.
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstdlib>

#include "common.cuh"
#include "gemm_tc.h"
#include "tcgen05.cuh"

namespace mmltk {

namespace {

using namespace tc;

constexpr int BM = 128, BK = 64;
constexpr int kATile = BM * BK * 2;                // 16 KB
constexpr int kThreads = 320;                      // 2 producer/MMA warps + 8 epilogue warps
constexpr int kEpiWarps = 8;
// two 32 x 32 bf16 tiles per epilogue warp, 64-byte rows in the TMA store's 64-byte swizzle (the tensor store clips rows / columns past the output, so tails need no masks)
constexpr int kTmaTileBytes = 32 * 64;
constexpr int kTmaStagingBytes = kEpiWarps * 2 * kTmaTileBytes;
constexpr int kMaxStages = 6;
constexpr int kSmemLimit = 227 * 1024;

// Tile configuration for a tile width BN (128, 192 or 256 output columns).
template <int BN_>
struct Tile {
    static constexpr int BN = BN_;
    static constexpr int kBTile = BN * BK * 2;
    static constexpr int kStageBytes = kATile + kBTile;
    static constexpr int kStages = (kSmemLimit - kTmaStagingBytes - 2048) / kStageBytes < kMaxStages
                                       ? (kSmemLimit - kTmaStagingBytes - 2048) / kStageBytes
                                       : kMaxStages;
    static constexpr int kAccCols = BN;            // fp32 accumulator columns per buffer
    static constexpr int kTmemCols = 2 * BN <= 256 ? 256 : 512;
    static constexpr size_t kSmemBytes = static_cast<size_t>(kStages) * kStageBytes + kTmaStagingBytes + 1024 + 256;
};

struct __align__(8) SmemCtl {
    uint64_t full[kMaxStages];
    uint64_t empty[kMaxStages];
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint32_t tmem_base;
    int abort;
};

__device__ __forceinline__ float gelu_f(float x) { return gelu_fwd(x); }
__device__ __forceinline__ float gelu_grad_f(float x) { return gelu_bwd(x); }

// This lane's row of a 32-row x `ncols` bf16 block (lane = row), straight from global memory: 16-byte
// loads of the row's contiguous 64 bytes (the rows' sectors are read whole across the 4 loads).
__device__ __forceinline__ void row_load(int lane, float* x, const __nv_bfloat16* base, int64_t ld, int rows_valid,
                                        int ncols) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint4 w = make_uint4(0, 0, 0, 0);
        if (lane < rows_valid && 8 * j < ncols) w = *reinterpret_cast<const uint4*>(base + lane * ld + 8 * j);
        const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 t = unpack_bf16x2(u[i]);
            x[8 * j + 2 * i] = t.x;
            x[8 * j + 2 * i + 1] = t.y;
        }
    }
}

// Where one epilogue warp's chunks go: tensor stores through 3-D maps (column, row, batch) from two
// rotating swizzled tiles of this warp.
struct EpiOut {
    unsigned char* tbuf;                 // two kTmaTileBytes tiles
    const CUtensorMap* mapC;
    const CUtensorMap* mapAux;
    int bt;
    int turn;
};

// Tensor store of this warp's 32 x 32 block (lane = row, x = 32 values) at (col, row0, batch bt).
__device__ __forceinline__ void tma_store_tile(EpiOut& eo, const CUtensorMap* map, int lane, const float* x, int col,
                                               int row0) {
    unsigned char* buf = eo.tbuf + eo.turn * kTmaTileBytes;
    // the store issued from this tile two chunks ago has finished reading it
    if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
    __syncwarp();
    unsigned char* rowp = buf + lane * 64;
    const int sw = (lane >> 1) & 3;     // 64-byte swizzle: 16-byte chunk c of row r at c ^ ((r >> 1) & 3)
#pragma unroll
    for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(rowp + ((c ^ sw) << 4)) =
            make_uint4(pack_bf16x2(x[8 * c], x[8 * c + 1]), pack_bf16x2(x[8 * c + 2], x[8 * c + 3]),
                       pack_bf16x2(x[8 * c + 4], x[8 * c + 5]), pack_bf16x2(x[8 * c + 6], x[8 * c + 7]));
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) {
        asm volatile(
            "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(map),
            "r"(smem_u32(buf)), "r"(col), "r"(row0), "r"(eo.bt)
            : "memory");
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
    eo.turn ^= 1;
}

// Epilogue of one warp's 32 rows x `ncols` (16 or 32) columns; lane = row.
__device__ __forceinline__ void epilogue_chunk(const GemmArgs& g, EpiOut& eo, int lane, int row0, int col,
                                               int ncols, float* v, bool rmax_first = true) {
    const int rows_valid = min(32, g.M - row0);
    const int row = row0 + lane;
    if (g.ws) {  // split-K partial: fp32 vector atomics into the workspace
        if (row < g.M) {
            float4* w = reinterpret_cast<float4*>(g.ws + static_cast<int64_t>(row) * g.ldc + col);
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (4 * i < ncols)
                    atomicAdd(w + i, make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]));
        }
        return;
    }
    if (g.bias) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (8 * j < ncols) {
                float b[8];
                load8(g.bias + col + 8 * j, b);
#pragma unroll
                for (int i = 0; i < 8; ++i) v[8 * j + i] += b[i];
            }
        }
    }
    const int64_t base = static_cast<int64_t>(row0) * g.ldc + col;
    if (g.epi == 7) {
        // running row maximum over this warp's columns (the caller passes rmax already offset to
        // this warp's half and batch; the first chunk of a half stores, later ones combine)
        float m = -__int_as_float(0x7f800000);
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (i < ncols) m = fmaxf(m, v[i]);
        if (row < g.M) {
            float* dst = g.rmax + row;
            *dst = (rmax_first ? m : fmaxf(*dst, m));
        }
        return;
    }
    if (g.aux) tma_store_tile(eo, eo.mapAux, lane, v, col, row0);   // pre-activation for backward
    if (g.epi == 1) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = gelu_f(v[i]);
    } else if (g.epi == 2) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = fmaxf(v[i], 0.f);
    } else if (g.epi == 3) {
        float r[32];
        row_load(lane, r, g.res + base, g.ldc, rows_valid, ncols);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (8 * j < ncols) {
                float gm[8];
                load8(g.gamma + col + 8 * j, gm);
#pragma unroll
                for (int i = 0; i < 8; ++i) v[8 * j + i] = r[8 * j + i] + gm[i] * v[8 * j + i];
            }
        }
    } else if (g.epi == 6) {
        float r[32];
        row_load(lane, r, g.res + base, g.ldc, rows_valid, ncols);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = g.alpha * v[i] + g.beta * r[i];
    } else if (g.epi == 4 || g.epi == 5 || g.epi == 8) {
        // activation backward: the product is the gradient w.r.t. the activation output
        float p[32];
        row_load(lane, p, g.res + base, g.ldc, rows_valid, ncols);
        if (g.epi == 4) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] *= gelu_grad_f(p[i]);
        } else if (g.epi == 8) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] *= p[i];     // res holds the stored derivative
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = p[i] > 0.f ? v[i] : 0.f;
        }
    }
    tma_store_tile(eo, eo.mapC, lane, v, col, row0);
    if (g.colacc) {
        // column sums of the stored (bf16-rounded) tile, read back from the staging: lane = column
        if (lane < ncols) {
            float s = 0.f;
            const unsigned char* buf = eo.tbuf + (eo.turn ^ 1) * kTmaTileBytes;   // the tile just stored
            for (int r = 0; r < rows_valid; ++r) {
                const unsigned char* p = buf + r * 64 + ((((lane >> 3) ^ ((r >> 1) & 3))) << 4) + (lane & 7) * 2;
                s += __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(p));
            }
            atomicAdd(g.colacc + col + lane, s);
        }
        __syncwarp();
    }
}

struct Sched {
    int m_tiles, n_tiles, splits, ktiles, kt_per_split, bn, rows;
    __device__ int batch_of(int u) const { return u / (m_tiles * n_tiles * splits); }
    __device__ void unit(int u, int& m0, int& n0, int& kt0, int& kt1) const {
        u %= m_tiles * n_tiles * splits;
        const int tile = u / splits, s = u % splits;
        m0 = (tile / n_tiles) * rows;
        n0 = (tile % n_tiles) * bn;
        kt0 = s * kt_per_split;
        kt1 = min(ktiles, kt0 + kt_per_split);
    }
};

template <bool A_MN, bool B_MN, int BN_>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                                                              const __grid_constant__ CUtensorMap tmB,
                                                              const __grid_constant__ CUtensorMap tmC,
                                                              const __grid_constant__ CUtensorMap tmAux, GemmArgs g,
                                                              Sched sch) {
    using T = Tile<BN_>;
    constexpr int BN = T::BN, kStages = T::kStages, kBTile = T::kBTile, kAccCols = T::kAccCols;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* tilesA = smem;
    unsigned char* tilesB = smem + kStages * kATile;
    unsigned char* tstage = smem + kStages * (kATile + kBTile);     // 1024-aligned TMA store tiles
    SmemCtl* ctl = reinterpret_cast<SmemCtl*>(tstage + kTmaStagingBytes);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int units = sch.m_tiles * sch.n_tiles * sch.splits * g.batch;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&ctl->full[s], 1);
            mbar_init(&ctl->empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&ctl->acc_full[b], 1);
            mbar_init(&ctl->acc_empty[b], kEpiWarps);  // one arrival per epilogue warp
        }
        ctl->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&ctl->tmem_base)),
                     "r"(T::kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            int it = 0;  // global k-tile counter across units -> ring position
            for (int u = blockIdx.x; u < units; u += gridDim.x) {
                int m0, n0, kt0, kt1;
                sch.unit(u, m0, n0, kt0, kt1);
                // MN-major operands are loaded as 64-wide boxes; boxes entirely past the
                // extent are skipped (they only feed output rows/columns that are masked)
                const int a_boxes = A_MN ? min(BM / 64, (g.M - m0 + 63) / 64) : 1;
                const int b_boxes = B_MN ? min(BN / 64, (g.N - n0 + 63) / 64) : 1;
                const uint32_t a_bytes = g.conv_w ? static_cast<uint32_t>(g.conv_w * g.conv_rows * 128)
                                                  : (A_MN ? a_boxes * 8192 : kATile);
                const uint32_t bytes = a_bytes + (B_MN ? b_boxes * 8192 : kBTile);
                // batch bt: the operands' tile coordinates shifted by bt * (shift along K, along M / N)
                const int bt = sch.batch_of(u);
                const int ak = bt * g.a_bk, am = bt * g.a_bm, bk = bt * g.b_bk, bn_ = bt * g.b_bn;
                // convolution tile bt: image and first output row
                const int cimg = g.conv_w ? bt / g.conv_groups : 0;
                const int cy0 = g.conv_w ? (bt % g.conv_groups) * g.conv_rows : 0;
                const int cchunks = g.conv_w ? g.conv_c / BK : 1;
                for (int kt = kt0; kt < kt1; ++kt, ++it) {
                    const int s = it % kStages;
                    const uint32_t ph = (it / kStages) & 1;
                    if (!mbar_wait(&ctl->empty[s], ph ^ 1, &ctl->abort)) {
                        ctl->abort = 1;
                        atomicCAS(g.status, 0, 1);
                        goto producer_done;
                    }
                    mbar_expect_tx(&ctl->full[s], bytes);
                    unsigned char* a = tilesA + s * kATile;
                    unsigned char* b = tilesB + s * kBTile;
                    const int k0 = kt * BK;
                    if (A_MN) {
                        for (int q = 0; q < a_boxes; ++q)
                            tma_load_2d(&tmA, &ctl->full[s], a + q * 8192, am + m0 + 64 * q, ak + k0);
                    } else if (g.conv_w) {
                        // tap (dy, dx) and channel chunk of this K tile; out-of-image pixels read as zero
                        const int tap = kt / cchunks, c0 = (kt % cchunks) * BK;
                        tma_load_4d(&tmA, &ctl->full[s], a, c0, tap % 3 - 1, cy0 + tap / 3 - 1, cimg);
                    } else {
                        tma_load_2d(&tmA, &ctl->full[s], a, ak + k0, am + m0);
                    }
                    if (B_MN) {
                        for (int q = 0; q < b_boxes; ++q)
                            tma_load_2d(&tmB, &ctl->full[s], b + q * 8192, bn_ + n0 + 64 * q, bk + k0);
                    } else {
                        tma_load_2d(&tmB, &ctl->full[s], b, bk + k0, bn_ + n0);
                    }
                }
            }
        producer_done:;
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = instr_desc(A_MN, B_MN, BN);
            int it = 0, local = 0;
            for (int u = blockIdx.x; u < units; u += gridDim.x, ++local) {
                int m0, n0, kt0, kt1;
                sch.unit(u, m0, n0, kt0, kt1);
                const int buf = local & 1;
                const uint32_t acc_ph = (local >> 1) & 1;
                if (!mbar_wait(&ctl->acc_empty[buf], acc_ph ^ 1, &ctl->abort)) {
                    ctl->abort = 1;
                    atomicCAS(g.status, 0, 2);
                    break;
                }
                tc_fence_after();
                const uint32_t acc = tmem + buf * kAccCols;
                bool ok = true;
                for (int kt = kt0; kt < kt1; ++kt, ++it) {
                    const int s = it % kStages;
                    const uint32_t ph = (it / kStages) & 1;
                    if (!mbar_wait(&ctl->full[s], ph, &ctl->abort)) {
                        ctl->abort = 1;
                        atomicCAS(g.status, 0, 2);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a = smem_u32(tilesA + s * kATile);
                    const uint32_t b = smem_u32(tilesB + s * kBTile);
                    if (!(g.diag & 2)) {
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk)
                            tc_mma(acc, operand_desc<A_MN>(a, kk), operand_desc<B_MN>(b, kk), idesc,
                                   (kt > kt0 || kk > 0) ? 1u : 0u);
                    }
                    tc_commit(&ctl->empty[s]);
                }
                if (!ok) break;
                tc_commit(&ctl->acc_full[buf]);
            }
        }
    } else {
        // epilogue: 8 warps; warp w reads TMEM lanes 32*(w%4) .. +31 (its quarter of the
        // tile's rows) and half of the tile's columns, 32 columns per tcgen05.wait
        const int q = warp & 3;
        const int half = (warp - 2) >> 2;
        EpiOut eo{tstage + (warp - 2) * 2 * kTmaTileBytes, &tmC, &tmAux, 0, 0};
        int local = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x, ++local) {
            int m0, n0, kt0, kt1;
            sch.unit(u, m0, n0, kt0, kt1);
            const int buf = local & 1;
            const uint32_t acc_ph = (local >> 1) & 1;
            if (!mbar_wait(&ctl->acc_full[buf], acc_ph, &ctl->abort)) {
                if (lane == 0) atomicCAS(g.status, 0, 3);
                ctl->abort = 1;
                break;
            }
            tc_fence_after();
            const int row0 = m0 + 32 * q;
            const uint32_t acc = tmem + buf * kAccCols + (static_cast<uint32_t>(32 * q) << 16);
            constexpr int kHalfCols = BN / 2;
            // this unit's batch: outputs (and the epilogue's side inputs) at their batch offsets; the
            // tensor stores address the batch by their third coordinate
            GemmArgs gb = g;
            const int bt = sch.batch_of(u);
            eo.bt = bt;
            if (bt) {
                gb.C += bt * g.bs_c;
                if (gb.aux) gb.aux += bt * g.bs_c;
                if (gb.res) gb.res += bt * g.bs_c;
                if (gb.bias) gb.bias += bt * g.bs_bias;
            }
            if (g.epi == 7) gb.rmax += (static_cast<int64_t>(half) * g.batch + bt) * g.M;
            for (int c = half * kHalfCols; c < (half + 1) * kHalfCols; c += 32) {
                if (n0 + c >= g.N || row0 >= g.M) break;  // warp-uniform
                const int ncols = min(min(32, (half + 1) * kHalfCols - c), g.N - n0 - c);
                float v[32];
                if (ncols > 16) {
                    tmem_ld32(acc + c, v);
                } else {
                    tmem_ld16(acc + c, v);
                }
                if (g.diag & 1) continue;
                epilogue_chunk(gb, eo, lane, row0, n0 + c, ncols, v, c == half * kHalfCols);
            }
            // accumulator buffer free again
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ctl->acc_empty[buf]);
        }
        // every tensor store of this warp has completed before the CTA (and its shared memory) ends
        if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(T::kTmemCols));
    }
}

// ------------------------------------------------------------------ CTA-pair variant

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank` of this cluster
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// bounded wait on a barrier that receives arrivals from the other CTA of the pair
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, const volatile int* abort) {
    for (long long i = 0; i < kWaitLimit; ++i) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if ((i & 255) == 255 && *abort) return false;
    }
    return false;
}
// 2-D TMA tile load into this CTA's shared memory whose completion is counted on an mbarrier
// of either CTA of the pair (given as a shared::cluster address)
__device__ __forceinline__ void tma_load_2d_pair(const CUtensorMap* map, uint32_t bar_cluster, void* dst, int c0,
                                                 int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
        "[%2];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(bar_cluster), "r"(c0), "r"(c1)
        : "memory");
}
__device__ __forceinline__ void tc_mma_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
// arrive on an mbarrier (shared::cluster address, either CTA) once the pair's earlier MMAs are done
__device__ __forceinline__ void tc_commit_pair(uint32_t bar_cluster) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
                 : "memory");
}

constexpr int kPairRows = 256;                     // output rows of one pair tile (128 per CTA)

template <int BN_>
struct PairTile {
    static constexpr int BN = BN_;                 // output columns of a pair tile (the MMA's N)
    static constexpr int kBHalf = BN / 2;          // B rows (N) held by each CTA
    static constexpr int kBTile = kBHalf * BK * 2;
    static constexpr int kStageBytes = kATile + kBTile;
    static constexpr int kStages = (kSmemLimit - kTmaStagingBytes - 2048) / kStageBytes < kMaxStages
                                       ? (kSmemLimit - kTmaStagingBytes - 2048) / kStageBytes
                                       : kMaxStages;
    static constexpr int kAccCols = BN;
    static constexpr int kTmemCols = 2 * BN <= 256 ? 256 : 512;
    static constexpr size_t kSmemBytes = static_cast<size_t>(kStages) * kStageBytes + kTmaStagingBytes + 1024 + 256;
};

// bytes one CTA's loads deliver for a stage (MN-major boxes past the extent are not loaded)
template <bool A_MN, bool B_MN, int BN>
__device__ __forceinline__ uint32_t pair_stage_bytes(const GemmArgs& g, int m_cta, int n_cta) {
    using T = PairTile<BN>;
    const int a_boxes = A_MN ? max(0, min(BM / 64, (g.M - m_cta + 63) / 64)) : 0;
    const int b_boxes = B_MN ? max(0, min(T::kBHalf / 64, (g.N - n_cta + 63) / 64)) : 0;
    return (A_MN ? a_boxes * 8192 : kATile) + (B_MN ? b_boxes * 8192 : T::kBTile);
}

template <bool A_MN, bool B_MN, int BN_>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmAux, GemmArgs g,
                    Sched sch) {
    using T = PairTile<BN_>;
    constexpr int BN = T::BN, kStages = T::kStages, kBTile = T::kBTile, kAccCols = T::kAccCols, kBHalf = T::kBHalf;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* tilesA = smem;
    unsigned char* tilesB = smem + kStages * kATile;
    unsigned char* tstage = smem + kStages * (kATile + kBTile);     // 1024-aligned TMA store tiles
    SmemCtl* ctl = reinterpret_cast<SmemCtl*>(tstage + kTmaStagingBytes);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int units = sch.m_tiles * sch.n_tiles * sch.splits;   // unbatched products only

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&ctl->full[s], 1);
            mbar_init(&ctl->empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&ctl->acc_full[b], 1);
            mbar_init(&ctl->acc_empty[b], 2 * kEpiWarps);   // every epilogue warp of both CTAs
        }
        ctl->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 0) {
        // one warp of each CTA allocates together: both get the same columns
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&ctl->tmem_base)),
                     "r"(T::kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();   // the peer's barriers are initialised before anything targets them
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            int it = 0;
            for (int u = pair; u < units; u += npairs) {
                int m0, n0, kt0, kt1;
                sch.unit(u, m0, n0, kt0, kt1);
                const int m_cta = m0 + static_cast<int>(rank) * BM;
                const int n_cta = n0 + static_cast<int>(rank) * kBHalf;
                const int a_boxes = A_MN ? max(0, min(BM / 64, (g.M - m_cta + 63) / 64)) : 1;
                const int b_boxes = B_MN ? max(0, min(kBHalf / 64, (g.N - n_cta + 63) / 64)) : 1;
                const uint32_t pair_bytes = pair_stage_bytes<A_MN, B_MN, BN>(g, m0, n0) +
                                            pair_stage_bytes<A_MN, B_MN, BN>(g, m0 + BM, n0 + kBHalf);
                for (int kt = kt0; kt < kt1; ++kt, ++it) {
                    const int s = it % kStages;
                    const uint32_t ph = (it / kStages) & 1;
                    if (!mbar_wait(&ctl->empty[s], ph ^ 1, &ctl->abort)) {
                        ctl->abort = 1;
                        atomicCAS(g.status, 0, 1);
                        goto producer_done;
                    }
                    // both CTAs' loads complete on the even CTA's barrier, which expects them all
                    if (rank == 0) mbar_expect_tx(&ctl->full[s], pair_bytes);
                    const uint32_t fullb = mapa_shared(smem_u32(&ctl->full[s]), 0);
                    unsigned char* a = tilesA + s * kATile;
                    unsigned char* b = tilesB + s * kBTile;
                    const int k0 = kt * BK;
                    if (A_MN) {
                        for (int q = 0; q < a_boxes; ++q) tma_load_2d_pair(&tmA, fullb, a + q * 8192, m_cta + 64 * q, k0);
                    } else {
                        tma_load_2d_pair(&tmA, fullb, a, k0, m_cta);
                    }
                    if (B_MN) {
                        for (int q = 0; q < b_boxes; ++q) tma_load_2d_pair(&tmB, fullb, b + q * 8192, n_cta + 64 * q, k0);
                    } else {
                        tma_load_2d_pair(&tmB, fullb, b, k0, n_cta);
                    }
                }
            }
        producer_done:;
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            const uint32_t idesc = instr_desc(A_MN, B_MN, BN, kPairRows);
            int it = 0, local = 0;
            for (int u = pair; u < units; u += npairs, ++local) {
                int m0, n0, kt0, kt1;
                sch.unit(u, m0, n0, kt0, kt1);
                const int buf = local & 1;
                const uint32_t acc_ph = (local >> 1) & 1;
                if (!mbar_wait_cluster(&ctl->acc_empty[buf], acc_ph ^ 1, &ctl->abort)) {
                    ctl->abort = 1;
                    atomicCAS(g.status, 0, 2);
                    break;
                }
                tc_fence_after();
                const uint32_t acc = tmem + buf * kAccCols;
                bool ok = true;
                for (int kt = kt0; kt < kt1; ++kt, ++it) {
                    const int s = it % kStages;
                    const uint32_t ph = (it / kStages) & 1;
                    if (!mbar_wait(&ctl->full[s], ph, &ctl->abort)) {
                        ctl->abort = 1;
                        atomicCAS(g.status, 0, 2);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a = smem_u32(tilesA + s * kATile);
                    const uint32_t b = smem_u32(tilesB + s * kBTile);
                    if (!(g.diag & 2)) {
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk)
                            tc_mma_pair(acc, operand_desc<A_MN>(a, kk), operand_desc<B_MN>(b, kk), idesc,
                                        (kt > kt0 || kk > 0) ? 1u : 0u);
                    }
                    // the stage is free in both CTAs once these MMAs are done
                    tc_commit_pair(mapa_shared(smem_u32(&ctl->empty[s]), 0));
                    tc_commit_pair(mapa_shared(smem_u32(&ctl->empty[s]), 1));
                }
                if (!ok) break;
                tc_commit_pair(mapa_shared(smem_u32(&ctl->acc_full[buf]), 0));
                tc_commit_pair(mapa_shared(smem_u32(&ctl->acc_full[buf]), 1));
            }
        }
    } else {
        // epilogue: this CTA's 128 rows of the pair tile (TMEM lanes), all BN columns; warp w reads
        // lane quadrant w % 4 and half (w - 2) / 4 of the columns
        const int q = warp & 3;
        const int half = (warp - 2) >> 2;
        EpiOut eo{tstage + (warp - 2) * 2 * kTmaTileBytes, &tmC, &tmAux, 0, 0};
        int local = 0;
        for (int u = pair; u < units; u += npairs, ++local) {
            int m0, n0, kt0, kt1;
            sch.unit(u, m0, n0, kt0, kt1);
            const int buf = local & 1;
            const uint32_t acc_ph = (local >> 1) & 1;
            if (!mbar_wait(&ctl->acc_full[buf], acc_ph, &ctl->abort)) {
                if (lane == 0) atomicCAS(g.status, 0, 3);
                ctl->abort = 1;
                break;
            }
            tc_fence_after();
            const int row0 = m0 + static_cast<int>(rank) * BM + 32 * q;
            const uint32_t acc = tmem + buf * kAccCols + (static_cast<uint32_t>(32 * q) << 16);
            constexpr int kHalfCols = BN / 2;
            for (int c = half * kHalfCols; c < (half + 1) * kHalfCols; c += 32) {
                if (n0 + c >= g.N || row0 >= g.M) break;  // warp-uniform
                const int ncols = min(min(32, (half + 1) * kHalfCols - c), g.N - n0 - c);
                float v[32];
                if (ncols > 16) {
                    tmem_ld32(acc + c, v);
                } else {
                    tmem_ld16(acc + c, v);
                }
                if (g.diag & 1) continue;
                epilogue_chunk(g, eo, lane, row0, n0 + c, ncols, v);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(mapa_shared(smem_u32(&ctl->acc_empty[buf]), 0));
        }
        if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();   // no CTA leaves while the pair's MMAs may still read its shared memory
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(T::kTmemCols));
    }
}

__global__ void ws_to_bf16_kernel(const float* __restrict__ ws, __nv_bfloat16* __restrict__ c, int64_t n, int acc) {
    for (int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x * 8) {
        float v[8];
        load8(ws + i, v);
        if (acc) {
            float o[8];
            load8(c + i, o);
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] += o[j];
        }
        store8(c + i, v);
    }
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

// 2-D bf16 tensor [outer, inner] (row pitch in elements), box {64, box_rows}, 128B swizzle, zero OOB fill.
bool make_map(CUtensorMap* map, const void* ptr, int64_t inner, int64_t outer, int64_t pitch, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(pitch * 2)};
    cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        std::fprintf(stderr, "gemm_tc: cuTensorMapEncodeTiled failed (%d): inner %lld outer %lld pitch %lld box %d\n",
                     static_cast<int>(r), static_cast<long long>(inner), static_cast<long long>(outer),
                     static_cast<long long>(pitch), box_rows);
    return r == CUDA_SUCCESS;
}

// Input map of the implicit-GEMM convolution: channels-last bf16 [images, H, W, C], box {64 channels,
// W, rows, 1}, 128B swizzle (each pixel's 64 channels are one 128-byte row of the A tile), zero fill
// outside the image.
bool make_conv_map(CUtensorMap* map, const void* ptr, int64_t C, int64_t W, int64_t H, int64_t images, int rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[4] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(W), static_cast<cuuint64_t>(H),
                          static_cast<cuuint64_t>(images)};
    cuuint64_t strides[3] = {static_cast<cuuint64_t>(C * 2), static_cast<cuuint64_t>(C * W * 2),
                             static_cast<cuuint64_t>(C * W * H * 2)};
    cuuint32_t box[4] = {64, static_cast<cuuint32_t>(W), static_cast<cuuint32_t>(rows), 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        std::fprintf(stderr, "gemm_tc: convolution input map failed (%d): C %lld W %lld H %lld images %lld rows %d\n",
                     static_cast<int>(r), static_cast<long long>(C), static_cast<long long>(W),
                     static_cast<long long>(H), static_cast<long long>(images), rows);
    return r == CUDA_SUCCESS;
}

// Output map for the epilogue's tensor stores: bf16 [batch, rows, cols] (row pitch `pitch`, batch
// stride `bstride`, elements), 32 x 32 boxes, 64-byte swizzle; stores past the extents are clipped.
bool make_store_map(CUtensorMap* map, const void* ptr, int64_t cols, int64_t rows, int64_t batch, int64_t pitch,
                    int64_t bstride) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows),
                          static_cast<cuuint64_t>(std::max<int64_t>(1, batch))};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(pitch * 2), static_cast<cuuint64_t>(bstride * 2)};
    cuuint32_t box[3] = {32, 32, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        std::fprintf(stderr, "gemm_tc: output tensor map failed (%d): cols %lld rows %lld batch %lld pitch %lld\n",
                     static_cast<int>(r), static_cast<long long>(cols), static_cast<long long>(rows),
                     static_cast<long long>(batch), static_cast<long long>(pitch));
    return r == CUDA_SUCCESS;
}

}  // namespace

// Tile width for an M x N output: maximise (useful columns) x (wave occupancy of the
// persistent grid) x (per-tile efficiency of the width), e.g. N = 1536 -> 192,
// N = 384 with 82 row tiles -> 128 (246 tiles fill 2 waves of 148 SMs better than 164).
int pick_bn(int M, int N) {
    const int sms = num_sms();
    const int widths[3] = {256, 192, 128};
    const double tile_eff[3] = {1.0, 0.96, 0.88};
    int best = 256;
    double best_score = -1.0;
    for (int i = 0; i < 3; ++i) {
        const int bn = widths[i];
        const int tn = (N + bn - 1) / bn;
        const double col_eff = static_cast<double>(N) / (static_cast<double>(tn) * bn);
        const long long units = static_cast<long long>((M + BM - 1) / BM) * tn;
        const long long waves = (units + sms - 1) / sms;
        const double wave_eff = static_cast<double>(units) / static_cast<double>(waves * sms);
        const double score = col_eff * wave_eff * tile_eff[i];
        if (score > best_score + 1e-9) {
            best_score = score;
            best = bn;
        }
    }
    return best;
}

size_t gemm_tc_smem_bytes() { return Tile<256>::kSmemBytes; }

int conv3x3_tc_rows(int H, int W) {
    for (int r = std::min(H, BM / std::max(1, W)); r >= 1; --r)
        if (H % r == 0) return r;
    return 0;
}

namespace {

// 0: choose per shape, 1: single-CTA tiles only, 2: CTA-pair tiles whenever the shape allows
int g_variant = 0;

// Pair-tile width (MMA N) for an M x N output: useful columns x wave occupancy of the pairs.
int pick_bn_pair(int M, int N) {
    const int pairs = std::max(1, num_sms() / 2);
    const int widths[2] = {256, 128};
    const double tile_eff[2] = {1.0, 0.92};
    int best = 256;
    double best_score = -1.0;
    for (int i = 0; i < 2; ++i) {
        const int bn = widths[i];
        const int tn = (N + bn - 1) / bn;
        const double col_eff = static_cast<double>(N) / (static_cast<double>(tn) * bn);
        const long long units = static_cast<long long>((M + kPairRows - 1) / kPairRows) * tn;
        const long long waves = (units + pairs - 1) / pairs;
        const double wave_eff = static_cast<double>(units) / static_cast<double>(waves * pairs);
        const double score = col_eff * wave_eff * tile_eff[i];
        if (score > best_score + 1e-9) {
            best_score = score;
            best = bn;
        }
    }
    return best;
}

struct Plan {
    bool pair;
    int bn, splits;
};

// Variant, tile width and K splits for a product.  Pair tiles halve the per-SM shared-memory
// operand traffic, so they are used whenever the output (or its K splits) still gives every
// pair of SMs work; narrow outputs keep the single-CTA tiles.  MN-major B needs whole 64-column
// boxes per CTA half, hence N % 128 == 0 for pair tiles.
// K splits for `tiles` output tiles on `slots` persistent workers: the count (each split at least
// four K tiles) whose units fill the last wave best, fewer splits on a tie (every split adds an fp32
// partial tile of atomics).  E.g. 36 tiles on 148 SMs -> 4 splits (144 units, one wave), not 5
// (180 units: a second, mostly idle wave).
int best_splits(int tiles, int ktiles, int slots, double* eff_out) {
    int best = 1;
    double best_eff = -1.0;
    for (int s = 1; s <= std::max(1, ktiles / 4); ++s) {
        const long long units = static_cast<long long>(tiles) * s;
        const long long waves = (units + slots - 1) / slots;
        const double eff = static_cast<double>(units) / static_cast<double>(waves * slots) - 0.002 * s;
        if (eff > best_eff + 1e-9) {
            best_eff = eff;
            best = s;
        }
    }
    if (eff_out) *eff_out = best_eff;
    return best;
}

Plan plan_for(int M, int N, int K, bool b_mn, bool splittable) {
    const int sms = num_sms();
    const int ktiles = (K + BK - 1) / BK;
    Plan p{false, pick_bn(M, N), 1};
    const int bn2 = pick_bn_pair(M, N);
    // per shape (variant 0) the single-CTA tiles are used until the pair tiles measure faster
    const bool pair_ok = g_variant == 2 && (!b_mn || N % 128 == 0) && M > BM;
    if (pair_ok) {
        const int tiles2 = ((M + kPairRows - 1) / kPairRows) * ((N + bn2 - 1) / bn2);
        int splits2 = 1;
        if (splittable && tiles2 < sms / 4 && ktiles >= 8) splits2 = best_splits(tiles2, ktiles, sms / 2, nullptr);
        if (g_variant == 2 || tiles2 * splits2 >= sms / 2) return Plan{true, bn2, splits2};
    }
    const int tiles = ((M + BM - 1) / BM) * ((N + p.bn - 1) / p.bn);
    if (splittable && tiles < sms / 2 && ktiles >= 8) {
        // few output tiles, long reduction: tile width and split count together (wider tiles move
        // fewer operand bytes per product, and a width that divides N wastes no columns)
        const int widths[3] = {256, 192, 128};
        const double tile_eff[3] = {1.0, 0.96, 0.88};
        double best_score = -1.0;
        for (int i = 0; i < 3; ++i) {
            const int tn = (N + widths[i] - 1) / widths[i];
            const double col_eff = static_cast<double>(N) / (static_cast<double>(tn) * widths[i]);
            double eff = 0.0;
            const int s = best_splits(((M + BM - 1) / BM) * tn, ktiles, sms, &eff);
            const double score = col_eff * eff * tile_eff[i];
            if (score > best_score + 1e-9) {
                best_score = score;
                p.bn = widths[i];
                p.splits = s;
            }
        }
    }
    return p;
}

}  // namespace

void gemm_tc_set_variant(int v) { g_variant = v; }
int gemm_tc_variant() { return g_variant; }

int gemm_tc_splits(int M, int N, int K, bool b_mn) { return plan_for(M, N, K, b_mn, true).splits; }

cudaError_t launch_gemm_tc(const GemmArgs& g_in, bool a_mn, bool b_mn, int64_t lda, int64_t ldb, cudaStream_t st) {
    GemmArgs g = g_in;
    // The tensor maps are encoded through the driver API, which needs a current
    // context; threads that only used the runtime lazily (e.g. the autograd
    // worker thread) may not have one yet.
    int dev = 0;
    cudaError_t de = cudaGetDevice(&dev);
    if (de == cudaSuccess) de = cudaSetDevice(dev);
    if (de != cudaSuccess) return de;
    if (g.batch < 1) g.batch = 1;
    {
        static const int diag = [] {
            const char* e = std::getenv("MMLTK_GEMM_DIAG");
            return e ? std::atoi(e) : 0;
        }();
        g.diag = diag;
    }
    if (g.batch > 1 && (g.K % BK != 0 || g.ws != nullptr)) return cudaErrorInvalidValue;
    if (g.epi == 7 && (g.rmax == nullptr || g.N > 256)) return cudaErrorInvalidValue;
    Plan plan = plan_for(g.M, g.N, g.K, b_mn, g.ws != nullptr);
    if (g.batch > 1 || g.epi == 7) {
        plan.pair = false;
        plan.bn = pick_bn(g.M, g.N);
    }
    if (g.epi == 7) plan.bn = g.N <= 128 ? 128 : (g.N <= 192 ? 192 : 256);   // one column tile
    const int bn = plan.bn;
    const int rows = plan.pair ? kPairRows : BM;
    const int b_rows = plan.pair ? bn / 2 : bn;     // B rows per CTA (K-major box height)
    CUtensorMap ta, tb;
    // batched products read every batch through one map over the whole operand matrix
    const int64_t ai = g.a_inner ? g.a_inner : (a_mn ? g.M : g.K), ao = g.a_outer ? g.a_outer : (a_mn ? g.K : g.M);
    const int64_t bi = g.b_inner ? g.b_inner : (b_mn ? g.N : g.K), bo = g.b_outer ? g.b_outer : (b_mn ? g.K : g.N);
    bool ok;
    if (g.conv_w) {
        if (a_mn || b_mn || g.conv_c % BK != 0 || g.K != 9 * g.conv_c || g.M != g.conv_w * g.conv_rows ||
            g.M > BM || g.batch % g.conv_groups != 0 || g.ws != nullptr)
            return cudaErrorInvalidValue;
        ok = make_conv_map(&ta, g.A, g.conv_c, g.conv_w, static_cast<int64_t>(g.conv_groups) * g.conv_rows,
                           g.batch / g.conv_groups, g.conv_rows);
    } else {
        ok = a_mn ? make_map(&ta, g.A, ai, ao, lda, 64) : make_map(&ta, g.A, ai, ao, lda, BM);
    }
    ok = ok && (b_mn ? make_map(&tb, g.B, bi, bo, ldb, 64) : make_map(&tb, g.B, bi, bo, ldb, b_rows));
    if (!ok) return cudaErrorInvalidValue;
    Sched sch;
    sch.bn = bn;
    sch.rows = rows;
    sch.m_tiles = (g.M + rows - 1) / rows;
    sch.n_tiles = (g.N + bn - 1) / bn;
    sch.ktiles = (g.K + BK - 1) / BK;
    sch.splits = g.ws ? std::max(1, g.splits) : 1;
    sch.kt_per_split = (sch.ktiles + sch.splits - 1) / sch.splits;
    sch.splits = (sch.ktiles + sch.kt_per_split - 1) / sch.kt_per_split;
    const int units = sch.m_tiles * sch.n_tiles * sch.splits * g.batch;
    const int grid = plan.pair ? 2 * std::min(units, std::max(1, num_sms() / 2)) : std::min(units, num_sms());
    cudaError_t e = cudaSuccess;
    if (g.ws) {
        e = cudaMemsetAsync(g.ws, 0, static_cast<size_t>(g.M) * g.ldc * sizeof(float), st);
        if (e != cudaSuccess) return e;
    }
    // output tensor maps of the single-CTA kernel's epilogue (C, pre-activation): 32 x 32 boxes over
    // [batch, M, N] (pitch ldc, batch stride bs_c), 64-byte swizzle
    CUtensorMap tc_map{}, taux_map{};
    if (g.ws == nullptr && g.epi != 7) {
        const int64_t bs = g.batch > 1 ? g.bs_c : static_cast<int64_t>(g.M) * g.ldc;
        ok = make_store_map(&tc_map, g.C, g.N, g.M, g.batch, g.ldc, bs);
        ok = ok && (g.aux == nullptr || make_store_map(&taux_map, g.aux, g.N, g.M, g.batch, g.ldc, bs));
        if (!ok) return cudaErrorInvalidValue;
    }
    auto launch1 = [&](auto kern, size_t smem) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) {
            std::fprintf(stderr, "gemm_tc: cudaFuncSetAttribute(%zu bytes) failed: %s\n", smem, cudaGetErrorString(e));
            return;
        }
        kern<<<grid, kThreads, smem, st>>>(ta, tb, tc_map, taux_map, g, sch);
        e = cudaGetLastError();
    };
    auto by_major = [&](auto bnc) {
        constexpr int BNv = decltype(bnc)::value;
        const size_t smem = Tile<BNv>::kSmemBytes;
        if (!a_mn && !b_mn) launch1(gemm_tc_kernel<false, false, BNv>, smem);
        else if (!a_mn && b_mn) launch1(gemm_tc_kernel<false, true, BNv>, smem);
        else if (a_mn && b_mn) launch1(gemm_tc_kernel<true, true, BNv>, smem);
        else launch1(gemm_tc_kernel<true, false, BNv>, smem);
    };
    auto by_major_pair = [&](auto bnc) {
        constexpr int BNv = decltype(bnc)::value;
        const size_t smem = PairTile<BNv>::kSmemBytes;
        if (!a_mn && !b_mn) launch1(gemm_tc2_kernel<false, false, BNv>, smem);
        else if (!a_mn && b_mn) launch1(gemm_tc2_kernel<false, true, BNv>, smem);
        else if (a_mn && b_mn) launch1(gemm_tc2_kernel<true, true, BNv>, smem);
        else launch1(gemm_tc2_kernel<true, false, BNv>, smem);
    };
    if (plan.pair) {
        if (bn == 256) by_major_pair(std::integral_constant<int, 256>{});
        else by_major_pair(std::integral_constant<int, 128>{});
    } else if (bn == 256) {
        by_major(std::integral_constant<int, 256>{});
    } else if (bn == 192) {
        by_major(std::integral_constant<int, 192>{});
    } else {
        by_major(std::integral_constant<int, 128>{});
    }
    if (e != cudaSuccess || !g.ws) return e;
    const int64_t n = static_cast<int64_t>(g.M) * g.ldc;
    ws_to_bf16_kernel<<<std::min<int64_t>((n / 8 + 255) / 256, num_sms() * 8), 256, 0, st>>>(g.ws, g.C, n, g.ws_acc);
    return cudaGetLastError();
}

}  // namespace mmltk
