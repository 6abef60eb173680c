// tcgen05 / TMA / mbarrier primitives shared by the sm_100a tensor-core kernels (inline PTX).
//
//   * mbarriers with transaction counts and BOUNDED waits (a wait that gives up returns false,
//     so a kernel can record an error and leave instead of spinning forever);
//   * 2-D TMA tile loads, each CTA loading its own tiles;
//   * tcgen05.mma kind::f16 (bf16 x bf16 -> fp32 in tensor memory), commit to an mbarrier,
//     shared-memory matrix descriptors for 128-byte swizzled tiles, tcgen05.ld / st of 32 lanes.
#pragma once

#include <cuda.h>

#include <cstdint>

namespace mmltk {
namespace tc {

constexpr long long kWaitLimit = 1ll << 22;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait; false on timeout or when another role has aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, const volatile int* abort) {
    for (long long i = 0; i < kWaitLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255) == 255 && *abort) return false;
    }
    return false;
}
__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* dst, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}
// 4-D TMA tile load (coordinates innermost first; negative / past-the-end coordinates read zeros)
__device__ __forceinline__ void tma_load_4d(const CUtensorMap* map, uint64_t* bar, void* dst, int c0, int c1, int c2,
                                            int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
        "[%2];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}
// Shared-memory matrix descriptor, 128-byte swizzle, sm_100 version field = 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr >> 4) & 0x3fff);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3fff) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3fff) << 32;
    d |= 1ull << 46;  // version
    d |= 2ull << 61;  // SWIZZLE_128B
    return d;
}
// Instruction descriptor: bf16 x bf16 -> f32, M=128, N=n, operand majors.
__host__ __device__ constexpr uint32_t instr_desc(bool a_mn, bool b_mn, int n, int m = 128) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
           (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}
// Descriptor of the 16-wide K slice kk (0..3) of an operand tile.
//   K-major : rows x 128 B, 8-row groups 1024 B apart; K advances 32 B inside the swizzled row.
//   MN-major: 64-wide MN groups (64 K-rows x 128 B = 8 KB) side by side; K advances 16 rows = 2 KB.
template <bool MN>
__device__ __forceinline__ uint64_t operand_desc(uint32_t tile, int kk) {
    if (MN) return smem_desc(tile + kk * 2048, 8192, 1024);
    return smem_desc(tile + kk * 32, 16, 1024);
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 consecutive accumulator columns of this thread's row: two loads, one wait.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr + 16));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 columns from each of two accumulators (e.g. S and dP) of this thread's row: four loads, one wait.
__device__ __forceinline__ void tmem_ld32x2(uint32_t ta, uint32_t tb, float* a, float* b) {
    uint32_t r[64];
#pragma unroll
    for (int c = 0; c < 4; ++c)
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
            : "=r"(r[16 * c + 0]), "=r"(r[16 * c + 1]), "=r"(r[16 * c + 2]), "=r"(r[16 * c + 3]), "=r"(r[16 * c + 4]),
              "=r"(r[16 * c + 5]), "=r"(r[16 * c + 6]), "=r"(r[16 * c + 7]), "=r"(r[16 * c + 8]), "=r"(r[16 * c + 9]),
              "=r"(r[16 * c + 10]), "=r"(r[16 * c + 11]), "=r"(r[16 * c + 12]), "=r"(r[16 * c + 13]),
              "=r"(r[16 * c + 14]), "=r"(r[16 * c + 15])
            : "r"((c < 2 ? ta : tb) + 16 * (c & 1)));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        a[i] = __uint_as_float(r[i]);
        b[i] = __uint_as_float(r[32 + i]);
    }
}

// 64 consecutive accumulator columns of this thread's row: four loads, one wait.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float* v) {
    uint32_t r[64];
#pragma unroll
    for (int c = 0; c < 4; ++c)
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
            : "=r"(r[16 * c + 0]), "=r"(r[16 * c + 1]), "=r"(r[16 * c + 2]), "=r"(r[16 * c + 3]), "=r"(r[16 * c + 4]),
              "=r"(r[16 * c + 5]), "=r"(r[16 * c + 6]), "=r"(r[16 * c + 7]), "=r"(r[16 * c + 8]), "=r"(r[16 * c + 9]),
              "=r"(r[16 * c + 10]), "=r"(r[16 * c + 11]), "=r"(r[16 * c + 12]), "=r"(r[16 * c + 13]),
              "=r"(r[16 * c + 14]), "=r"(r[16 * c + 15])
            : "r"(taddr + 16 * c));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// 128 consecutive accumulator columns of this thread's row: eight loads, one wait.
__device__ __forceinline__ void tmem_ld128(uint32_t taddr, float* v) {
    uint32_t r[128];
#pragma unroll
    for (int c = 0; c < 8; ++c)
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
            : "=r"(r[16 * c + 0]), "=r"(r[16 * c + 1]), "=r"(r[16 * c + 2]), "=r"(r[16 * c + 3]), "=r"(r[16 * c + 4]),
              "=r"(r[16 * c + 5]), "=r"(r[16 * c + 6]), "=r"(r[16 * c + 7]), "=r"(r[16 * c + 8]), "=r"(r[16 * c + 9]),
              "=r"(r[16 * c + 10]), "=r"(r[16 * c + 11]), "=r"(r[16 * c + 12]), "=r"(r[16 * c + 13]),
              "=r"(r[16 * c + 14]), "=r"(r[16 * c + 15])
            : "r"(taddr + 16 * c));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 128; ++i) v[i] = __uint_as_float(r[i]);
}

// Store 16 consecutive accumulator columns of this thread's row (caller issues tcgen05.wait::st).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
        "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
        "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
        : "memory");
}

}  // namespace tc
}  // namespace mmltk
