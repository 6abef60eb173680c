// Sine position embedding of decoder reference boxes (reference `model.cpp:234-261`):
//   for each row r and output block b (coordinate c = order[b]: y, x[, w, h]),
//   out[r, b*dim + 2i]   = sin(v * f_i),  out[r, b*dim + 2i+1] = cos(v * f_i),
//   v = pos[r, c],  f_i = 2 pi / 10000^(2i / dim).
// Forward reads 4 floats and writes dim*n bf16 per row in one pass; backward reduces
//   d pos[r, c] = sum_i f_i (g[2i] cos(v f_i) - g[2i+1] sin(v f_i))
// over the block with warp shuffles.  One warp per row, each lane owns a contiguous run of
// (n * dim / 32) outputs inside one block.
#include "common.cuh"

namespace mmltk {

namespace {

constexpr int kPeWarps = 8;

__device__ __forceinline__ int pe_coord(int block) { return block < 2 ? 1 - block : block; }

template <int PER_LANE>
__global__ void __launch_bounds__(kPeWarps * 32) sine_embed_fwd_kernel(const float* __restrict__ pos, int64_t rows,
                                                                        int n, int dim, const float* __restrict__ freq,
                                                                        __nv_bfloat16* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t r = static_cast<int64_t>(blockIdx.x) * kPeWarps + (threadIdx.x >> 5);
    if (r >= rows) return;
    const int j0 = lane * PER_LANE;            // first output column of this lane
    const int block = j0 / dim;
    const float v = pos[r * n + pe_coord(block)];
    const int i0 = (j0 % dim) >> 1;            // first frequency index
    uint32_t w[PER_LANE / 2];
#pragma unroll
    for (int k = 0; k < PER_LANE / 2; ++k) {
        float s, c;
        sincosf(v * __ldg(freq + i0 + k), &s, &c);
        w[k] = pack_bf16x2(s, c);
    }
    uint4* dst = reinterpret_cast<uint4*>(out + r * static_cast<int64_t>(n) * dim + j0);
#pragma unroll
    for (int q = 0; q < PER_LANE / 8; ++q) dst[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
}

template <int PER_LANE>
__global__ void __launch_bounds__(kPeWarps * 32) sine_embed_bwd_kernel(const float* __restrict__ pos, int64_t rows,
                                                                        int n, int dim, const float* __restrict__ freq,
                                                                        const __nv_bfloat16* __restrict__ gout,
                                                                        float* __restrict__ gpos) {
    const int lane = threadIdx.x & 31;
    const int64_t r = static_cast<int64_t>(blockIdx.x) * kPeWarps + (threadIdx.x >> 5);
    if (r >= rows) return;
    const int j0 = lane * PER_LANE;
    const int block = j0 / dim;
    const int c = pe_coord(block);
    const float v = pos[r * n + c];
    const int i0 = (j0 % dim) >> 1;
    const uint4* src = reinterpret_cast<const uint4*>(gout + r * static_cast<int64_t>(n) * dim + j0);
    float acc = 0.f;
#pragma unroll
    for (int q = 0; q < PER_LANE / 8; ++q) {
        const uint4 g4 = src[q];
        const uint32_t gw[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float f = __ldg(freq + i0 + 4 * q + k);
            float s, co;
            sincosf(v * f, &s, &co);
            const float2 g = unpack_bf16x2(gw[k]);
            acc += f * (g.x * co - g.y * s);
        }
    }
    // the lanes of one block are consecutive: reduce within groups of dim / PER_LANE lanes
    const int group = dim / PER_LANE;
    for (int o = group >> 1; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((lane % group) == 0) gpos[r * n + c] = acc;
}

template <typename F>
cudaError_t pe_dispatch(int n, int dim, F&& f) {
    const int total = n * dim;
    if (total % 32 != 0) return cudaErrorInvalidValue;
    const int per = total / 32;
    // a lane's run must stay inside one block and be a whole number of 16-byte vectors
    if (per % 8 != 0 || dim % per != 0) return cudaErrorInvalidValue;
    switch (per) {
        case 8: return f(std::integral_constant<int, 8>{});
        case 16: return f(std::integral_constant<int, 16>{});
        case 32: return f(std::integral_constant<int, 32>{});
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

cudaError_t launch_sine_embed_fwd(const float* pos, int64_t rows, int n, int dim, const float* freq, void* out,
                                  cudaStream_t st) {
    if (rows == 0) return cudaSuccess;
    const unsigned blocks = static_cast<unsigned>((rows + kPeWarps - 1) / kPeWarps);
    return pe_dispatch(n, dim, [&](auto pl) {
        sine_embed_fwd_kernel<decltype(pl)::value><<<blocks, kPeWarps * 32, 0, st>>>(
            pos, rows, n, dim, freq, static_cast<__nv_bfloat16*>(out));
        return cudaGetLastError();
    });
}

cudaError_t launch_sine_embed_bwd(const float* pos, int64_t rows, int n, int dim, const float* freq, const void* gout,
                                  float* gpos, cudaStream_t st) {
    if (rows == 0) return cudaSuccess;
    const unsigned blocks = static_cast<unsigned>((rows + kPeWarps - 1) / kPeWarps);
    return pe_dispatch(n, dim, [&](auto pl) {
        sine_embed_bwd_kernel<decltype(pl)::value><<<blocks, kPeWarps * 32, 0, st>>>(
            pos, rows, n, dim, freq, static_cast<const __nv_bfloat16*>(gout), gpos);
        return cudaGetLastError();
    });
}

}  // namespace mmltk
