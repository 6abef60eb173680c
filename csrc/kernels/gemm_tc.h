// Arguments of the tcgen05 GEMM (see gemm_tc.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace mmltk {

struct GemmArgs {
    const __nv_bfloat16* A;
    const __nv_bfloat16* B;
    __nv_bfloat16* C;           // [M, N], row pitch ldc
    __nv_bfloat16* aux;         // optional: pre-activation (acc + bias), same layout as C
    const __nv_bfloat16* bias;  // optional [N]
    const __nv_bfloat16* res;   // epi 3: residual [M, N] (pitch ldc)
    const __nv_bfloat16* gamma; // epi 3: LayerScale [N]
    int* status;                // 0 ok, else a bounded wait gave up (1 producer, 2 MMA, 3 epilogue)
    float* ws;                  // split-K: fp32 [M, N] workspace (zeroed by the launcher); nullptr = no split
    int splits;                 // K splits when ws != nullptr
    int ws_acc;                 // split-K: the conversion adds the existing C (C += product)
    int M, N, K;
    int64_t ldc;
    int epi;                    // 0 none, 1 GELU(erf), 2 ReLU, 3 res + gamma * (acc + bias),
                                // 4 acc * GELU'(res), 5 acc * [res > 0]   (res = pre-activation, backward)
                                // 8 acc * res (res = a stored activation derivative, backward)
                                // 6 alpha * (acc + bias) + beta * res,
                                // 7 row maximum of acc + bias -> rmax (C is not written)
    float* colacc;              // optional fp32 [N]: += column sums of the stored (bf16-rounded) output
    // Batched products: `batch` independent M x N x K products in one launch.  Batch b reads its
    // operands through the same tensor maps with the tile coordinates shifted by b * (a_bk, a_bm)
    // for A (along K, along M) and b * (b_bk, b_bn) for B, and writes C / aux / res at b * bs_c,
    // bias at b * bs_bias.  K must be a multiple of 64 when batch > 1 (a K tail would read the
    // next batch's operand).
    int batch;
    int a_bk, a_bm, b_bk, b_bn;
    int64_t bs_c, bs_bias;
    float alpha, beta;          // epi 6
    float* rmax;                // epi 7: fp32 [2, batch, M], one partial maximum per half of the columns
    // extents of the 2-D operand matrices the tensor maps cover (0: derived from M / N / K)
    int64_t a_inner, a_outer, b_inner, b_outer;
    // Implicit-GEMM 3 x 3 convolution (stride 1, zero padding 1) of a channels-last input [B, H, W, C]
    // (conv_w > 0): the product is batched over tiles of conv_rows image rows (batch index =
    // image * H / conv_rows + row group, M = conv_rows * W output pixels per tile), K = 9 taps x C
    // ordered (tap, channel) with taps row-major over (dy, dx); the A tile of K tile kt is the
    // input box at (channel chunk, x + dx - 1, y + dy - 1, image), loaded through a 4-D tensor map
    // whose zero fill provides the padding.  B = weights [N, 9 * C].
    int conv_w, conv_rows, conv_groups, conv_c;
    // diagnostics (environment MMLTK_GEMM_DIAG, bit mask): 1 = the epilogue reads the accumulator but
    // stores nothing, which times the main loop and the tensor-memory hand-off alone; 2 = the MMA warp
    // commits every stage without issuing its MMAs, which times the loads and the epilogue alone
    int diag;
};

size_t gemm_tc_smem_bytes();
// Image rows per tile of the implicit-GEMM 3 x 3 convolution: the largest r with r * W <= 128 that
// divides H (0 if none).
int conv3x3_tc_rows(int H, int W);
// K splits worth using for this shape (1 = none); only for plain products (no bias / epilogue).
int gemm_tc_splits(int M, int N, int K, bool b_mn);
// 0: single-CTA or CTA-pair tiles chosen per shape; 1: single-CTA only; 2: CTA pairs where allowed.
void gemm_tc_set_variant(int v);
int gemm_tc_variant();
// a_mn: A stored [K, M] (else [M, K]); b_mn: B stored [K, N] (else [N, K]); lda/ldb: row pitch in elements.
cudaError_t launch_gemm_tc(const GemmArgs& g, bool a_mn, bool b_mn, int64_t lda, int64_t ldb, cudaStream_t st);

}  // namespace mmltk
