// Raw-pointer launchers of the sm_100a kernels.  Compiled by nvcc without any
// torch header; the torch-facing wrappers (shape checks, allocation) are in
// the g++-compiled torch_ops.cpp.  Every launcher returns the launch status.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace mmltk {

enum class DType : int { kF32 = 0, kBF16 = 1 };

int num_sms();

// ---------------------------------------------------------------- LayerNorm
// res/sum (both or neither): normalise x + res and store the sum to `sum`; pos/y2 (both or
// neither): also store y + pos to y2.  All [rows, C] of the x dtype.  rscale (weight dtype [C], needs
// res): the normalised input is res + rscale * (x + rbias) instead.
cudaError_t launch_layernorm_fwd(DType xt, DType wt, const void* x, const void* w, const void* b, void* y, float* mean,
                                 float* rstd, int64_t rows, int C, float eps, cudaStream_t st,
                                 const void* res = nullptr, void* sum = nullptr, const void* pos = nullptr,
                                 void* y2 = nullptr, const void* rbias = nullptr, const void* rscale = nullptr,
                                 const int* ymap = nullptr, int64_t yld = 0, int64_t wgroup_rows = 0, int act = 0);
// act = 1: y = SiLU(normalised, affine row) (the backward recomputes the pre-activation from x).
// wgroup_rows > 0: the rows come in groups of that many and group g uses row g of w / b ([groups, C]).
// ymap (optional, int32 [rows]): y row of input row r is ymap[r] (none when negative), row pitch yld --
// a normalised row goes straight to its place in a differently laid out (e.g. un-windowed,
// channel-concatenated) output.
// One launch: gx, and gw / gb written (or added into, `accumulate`) by the last CTA.
// gy2 (optional): a second output gradient added to gy (the y + pos output of the forward).
// gres (optional): added to gx (the gradient x receives through a residual branch).
// gbias2 (optional, weight dtype [C]): column sums of gx (before gres) written / added
// (accumulate2) -- the gradient of a bias fused into the forward's residual input.
cudaError_t launch_layernorm_bwd(DType xt, DType wt, const void* gy, const void* x, const void* w, const float* mean,
                                 const float* rstd, void* gx, void* gw, void* gb, int64_t rows, int C,
                                 bool accumulate, cudaStream_t st, const void* gy2 = nullptr,
                                 const void* gres = nullptr, void* gbias2 = nullptr, bool accumulate2 = false,
                                 const int* gmap = nullptr, int64_t gld = 0, int64_t group_rows = 0,
                                 const void* bvec = nullptr, int act = 0);
// act = 1: backward of a forward with SiLU; bvec = the norm's bias (to recompute the pre-activation).
// group_rows > 0: per-group weights as in the forward; gw / gb are [groups, C].
// gmap (optional, int32 [rows]): the gradient of input row r is gy row gmap[r] (zero when negative),
// row pitch gld -- the backward of a forward with ymap.

// ---------------------------------------------------------------- attention (tcgen05)
// Softmax attention, head dim 64, from the packed projection qkv [nseq * L rows, >= 3 * H * 64]
// (row pitch ld; q / k / v of head h at columns h*64, C + h*64, 2C + h*64, C = H * 64) into
// o [nseq * L, >= C] (row pitch ldo).  lse (optional): [nseq, H, L] natural-log row log-sum-exp.
// status: set non-zero when a bounded wait gave up (the output is then invalid).
cudaError_t launch_attn_fwd_tc(const void* qkv, int64_t ld, int nseq, int L, int H, void* o, int64_t ldo, float* lse,
                               float scale, int* status, cudaStream_t st);
int attn_fwd_tc_blocks_per_sm();   // resident CTAs per SM (registers, shared memory)
// 2 (default): two CTAs per SM at 168 registers; 1: one CTA per SM, no register cap.
void attn_fwd_tc_set_variant(int min_blocks);

// Short-sequence attention (attn_short.cu): L <= 384, head dim 32 or 64, one CTA per (sequence, head).
// Each operand is a row-major bf16 matrix [nseq * L rows, cols] with row pitch ld (elements); head h
// of it starts at column col + h * D.  o / dq / dk / dv are written the same way (row pitch, first
// column); lse [nseq, H, L] natural log (forward output, backward input); delta [nseq, H, L] fp32
// scratch; dq_acc fp32 [nseq * H, L, 64] scratch (head dim 64 only).
struct AttnOperand {
    const void* base;
    int64_t ld;
    int64_t cols;
    int col;
};
bool attn_short_supported(int L, int D);
// forward kernel variant: 1 = one CTA per (sequence, head) with the whole score row in tensor memory,
// 2 = two ping-pong softmax warpgroups over 128-key chunks (online softmax)
void attn_short_set_fwd_variant(int v);
int attn_short_fwd_variant();
// head-dim-32 backward kernel variant: 1 = one 128 x 128 block at a time, 2 = pipelined half-blocks
void attn_short_set_bwd_variant(int v);
int attn_short_bwd_variant();
size_t attn_short_smem_bytes(bool backward);
cudaError_t launch_attn_short_fwd(const AttnOperand& q, const AttnOperand& k, const AttnOperand& v, int nseq, int L,
                                  int H, int D, void* o, int64_t ldo, int ocol, float* lse, float scale, int* status,
                                  cudaStream_t st);
cudaError_t launch_attn_short_bwd(const AttnOperand& q, const AttnOperand& k, const AttnOperand& v,
                                  const AttnOperand& dout, const void* o, int64_t ldo, int ocol, const float* lse,
                                  float* delta, float* dq_acc, int nseq, int L, int H, int D, void* dq, int64_t lddq,
                                  int dqcol, void* dk, int64_t lddk, int dkcol, void* dv, int64_t lddv, int dvcol,
                                  float scale, int* status, cudaStream_t st);

// ---------------------------------------------------------------- debug bounds checks
// A kernel file's reader of its debug status word (read and clear); see MMLTK_DEBUG_CHECK.
using DebugReader = unsigned (*)();
bool register_debug_reader(DebugReader reader);

// ---------------------------------------------------------------- RGBA overlays (overlay.cu)
// uint8 surfaces with a row pitch in bytes; rgba points at 4 host bytes (r, g, b, a)
cudaError_t launch_overlay_detections(uint8_t* ov, int64_t pitch, int W, int H, const float* boxes,
                                      const uint8_t* colors, const uint8_t* masks, int n, int thickness,
                                      uint8_t mask_alpha, cudaStream_t st);
cudaError_t launch_composite_rgba(uint8_t* dst, int64_t dpitch, int dst_channels, const uint8_t* src, int64_t spitch,
                                  int W, int H, bool swap_rb, cudaStream_t st);
cudaError_t launch_copy_rgb_to_rgba(const uint8_t* src, int64_t spitch, uint8_t* dst, int64_t dpitch, int W, int H,
                                    bool swap_rb, uint8_t alpha, cudaStream_t st);
cudaError_t launch_manual_mask(uint8_t* ov, int64_t pitch, int W, int H, int x0, int y0, int w, int h,
                               const uint8_t* mask, const uint8_t* rgba, cudaStream_t st);
cudaError_t launch_manual_mask_runs(uint8_t* ov, int64_t pitch, int W, int H, int x0, int y0, int w, int h,
                                    const uint32_t* runs, int nruns, const uint8_t* rgba, cudaStream_t st);
cudaError_t launch_box_outline(uint8_t* ov, int64_t pitch, int W, int H, int x1, int y1, int x2, int y2, int thickness,
                               const uint8_t* rgba, cudaStream_t st);
cudaError_t launch_selection_handles(uint8_t* ov, int64_t pitch, int W, int H, int x1, int y1, int x2, int y2,
                                     int radius, const uint8_t* rgba, cudaStream_t st);
// segments: edges [m, 2] point indices, or (edges == null) consecutive points, the last joined to the
// first when nsegments == npts (a closed polyline)
cudaError_t launch_segments(uint8_t* ov, int64_t pitch, int W, int H, const int* pts, int npts, const uint32_t* edges,
                            int nsegments, int thickness, const uint8_t* rgba, cudaStream_t st);
cudaError_t launch_points(uint8_t* ov, int64_t pitch, int W, int H, const int* pts, int npts, int radius,
                          const uint8_t* rgba, cudaStream_t st);
cudaError_t launch_label_colors(const int* labels, int n, uint8_t* rgb, cudaStream_t st);

// ---------------------------------------------------------------- sine position embedding
// pos [rows, n] fp32 (n = 2 or 4: x, y[, w, h]); out [rows, n * dim] bf16 in block order y, x[, w, h];
// freq [dim / 2] fp32.  n * dim / 32 must be 8, 16 or 32 and divide dim.
cudaError_t launch_sine_embed_fwd(const float* pos, int64_t rows, int n, int dim, const float* freq, void* out,
                                  cudaStream_t st);
cudaError_t launch_sine_embed_bwd(const float* pos, int64_t rows, int n, int dim, const float* freq, const void* gout,
                                  float* gpos, cudaStream_t st);

// ---------------------------------------------------------------- MSDeformAttn
struct MsdaDims {
    int B, S, Lq, H, L, P, D;
};
cudaError_t launch_msda_fwd(DType t, const void* value, const int* shapes, const int* starts, const void* ref,
                            const void* off, const void* logits, void* out, MsdaDims d, cudaStream_t st);
// gvalue_acc: fp32 [B*S*H*D], gref_acc: fp32 [B*Lq*L*4]; both zeroed by the launcher.
cudaError_t launch_msda_bwd(DType t, const void* gout, const void* value, const int* shapes, const int* starts,
                            const void* ref, const void* off, const void* logits, float* gvalue_acc, float* gref_acc,
                            void* gvalue, void* gref, void* goff, void* glogits, MsdaDims d, cudaStream_t st);

// ---------------------------------------------------------------- matcher
constexpr int kMatcherMaxLayers = 8;
struct MatcherLayers {
    const void* logits[kMatcherMaxLayers];
    const void* boxes[kMatcherMaxLayers];
};
cudaError_t launch_matcher_cost(DType lt, DType bt, MatcherLayers lp, int NL, const int64_t* labels,
                                const float* tboxes, const int32_t* counts, float* cost, int B, int Q, int C, int T,
                                float w_class, float w_bbox, float w_giou, float alpha, cudaStream_t st);
size_t lsap_shared_bytes(int Qg, int T, int warps_per_block);
int lsap_warps_per_block(int Qg, int T);
cudaError_t launch_lsap(const float* cost, const int32_t* counts, int32_t* match, int NL, int B, int G, int Qg, int T,
                        int* status, cudaStream_t st);

// ---------------------------------------------------------------- elementwise
cudaError_t launch_cast_f32(DType dst_t, const float* src, void* dst, int64_t n, cudaStream_t st);

// mode 0: out (+)= colsum(x); mode 1: gout = x * gamma (row-broadcast) and out (+)= colsum(x * pre).
// N % 8 == 0.  One launch (the last CTA of each column
// slab finishes the reduction); launches that share the per-device arrival counters must be
// stream-ordered.  accumulate: add into `out` instead of overwriting it.
constexpr int kMaxCounters = 4096;
constexpr int kReduceAccFloats = 16384;
struct ReduceScratch {
    unsigned* counters;
    float* acc;
};
ReduceScratch reduce_scratch();
// groups > 1: x is [groups, M, N] and out [groups, N] (one column sum per group).
cudaError_t launch_colsum(DType t, DType out_t, int mode, const void* x, const void* pre, const void* gamma,
                          void* gout, int64_t M, int N, void* out, cudaStream_t st, bool accumulate = false,
                          int groups = 1);
// LayerScale + bias backward in one pass: gpre = gy * gamma, ggamma (+)= colsum(gy * pre),
// gbias (+)= colsum(gpre).  2 N <= kReduceAccFloats.
cudaError_t launch_scale_bias_bwd(DType t, DType out_t, const void* gy, const void* pre, const void* gamma, void* gpre,
                                  int64_t M, int N, void* ggamma, bool acc_gamma, void* gbias, bool acc_bias,
                                  cudaStream_t st);
// gx = gy * act'(pre) and, when gb is given, gb (+)= colsum(gx) in the same pass.
cudaError_t launch_act_bwd_bias(DType t, DType out_t, const void* gy, const void* pre, void* gx, int64_t M, int N,
                                int act, void* gb, bool accumulate, cudaStream_t st);
// out (+)= acc; acc = 0 (acc: a column sum accumulated by atomics, e.g. in the GEMM epilogue)
// planar image [B, Cin, H, W] -> patch rows [B * H/p * W/p, Cin * p * p] (p % 8 == 0, W % 8 == 0)
cudaError_t launch_patch_unfold(DType t, const void* img, void* out, int B, int Cin, int H, int W, int p,
                                cudaStream_t st);
// out[rows[i], :] += src[i, :] (bf16 [n, C] -> [R, C], C % 8 == 0, out zeroed by the caller)
cudaError_t launch_index_add_rows(const void* src, const int64_t* rows, void* out, int64_t n, int C, cudaStream_t st);
cudaError_t launch_colacc_finalize(float* acc, DType out_t, void* out, int N, bool accumulate, cudaStream_t st);
// y = GELU(x), erf form; deriv (optional) = GELU'(x).  n % 8 == 0.
cudaError_t launch_gelu_fwd(DType t, const void* x, void* y, int64_t n, cudaStream_t st, void* deriv = nullptr);
// act: 1 = GELU(erf) from the pre-activation, 2 = ReLU, 3 = `pre` holds the stored GELU'.  n % 8 == 0.
cudaError_t launch_act_bwd(DType t, const void* gy, const void* pre, void* gx, int64_t n, int act, cudaStream_t st);

// ---------------------------------------------------------------- losses
int dense_neg_blocks(int64_t n);
// partials: fp32 [dense_neg_blocks(n)], counter: zeroed uint32 (reset by the kernel), out: fp32 [1]
cudaError_t launch_dense_neg_fwd(DType t, const void* x, int64_t n, float coef, float* partials,
                                 unsigned int* counter, float* out, cudaStream_t st);
cudaError_t launch_dense_neg_bwd(DType t, const void* x, const float* g, int64_t n, float coef, void* dx,
                                 cudaStream_t st);

// ---------------------------------------------------------------- matched-pair losses
constexpr int kMatchedMaxLayers = 16;
struct MatchedLayers {
    const void* logits[kMatchedMaxLayers];   // [B, Q, C] per layer
    const void* boxes[kMatchedMaxLayers];    // [B, Q, 4] cxcywh
    void* glogits[kMatchedMaxLayers];        // backward: dense-term gradients, matched terms added in place
    void* gboxes[kMatchedMaxLayers];         // backward: box gradients, written (arrive zeroed)
};
// forward: out [NL, 3] (zeroed by the caller) += per-layer sums (correction, L1, 1 - GIoU);
// backward: out_or_gout = upstream gradient [NL, 3].  match [NL, B, G, T] query or -1;
// tgt [B, T, 4] fp32 cxcywh; labels [B, T]; mode 0 IA-BCE, 1 sigmoid focal.
cudaError_t launch_matched_loss(bool backward, DType lt, DType bt, const MatchedLayers& L, int NL, int B, int Q,
                                int C, int G, int T, const int32_t* match, const float* tgt, const int64_t* labels,
                                int mode, float alpha, float* out_or_gout, cudaStream_t st);

// ---------------------------------------------------------------- augmentation
// in: [B,3,H,W] uint8 (k/255) or fp32 in [0,1]; out: normalised bf16 / fp32; rec: [B,64] host-drawn
// records or null (normalise only); donors: [slots,3,H,W] like `in`; donor_masks: [slots,H,W] uint8.
cudaError_t launch_augment(DType out_t, bool in_u8, const void* in, void* out, const float* rec, const void* donors,
                           const uint8_t* donor_masks, int B, int H, int W, cudaStream_t st);
cudaError_t launch_warp_masks(const uint8_t* src, const uint8_t* donor_masks, const int32_t* rows, const float* rec,
                              uint8_t* out, int N, int H, int W, cudaStream_t st);

// ---------------------------------------------------------------- image ops (imaging.cu)
// src: pitched 8-bit 3-channel frame; dst: [3, dh, dw] fp32 in [0,1] or normalised bf16
cudaError_t launch_letterbox(const uint8_t* src, int64_t pitch, int sw, int sh, bool bgr, void* dst, int dw, int dh,
                             bool normalize_bf16, cudaStream_t st);
cudaError_t launch_vflip(uint8_t* buf, int64_t pitch, int width, int height, cudaStream_t st);
cudaError_t launch_draw(uint8_t* img, int64_t pitch, int W, int H, const float* boxes, const uint8_t* colors,
                        const uint8_t* masks, const char* text, int text_len, int n, int thickness, float mask_alpha,
                        int scale, cudaStream_t st);
cudaError_t launch_composite(uint8_t* dst, int64_t dpitch, const uint8_t* rgba, int64_t spitch, int W, int H,
                             bool swap_rb, cudaStream_t st);
cudaError_t launch_resize_masks(const uint8_t* src, int n, int sh, int sw, uint8_t* dst, int dh, int dw,
                                cudaStream_t st);
cudaError_t launch_pack_masks(const uint8_t* m, int n, int64_t pixels, uint64_t* out, cudaStream_t st);
// bilinear, zero padding, align_corners = false; pts [N or 1, P, 2] normalised (x, y); gin fp32 [N, C, H, W]
// (accumulated: zero it first)
cudaError_t launch_point_sample_fwd(DType t, const void* inp, int N, int C, int H, int W, const float* pts, int P,
                                    bool pts_shared, void* out, cudaStream_t st);
cudaError_t launch_point_sample_bwd(DType t, const void* gout, int N, int C, int H, int W, const float* pts, int P,
                                    bool pts_shared, float* gin, cudaStream_t st);
cudaError_t launch_sample_packed(const uint64_t* bits, int n, int H, int W, const float* pts, int P, float* out,
                                 cudaStream_t st);

// ---------------------------------------------------------------- detection post-process
// logits [B,Q,C], boxes [B,Q,4] cxcywh (normalised); sizes [B,2] (h, w) fp32 or null (fixed_h/w).
// K <= 1024.  Outputs: scores [B,K] f32, labels [B,K] i64, boxes [B,K,4] xyxy pixels, queries [B,K] i32.
// idx [rows, K] (int64): indices of the K largest entries of each row of x [rows, N] (fp32 or bf16),
// value descending, lowest index first on ties; K <= 1024.
cudaError_t launch_row_topk(DType t, const void* x, int64_t rows, int64_t N, int K, int64_t* idx, cudaStream_t st);
cudaError_t launch_topk_postprocess(DType lt, DType bt, const void* logits, const void* boxes, const float* sizes,
                                    int B, int Q, int C, int K, float fixed_h, float fixed_w, float* scores,
                                    int64_t* labels, float* out_boxes, int32_t* queries, cudaStream_t st);

}  // namespace mmltk
