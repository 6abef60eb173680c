// Image-space kernels of the inference / live / visualisation paths (sm_100a):
//
//  * letterbox: a pitched 8-bit 3-channel frame (BGR or RGB) -> the model input in one pass:
//    aspect-preserving scale-to-fit, centred, grey (128) padding, bilinear sampling,
//    channel order, then either [0,1] fp32 planar (the reference's output,
//    `src/rfdetr/cuda/cuda_utils.cu:13-79`) or ImageNet-normalised bf16 planar
//    (fused normalisation -- what the model consumes);
//  * vflip: in-place vertical flip of a pitched 3-channel frame (`cuda_utils.cu:81-98`);
//  * draw: detections onto a pitched 8-bit 3-channel image -- mask alpha blend, box
//    outlines, a filled label bar with text from a built-in 5x7 font (counterpart of
//    `src/rfdetr/cuda/draw_cuda.cu`, headless: the output is a device buffer);
//  * composite: RGBA overlay over a 3-channel image;
//  * resize_masks: batched nearest resize of binary masks (the compiler's mask resize, K16);
//  * pack_masks / sample_packed: bool masks <-> 64-bit words, and nearest sampling of
//    packed masks at normalised points (`mask_pack_cuda.cu:11-31`,
//    `training_mask_ops_cuda.cu:75-159`);
//  * point_sample: bilinear sampling of [N, C, H, W] maps at normalised points with zero
//    padding, align_corners = false (grid_sample semantics), and its input gradient
//    (`training_mask_ops_cuda.cu:34-73`, K6).
#include "common.cuh"

namespace mmltk {

namespace {

// ---------------------------------------------------------------- letterbox
template <bool NORM>
__global__ void letterbox_kernel(const uint8_t* __restrict__ src, int64_t pitch, int sw, int sh, int bgr,
                                 void* __restrict__ dst, int dw, int dh, float scale, float tx, float ty) {
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y;
    if (x >= dw) return;
    // destination pixel centre -> source continuous coordinate (pixel centres at +0.5)
    const float sx = (x + 0.5f - tx) / scale - 0.5f, sy = (y + 0.5f - ty) / scale - 0.5f;
    float c[3] = {128.f, 128.f, 128.f};
    if (sx > -0.5f && sy > -0.5f && sx < sw - 0.5f && sy < sh - 0.5f) {
        const float fx = fminf(fmaxf(sx, 0.f), float(sw - 1)), fy = fminf(fmaxf(sy, 0.f), float(sh - 1));
        const int x0 = int(fx), y0 = int(fy), x1 = min(x0 + 1, sw - 1), y1 = min(y0 + 1, sh - 1);
        const float ax = fx - x0, ay = fy - y0;
        const uint8_t* r0 = src + int64_t(y0) * pitch;
        const uint8_t* r1 = src + int64_t(y1) * pitch;
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const float top = r0[3 * x0 + k] + ax * (r0[3 * x1 + k] - r0[3 * x0 + k]);
            const float bot = r1[3 * x0 + k] + ax * (r1[3 * x1 + k] - r1[3 * x0 + k]);
            c[k] = top + ay * (bot - top);
        }
    }
    const float rgb[3] = {bgr ? c[2] : c[0], c[1], bgr ? c[0] : c[2]};
    const int64_t plane = int64_t(dw) * dh, o = int64_t(y) * dw + x;
    if (NORM) {
        const float mean[3] = {0.485f, 0.456f, 0.406f}, istd[3] = {1.f / 0.229f, 1.f / 0.224f, 1.f / 0.225f};
        auto* d = static_cast<__nv_bfloat16*>(dst);
#pragma unroll
        for (int k = 0; k < 3; ++k) d[k * plane + o] = __float2bfloat16_rn((rgb[k] / 255.f - mean[k]) * istd[k]);
    } else {
        auto* d = static_cast<float*>(dst);
#pragma unroll
        for (int k = 0; k < 3; ++k) d[k * plane + o] = rgb[k] / 255.f;
    }
}

__global__ void vflip_kernel(uint8_t* buf, int64_t pitch, int width, int height) {
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y;
    if (x >= width * 3 || y >= height / 2) return;
    uint8_t* a = buf + int64_t(y) * pitch + x;
    uint8_t* b = buf + int64_t(height - 1 - y) * pitch + x;
    const uint8_t t = *a;
    *a = *b;
    *b = t;
}

// ---------------------------------------------------------------- draw
// 5x7 glyphs, one byte per row (bit 4 = leftmost column).  Index: see glyph_index().
__constant__ uint8_t kFont[][7] = {
    {0x0E, 0x11, 0x13, 0x15, 0x19, 0x11, 0x0E},  // 0
    {0x04, 0x0C, 0x04, 0x04, 0x04, 0x04, 0x0E},  // 1
    {0x0E, 0x11, 0x01, 0x02, 0x04, 0x08, 0x1F},  // 2
    {0x1F, 0x02, 0x04, 0x02, 0x01, 0x11, 0x0E},  // 3
    {0x02, 0x06, 0x0A, 0x12, 0x1F, 0x02, 0x02},  // 4
    {0x1F, 0x10, 0x1E, 0x01, 0x01, 0x11, 0x0E},  // 5
    {0x06, 0x08, 0x10, 0x1E, 0x11, 0x11, 0x0E},  // 6
    {0x1F, 0x01, 0x02, 0x04, 0x08, 0x08, 0x08},  // 7
    {0x0E, 0x11, 0x11, 0x0E, 0x11, 0x11, 0x0E},  // 8
    {0x0E, 0x11, 0x11, 0x0F, 0x01, 0x02, 0x0C},  // 9
    {0x0E, 0x11, 0x11, 0x1F, 0x11, 0x11, 0x11},  // A
    {0x1E, 0x11, 0x11, 0x1E, 0x11, 0x11, 0x1E},  // B
    {0x0E, 0x11, 0x10, 0x10, 0x10, 0x11, 0x0E},  // C
    {0x1C, 0x12, 0x11, 0x11, 0x11, 0x12, 0x1C},  // D
    {0x1F, 0x10, 0x10, 0x1E, 0x10, 0x10, 0x1F},  // E
    {0x1F, 0x10, 0x10, 0x1E, 0x10, 0x10, 0x10},  // F
    {0x0E, 0x11, 0x10, 0x17, 0x11, 0x11, 0x0F},  // G
    {0x11, 0x11, 0x11, 0x1F, 0x11, 0x11, 0x11},  // H
    {0x0E, 0x04, 0x04, 0x04, 0x04, 0x04, 0x0E},  // I
    {0x07, 0x02, 0x02, 0x02, 0x02, 0x12, 0x0C},  // J
    {0x11, 0x12, 0x14, 0x18, 0x14, 0x12, 0x11},  // K
    {0x10, 0x10, 0x10, 0x10, 0x10, 0x10, 0x1F},  // L
    {0x11, 0x1B, 0x15, 0x15, 0x11, 0x11, 0x11},  // M
    {0x11, 0x11, 0x19, 0x15, 0x13, 0x11, 0x11},  // N
    {0x0E, 0x11, 0x11, 0x11, 0x11, 0x11, 0x0E},  // O
    {0x1E, 0x11, 0x11, 0x1E, 0x10, 0x10, 0x10},  // P
    {0x0E, 0x11, 0x11, 0x11, 0x15, 0x12, 0x0D},  // Q
    {0x1E, 0x11, 0x11, 0x1E, 0x14, 0x12, 0x11},  // R
    {0x0F, 0x10, 0x10, 0x0E, 0x01, 0x01, 0x1E},  // S
    {0x1F, 0x04, 0x04, 0x04, 0x04, 0x04, 0x04},  // T
    {0x11, 0x11, 0x11, 0x11, 0x11, 0x11, 0x0E},  // U
    {0x11, 0x11, 0x11, 0x11, 0x11, 0x0A, 0x04},  // V
    {0x11, 0x11, 0x11, 0x15, 0x15, 0x15, 0x0A},  // W
    {0x11, 0x11, 0x0A, 0x04, 0x0A, 0x11, 0x11},  // X
    {0x11, 0x11, 0x11, 0x0A, 0x04, 0x04, 0x04},  // Y
    {0x1F, 0x01, 0x02, 0x04, 0x08, 0x10, 0x1F},  // Z
    {0x00, 0x00, 0x00, 0x00, 0x00, 0x0C, 0x0C},  // .
    {0x18, 0x19, 0x02, 0x04, 0x08, 0x13, 0x03},  // %
    {0x00, 0x0C, 0x0C, 0x00, 0x0C, 0x0C, 0x00},  // :
    {0x00, 0x00, 0x00, 0x1F, 0x00, 0x00, 0x00},  // -
    {0x00, 0x00, 0x00, 0x00, 0x00, 0x00, 0x1F},  // _
};

__device__ __forceinline__ int glyph_index(int ch) {
    if (ch >= '0' && ch <= '9') return ch - '0';
    if (ch >= 'a' && ch <= 'z') ch -= 32;
    if (ch >= 'A' && ch <= 'Z') return 10 + ch - 'A';
    switch (ch) {
        case '.': return 36;
        case '%': return 37;
        case ':': return 38;
        case '-': return 39;
        case '_': return 40;
        default: return -1;   // space and anything else: blank
    }
}

// one thread per output pixel; detections are few, so every pixel scans them (masks first, then
// boxes, then label bars + text on top).  boxes [n,4] xyxy px; colors [n,3] uint8 (image channel
// order); masks [n,H,W] uint8 (optional); text [n, text_len] chars (optional).
__global__ void draw_kernel(uint8_t* __restrict__ img, int64_t pitch, int W, int H, const float* __restrict__ boxes,
                            const uint8_t* __restrict__ colors, const uint8_t* __restrict__ masks,
                            const char* __restrict__ text, int text_len, int n, int thickness, float mask_alpha,
                            int scale) {
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y;
    if (x >= W || y >= H) return;
    uint8_t* p = img + int64_t(y) * pitch + 3 * x;
    float c[3] = {float(p[0]), float(p[1]), float(p[2])};
    const int64_t plane = int64_t(W) * H;
    if (masks) {
        for (int i = 0; i < n; ++i) {
            if (masks[i * plane + int64_t(y) * W + x]) {
#pragma unroll
                for (int k = 0; k < 3; ++k) c[k] += mask_alpha * (colors[3 * i + k] - c[k]);
            }
        }
    }
    const int gw = 6 * scale, gh = 9 * scale;   // glyph cell incl. spacing
    for (int i = 0; i < n; ++i) {
        const float x0 = boxes[4 * i], y0 = boxes[4 * i + 1], x1 = boxes[4 * i + 2], y1 = boxes[4 * i + 3];
        const bool inside = x >= x0 - thickness && x <= x1 + thickness && y >= y0 - thickness && y <= y1 + thickness;
        const bool core = x > x0 + thickness - 1 && x < x1 - thickness + 1 && y > y0 + thickness - 1 &&
                          y < y1 - thickness + 1;
        if (inside && !core) {
#pragma unroll
            for (int k = 0; k < 3; ++k) c[k] = colors[3 * i + k];
        }
        if (text && text_len > 0) {
            // label bar above the box (inside the image)
            const int bx = int(fmaxf(x0, 0.f)), by = int(fmaxf(y0 - gh, 0.f));
            int len = 0;
            while (len < text_len && text[i * text_len + len]) ++len;
            if (len > 0 && x >= bx && x < bx + len * gw + scale && y >= by && y < by + gh) {
#pragma unroll
                for (int k = 0; k < 3; ++k) c[k] = colors[3 * i + k];
                const int cx = (x - bx - scale) / gw, px = (x - bx - scale) % gw, py = (y - by - scale);
                if (x - bx >= scale && cx < len && px < 5 * scale && py >= 0 && py < 7 * scale) {
                    const int gi = glyph_index(text[i * text_len + cx]);
                    if (gi >= 0 && (kFont[gi][py / scale] >> (4 - px / scale)) & 1) {
                        // text in black or white, whichever contrasts with the bar
                        const float lum = 0.3f * colors[3 * i] + 0.59f * colors[3 * i + 1] + 0.11f * colors[3 * i + 2];
                        const float v = lum > 128.f ? 0.f : 255.f;
                        c[0] = c[1] = c[2] = v;
                    }
                }
            }
        }
    }
#pragma unroll
    for (int k = 0; k < 3; ++k) p[k] = uint8_t(fminf(fmaxf(c[k] + 0.5f, 0.f), 255.f));
}

__global__ void composite_kernel(uint8_t* __restrict__ dst, int64_t dpitch, const uint8_t* __restrict__ rgba,
                                 int64_t spitch, int W, int H, int swap_rb) {
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y;
    if (x >= W || y >= H) return;
    const uint8_t* s = rgba + int64_t(y) * spitch + 4 * x;
    uint8_t* d = dst + int64_t(y) * dpitch + 3 * x;
    const float a = s[3] / 255.f;
    const int src_idx[3] = {swap_rb ? 2 : 0, 1, swap_rb ? 0 : 2};
#pragma unroll
    for (int k = 0; k < 3; ++k) d[k] = uint8_t(fminf(d[k] + a * (float(s[src_idx[k]]) - d[k]) + 0.5f, 255.f));
}

// ---------------------------------------------------------------- masks
__global__ void resize_masks_kernel(const uint8_t* __restrict__ src, int sh, int sw, uint8_t* __restrict__ dst,
                                    int dh, int dw) {
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y, n = blockIdx.z;
    if (x >= dw) return;
    const int sy = min(sh - 1, int((y + 0.5f) * sh / dh));
    const int sx = min(sw - 1, int((x + 0.5f) * sw / dw));
    dst[(int64_t(n) * dh + y) * dw + x] = src[(int64_t(n) * sh + sy) * sw + sx] ? 1 : 0;
}

// one warp per 64-bit word: two ballots of 32 pixels each (bit i = pixel 64 * word + i)
__global__ void pack_masks_kernel(const uint8_t* __restrict__ m, int64_t pixels, int64_t words,
                                  unsigned long long* __restrict__ out, int n) {
    const int64_t gw = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) / 32;   // global word index
    const int lane = threadIdx.x & 31;
    if (gw >= int64_t(n) * words) return;   // uniform per warp (blockDim is a multiple of 32)
    const int img = int(gw / words);
    const int64_t word = gw % words;
    const uint8_t* row = m + int64_t(img) * pixels;
    const int64_t p0 = word * 64 + lane, p1 = p0 + 32;
    const unsigned lo = __ballot_sync(0xffffffffu, p0 < pixels && row[p0] != 0);
    const unsigned hi = __ballot_sync(0xffffffffu, p1 < pixels && row[p1] != 0);
    if (lane == 0) out[gw] = (static_cast<unsigned long long>(hi) << 32) | lo;
}

// packed [n, words] masks of H x W, points [n, P, 2] normalised (x, y) -> [n, P] fp32 (nearest)
__global__ void sample_packed_kernel(const unsigned long long* __restrict__ bits, int64_t words, int H, int W,
                                     const float* __restrict__ pts, int P, float* __restrict__ out, int64_t total) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const int64_t n = i / P;
    const float px = pts[2 * i], py = pts[2 * i + 1];
    float v = 0.f;
    if (px >= 0.f && px <= 1.f && py >= 0.f && py <= 1.f) {
        const int x = min(W - 1, max(0, __float2int_rn(px * W - 0.5f)));
        const int y = min(H - 1, max(0, __float2int_rn(py * H - 0.5f)));
        const int64_t pix = int64_t(y) * W + x;
        v = float((bits[n * words + (pix >> 6)] >> (pix & 63)) & 1ull);
    }
    out[i] = v;
}


// ---------------------------------------------------------------- bilinear point sampling
// Corner (k = 0..3) of point (px, py) in an H x W map: index (or -1 outside) and weight.
__device__ __forceinline__ void ps_corner(float px, float py, int H, int W, int k, int& idx, float& w) {
    const float ix = px * W - 0.5f, iy = py * H - 0.5f;
    const float fx = floorf(ix), fy = floorf(iy);
    const int x = int(fx) + (k & 1), y = int(fy) + (k >> 1);
    const float ax = ix - fx, ay = iy - fy;
    w = ((k & 1) ? ax : 1.f - ax) * ((k >> 1) ? ay : 1.f - ay);
    idx = (x >= 0 && x < W && y >= 0 && y < H) ? y * W + x : -1;
}

template <typename T>
__global__ void point_sample_fwd_kernel(const T* __restrict__ inp, int C, int H, int W, const float* __restrict__ pts,
                                        int P, int pts_shared, T* __restrict__ out, int64_t total) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const int p = int(i % P);
    const int64_t nc = i / P;
    const int64_t n = nc / C;
    const float* q = pts + 2 * ((pts_shared ? 0 : n) * P + p);
    const T* m = inp + nc * int64_t(H) * W;
    float v = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        int idx;
        float w;
        ps_corner(q[0], q[1], H, W, k, idx, w);
        if (idx >= 0) v += w * to_f(m[idx]);
    }
    out[i] = from_f<T>(v);
}

template <typename T>
__global__ void point_sample_bwd_kernel(const T* __restrict__ gout, int C, int H, int W, const float* __restrict__ pts,
                                        int P, int pts_shared, float* __restrict__ gin, int64_t total) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const int p = int(i % P);
    const int64_t nc = i / P;
    const int64_t n = nc / C;
    const float* q = pts + 2 * ((pts_shared ? 0 : n) * P + p);
    float* g = gin + nc * int64_t(H) * W;
    const float go = to_f(gout[i]);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        int idx;
        float w;
        ps_corner(q[0], q[1], H, W, k, idx, w);
        if (idx >= 0 && w != 0.f) atomicAdd(g + idx, w * go);
    }
}

}  // namespace

cudaError_t launch_letterbox(const uint8_t* src, int64_t pitch, int sw, int sh, bool bgr, void* dst, int dw, int dh,
                             bool normalize_bf16, cudaStream_t st) {
    if (sw <= 0 || sh <= 0 || dw <= 0 || dh <= 0 || pitch < int64_t(sw) * 3) return cudaErrorInvalidValue;
    const float scale = fminf(float(dw) / sw, float(dh) / sh);
    const float tx = 0.5f * (dw - scale * sw), ty = 0.5f * (dh - scale * sh);
    const dim3 grid((dw + 127) / 128, dh);
    if (normalize_bf16)
        letterbox_kernel<true><<<grid, 128, 0, st>>>(src, pitch, sw, sh, bgr ? 1 : 0, dst, dw, dh, scale, tx, ty);
    else
        letterbox_kernel<false><<<grid, 128, 0, st>>>(src, pitch, sw, sh, bgr ? 1 : 0, dst, dw, dh, scale, tx, ty);
    return cudaGetLastError();
}

cudaError_t launch_vflip(uint8_t* buf, int64_t pitch, int width, int height, cudaStream_t st) {
    if (height < 2) return cudaSuccess;
    const dim3 grid((width * 3 + 255) / 256, height / 2);
    vflip_kernel<<<grid, 256, 0, st>>>(buf, pitch, width, height);
    return cudaGetLastError();
}

cudaError_t launch_draw(uint8_t* img, int64_t pitch, int W, int H, const float* boxes, const uint8_t* colors,
                        const uint8_t* masks, const char* text, int text_len, int n, int thickness, float mask_alpha,
                        int scale, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    const dim3 grid((W + 127) / 128, H);
    draw_kernel<<<grid, 128, 0, st>>>(img, pitch, W, H, boxes, colors, masks, text, text_len, n, thickness,
                                      mask_alpha, max(1, scale));
    return cudaGetLastError();
}

cudaError_t launch_composite(uint8_t* dst, int64_t dpitch, const uint8_t* rgba, int64_t spitch, int W, int H,
                             bool swap_rb, cudaStream_t st) {
    const dim3 grid((W + 127) / 128, H);
    composite_kernel<<<grid, 128, 0, st>>>(dst, dpitch, rgba, spitch, W, H, swap_rb ? 1 : 0);
    return cudaGetLastError();
}

cudaError_t launch_resize_masks(const uint8_t* src, int n, int sh, int sw, uint8_t* dst, int dh, int dw,
                                cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    if (n > 65535) return cudaErrorInvalidValue;
    const dim3 grid((dw + 127) / 128, dh, n);
    resize_masks_kernel<<<grid, 128, 0, st>>>(src, sh, sw, dst, dh, dw);
    return cudaGetLastError();
}

cudaError_t launch_pack_masks(const uint8_t* m, int n, int64_t pixels, uint64_t* out, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    const int64_t words = (pixels + 63) / 64;
    const int64_t threads = int64_t(n) * words * 32;
    pack_masks_kernel<<<unsigned((threads + 255) / 256), 256, 0, st>>>(
        m, pixels, words, reinterpret_cast<unsigned long long*>(out), n);
    return cudaGetLastError();
}

cudaError_t launch_sample_packed(const uint64_t* bits, int n, int H, int W, const float* pts, int P, float* out,
                                 cudaStream_t st) {
    const int64_t total = int64_t(n) * P;
    if (total == 0) return cudaSuccess;
    const int64_t words = (int64_t(H) * W + 63) / 64;
    sample_packed_kernel<<<unsigned((total + 255) / 256), 256, 0, st>>>(
        reinterpret_cast<const unsigned long long*>(bits), words, H, W, pts, P, out, total);
    return cudaGetLastError();
}

cudaError_t launch_point_sample_fwd(DType t, const void* inp, int N, int C, int H, int W, const float* pts, int P,
                                    bool pts_shared, void* out, cudaStream_t st) {
    const int64_t total = int64_t(N) * C * P;
    if (total == 0) return cudaSuccess;
    return MMLTK_DISPATCH_DT(t, [&] {
        point_sample_fwd_kernel<scalar_t><<<unsigned((total + 255) / 256), 256, 0, st>>>(
            static_cast<const scalar_t*>(inp), C, H, W, pts, P, pts_shared ? 1 : 0, static_cast<scalar_t*>(out), total);
        return cudaGetLastError();
    });
}

cudaError_t launch_point_sample_bwd(DType t, const void* gout, int N, int C, int H, int W, const float* pts, int P,
                                    bool pts_shared, float* gin, cudaStream_t st) {
    const int64_t total = int64_t(N) * C * P;
    if (total == 0) return cudaSuccess;
    return MMLTK_DISPATCH_DT(t, [&] {
        point_sample_bwd_kernel<scalar_t><<<unsigned((total + 255) / 256), 256, 0, st>>>(
            static_cast<const scalar_t*>(gout), C, H, W, pts, P, pts_shared ? 1 : 0, gin, total);
        return cudaGetLastError();
    });
}

}  // namespace mmltk
