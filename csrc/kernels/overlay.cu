// RGBA overlay rasterisation for the headless live / annotation path (reference: the draw kernels of
// `src/rfdetr/cuda/draw_cuda.cu:207-708`, whose results there are shared with a browser through
// EGL/DMA-BUF; here they land in plain pitched device buffers).
//
// All surfaces are uint8, row pitch in bytes, RGBA = 4 bytes per pixel.  Geometry is integer
// pixel coordinates; a pixel is covered by a stroke when the distance from its centre to the
// stroke's centre line is at most half the thickness (+0.5 so a 1-pixel stroke is one pixel wide),
// and by a disc when its centre lies within the radius.  Each kernel writes colour and alpha; the
// overlay is blended onto a frame by `launch_composite_rgba` ("over" operator).
#include <cstdint>

#include "launch_api.h"

namespace mmltk {

namespace {

__device__ __forceinline__ void put_rgba(uint8_t* img, int64_t pitch, int x, int y, uint8_t r, uint8_t g, uint8_t b,
                                         uint8_t a) {
    uint8_t* p = img + int64_t(y) * pitch + 4 * x;
    p[0] = r;
    p[1] = g;
    p[2] = b;
    p[3] = a;
}

// squared distance from pixel centre (px, py) to segment a-b (integer end points)
__device__ __forceinline__ float seg_dist2(float px, float py, float ax, float ay, float bx, float by) {
    const float dx = bx - ax, dy = by - ay;
    const float len2 = dx * dx + dy * dy;
    float t = len2 > 0.f ? ((px - ax) * dx + (py - ay) * dy) / len2 : 0.f;
    t = fminf(fmaxf(t, 0.f), 1.f);
    const float ex = px - (ax + t * dx), ey = py - (ay + t * dy);
    return ex * ex + ey * ey;
}

// detections into an RGBA overlay: mask pixels get the instance colour at mask_alpha, box
// outlines the instance colour at full alpha, everything else is left as it is
__global__ void overlay_detections_kernel(uint8_t* __restrict__ ov, int64_t pitch, int W, int H,
                                          const float* __restrict__ boxes, const uint8_t* __restrict__ colors,
                                          const uint8_t* __restrict__ masks, int n, int thickness,
                                          uint8_t mask_alpha) {
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y;
    if (x >= W || y >= H) return;
    int hit = -1;
    bool outline = false;
    const int64_t plane = int64_t(W) * H;
    for (int i = 0; i < n; ++i) {
        if (masks && masks[i * plane + int64_t(y) * W + x]) hit = i;
    }
    for (int i = 0; i < n; ++i) {
        const float x0 = boxes[4 * i], y0 = boxes[4 * i + 1], x1 = boxes[4 * i + 2], y1 = boxes[4 * i + 3];
        const bool in = x >= x0 - thickness && x <= x1 + thickness && y >= y0 - thickness && y <= y1 + thickness;
        const bool core = x > x0 + thickness - 1 && x < x1 - thickness + 1 && y > y0 + thickness - 1 &&
                          y < y1 - thickness + 1;
        if (in && !core) {
            hit = i;
            outline = true;
        }
    }
    if (hit < 0) return;
    put_rgba(ov, pitch, x, y, colors[3 * hit], colors[3 * hit + 1], colors[3 * hit + 2], outline ? 255 : mask_alpha);
}

// "over": dst (RGBA or 3-channel) <- src RGBA over dst
__global__ void composite_rgba_kernel(uint8_t* __restrict__ dst, int64_t dpitch, int dch, const uint8_t* __restrict__ src,
                                      int64_t spitch, int W, int H, int swap_rb) {
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y;
    if (x >= W || y >= H) return;
    const uint8_t* s = src + int64_t(y) * spitch + 4 * x;
    uint8_t* d = dst + int64_t(y) * dpitch + dch * x;
    const float a = s[3] * (1.f / 255.f);
    const int si[3] = {swap_rb ? 2 : 0, 1, swap_rb ? 0 : 2};
#pragma unroll
    for (int k = 0; k < 3; ++k) d[k] = uint8_t(fminf(d[k] + a * (float(s[si[k]]) - d[k]) + 0.5f, 255.f));
    if (dch == 4) d[3] = uint8_t(fminf(s[3] + d[3] * (1.f - a) + 0.5f, 255.f));
}

__global__ void copy_rgb_to_rgba_kernel(const uint8_t* __restrict__ src, int64_t spitch, uint8_t* __restrict__ dst,
                                        int64_t dpitch, int W, int H, int swap_rb, uint8_t alpha) {
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y;
    if (x >= W || y >= H) return;
    const uint8_t* s = src + int64_t(y) * spitch + 3 * x;
    put_rgba(dst, dpitch, x, y, s[swap_rb ? 2 : 0], s[1], s[swap_rb ? 0 : 2], alpha);
}

// a binary mask [h, w] written into the overlay region at (x0, y0)
__global__ void manual_mask_kernel(uint8_t* __restrict__ ov, int64_t pitch, int W, int H, int x0, int y0, int w, int h,
                                   const uint8_t* __restrict__ mask, uchar4 color) {
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y;
    if (x >= w || y >= h) return;
    const int gx = x0 + x, gy = y0 + y;
    if (gx < 0 || gy < 0 || gx >= W || gy >= H || !mask[int64_t(y) * w + x]) return;
    put_rgba(ov, pitch, gx, gy, color.x, color.y, color.z, color.w);
}

// run-length mask: pairs (start, length) of row-major indices inside a w-wide region at (x0, y0);
// one block per run
__global__ void manual_mask_runs_kernel(uint8_t* __restrict__ ov, int64_t pitch, int W, int H, int x0, int y0, int w,
                                        int h, const uint32_t* __restrict__ runs, uchar4 color) {
    const uint32_t start = runs[2 * blockIdx.x], len = runs[2 * blockIdx.x + 1];
    for (uint32_t i = threadIdx.x; i < len; i += blockDim.x) {
        const uint32_t idx = start + i;
        const int rx = int(idx % uint32_t(w)), ry = int(idx / uint32_t(w));
        if (ry >= h) break;
        const int gx = x0 + rx, gy = y0 + ry;
        if (gx >= 0 && gy >= 0 && gx < W && gy < H) put_rgba(ov, pitch, gx, gy, color.x, color.y, color.z, color.w);
    }
}

// rectangle outline of the given thickness (inside and outside the box edge), over its padded
// bounding rectangle
__global__ void box_outline_kernel(uint8_t* __restrict__ ov, int64_t pitch, int W, int H, int x1, int y1, int x2, int y2,
                                   int t, int cx0, int cy0, int cx1, int cy1, uchar4 color) {
    const int x = cx0 + blockIdx.x * blockDim.x + threadIdx.x, y = cy0 + blockIdx.y;
    if (x > cx1 || y > cy1) return;
    const bool core = x > x1 + t - 1 && x < x2 - t + 1 && y > y1 + t - 1 && y < y2 - t + 1;
    if (!core) put_rgba(ov, pitch, x, y, color.x, color.y, color.z, color.w);
}

// eight square handles (corners and edge midpoints) of half-size r; block z = handle
__global__ void selection_handles_kernel(uint8_t* __restrict__ ov, int64_t pitch, int W, int H, int x1, int y1, int x2,
                                         int y2, int r, uchar4 color) {
    const int hx[8] = {x1, (x1 + x2) / 2, x2, x2, x2, (x1 + x2) / 2, x1, x1};
    const int hy[8] = {y1, y1, y1, (y1 + y2) / 2, y2, y2, y2, (y1 + y2) / 2};
    const int k = blockIdx.z;
    const int x = hx[k] - r + blockIdx.x * blockDim.x + threadIdx.x, y = hy[k] - r + blockIdx.y;
    if (x > hx[k] + r || x < 0 || y < 0 || x >= W || y >= H) return;
    put_rgba(ov, pitch, x, y, color.x, color.y, color.z, color.w);
}

// thick line segments: block = (segment, row of its padded bounding box); points [n, 2] int xy,
// edges [m, 2] uint32 point indices (or consecutive points when edges is null)
__global__ void segments_kernel(uint8_t* __restrict__ ov, int64_t pitch, int W, int H, const int* __restrict__ pts,
                                int npts, const uint32_t* __restrict__ edges, int thickness, uchar4 color) {
    const int s = blockIdx.y;
    uint32_t ia, ib;
    if (edges) {
        ia = edges[2 * s];
        ib = edges[2 * s + 1];
    } else {
        ia = uint32_t(s);
        ib = uint32_t(s + 1 < npts ? s + 1 : 0);
    }
    if (ia >= uint32_t(npts) || ib >= uint32_t(npts)) return;
    const int ax = pts[2 * ia], ay = pts[2 * ia + 1], bx = pts[2 * ib], by = pts[2 * ib + 1];
    const float half = 0.5f * thickness;
    const int pad = (thickness + 1) / 2;
    // the stroke's bounding box, clipped to the image (so far-off coordinates cost nothing)
    const int xmin = max(min(ax, bx) - pad, 0), xmax = min(max(ax, bx) + pad, W - 1);
    const int ymin = max(min(ay, by) - pad, 0), ymax = min(max(ay, by) + pad, H - 1);
    for (int y = ymin + blockIdx.x; y <= ymax; y += gridDim.x) {
        for (int x = xmin + int(threadIdx.x); x <= xmax; x += blockDim.x) {
            if (seg_dist2(float(x), float(y), float(ax), float(ay), float(bx), float(by)) <= half * half + 0.25f)
                put_rgba(ov, pitch, x, y, color.x, color.y, color.z, color.w);
        }
    }
}

// filled discs of radius r; block = point
__global__ void points_kernel(uint8_t* __restrict__ ov, int64_t pitch, int W, int H, const int* __restrict__ pts, int r,
                              uchar4 color) {
    const int cx = pts[2 * blockIdx.x], cy = pts[2 * blockIdx.x + 1];
    const int side = 2 * r + 1;
    for (int i = threadIdx.x; i < side * side; i += blockDim.x) {
        const int dx = i % side - r, dy = i / side - r;
        const int x = cx + dx, y = cy + dy;
        if (dx * dx + dy * dy > r * r || x < 0 || y < 0 || x >= W || y >= H) continue;
        put_rgba(ov, pitch, x, y, color.x, color.y, color.z, color.w);
    }
}

// per-instance colour from a label: an evenly spread hue wheel (golden-angle steps), full
// saturation / value, so neighbouring class ids get distant colours
__global__ void label_colors_kernel(const int* __restrict__ labels, int n, uint8_t* __restrict__ rgb) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float hue = fmodf(float(max(labels[i], 0)) * 0.618033988749895f, 1.f) * 6.f;
    const int sector = int(hue);
    const float f = hue - float(sector);
    const float q = 1.f - f;
    float r, g, b;
    switch (sector % 6) {
        case 0: r = 1.f, g = f, b = 0.f; break;
        case 1: r = q, g = 1.f, b = 0.f; break;
        case 2: r = 0.f, g = 1.f, b = f; break;
        case 3: r = 0.f, g = q, b = 1.f; break;
        case 4: r = f, g = 0.f, b = 1.f; break;
        default: r = 1.f, g = 0.f, b = q; break;
    }
    rgb[3 * i] = uint8_t(r * 255.f + 0.5f);
    rgb[3 * i + 1] = uint8_t(g * 255.f + 0.5f);
    rgb[3 * i + 2] = uint8_t(b * 255.f + 0.5f);
}

inline dim3 rows_grid(int w, int h) { return dim3((w + 127) / 128, h); }

}  // namespace

cudaError_t launch_overlay_detections(uint8_t* ov, int64_t pitch, int W, int H, const float* boxes,
                                      const uint8_t* colors, const uint8_t* masks, int n, int thickness,
                                      uint8_t mask_alpha, cudaStream_t st) {
    if (W <= 0 || H <= 0 || n <= 0) return cudaSuccess;
    overlay_detections_kernel<<<rows_grid(W, H), 128, 0, st>>>(ov, pitch, W, H, boxes, colors, masks, n, thickness,
                                                               mask_alpha);
    return cudaGetLastError();
}

cudaError_t launch_composite_rgba(uint8_t* dst, int64_t dpitch, int dst_channels, const uint8_t* src, int64_t spitch,
                                  int W, int H, bool swap_rb, cudaStream_t st) {
    if (W <= 0 || H <= 0) return cudaSuccess;
    if (dst_channels != 3 && dst_channels != 4) return cudaErrorInvalidValue;
    composite_rgba_kernel<<<rows_grid(W, H), 128, 0, st>>>(dst, dpitch, dst_channels, src, spitch, W, H, swap_rb ? 1 : 0);
    return cudaGetLastError();
}

cudaError_t launch_copy_rgb_to_rgba(const uint8_t* src, int64_t spitch, uint8_t* dst, int64_t dpitch, int W, int H,
                                    bool swap_rb, uint8_t alpha, cudaStream_t st) {
    if (W <= 0 || H <= 0) return cudaSuccess;
    copy_rgb_to_rgba_kernel<<<rows_grid(W, H), 128, 0, st>>>(src, spitch, dst, dpitch, W, H, swap_rb ? 1 : 0, alpha);
    return cudaGetLastError();
}

cudaError_t launch_manual_mask(uint8_t* ov, int64_t pitch, int W, int H, int x0, int y0, int w, int h,
                               const uint8_t* mask, const uint8_t* rgba, cudaStream_t st) {
    if (w <= 0 || h <= 0) return cudaSuccess;
    manual_mask_kernel<<<rows_grid(w, h), 128, 0, st>>>(ov, pitch, W, H, x0, y0, w, h, mask,
                                                        make_uchar4(rgba[0], rgba[1], rgba[2], rgba[3]));
    return cudaGetLastError();
}

cudaError_t launch_manual_mask_runs(uint8_t* ov, int64_t pitch, int W, int H, int x0, int y0, int w, int h,
                                    const uint32_t* runs, int nruns, const uint8_t* rgba, cudaStream_t st) {
    if (nruns <= 0 || w <= 0) return cudaSuccess;
    manual_mask_runs_kernel<<<nruns, 128, 0, st>>>(ov, pitch, W, H, x0, y0, w, h, runs,
                                                   make_uchar4(rgba[0], rgba[1], rgba[2], rgba[3]));
    return cudaGetLastError();
}

cudaError_t launch_box_outline(uint8_t* ov, int64_t pitch, int W, int H, int x1, int y1, int x2, int y2, int thickness,
                               const uint8_t* rgba, cudaStream_t st) {
    const int t = thickness < 1 ? 1 : thickness;
    // the outline's padded rectangle clipped to the image
    const int cx0 = x1 - t > 0 ? x1 - t : 0, cy0 = y1 - t > 0 ? y1 - t : 0;
    const int cx1 = x2 + t < W - 1 ? x2 + t : W - 1, cy1 = y2 + t < H - 1 ? y2 + t : H - 1;
    if (cx1 < cx0 || cy1 < cy0) return cudaSuccess;
    box_outline_kernel<<<rows_grid(cx1 - cx0 + 1, cy1 - cy0 + 1), 128, 0, st>>>(
        ov, pitch, W, H, x1, y1, x2, y2, t, cx0, cy0, cx1, cy1, make_uchar4(rgba[0], rgba[1], rgba[2], rgba[3]));
    return cudaGetLastError();
}

cudaError_t launch_selection_handles(uint8_t* ov, int64_t pitch, int W, int H, int x1, int y1, int x2, int y2,
                                     int radius, const uint8_t* rgba, cudaStream_t st) {
    const int r = radius < 1 ? 1 : radius;
    dim3 grid((2 * r + 1 + 127) / 128, 2 * r + 1, 8);
    selection_handles_kernel<<<grid, 128, 0, st>>>(ov, pitch, W, H, x1, y1, x2, y2, r,
                                                   make_uchar4(rgba[0], rgba[1], rgba[2], rgba[3]));
    return cudaGetLastError();
}

cudaError_t launch_segments(uint8_t* ov, int64_t pitch, int W, int H, const int* pts, int npts, const uint32_t* edges,
                            int nsegments, int thickness, const uint8_t* rgba, cudaStream_t st) {
    if (nsegments <= 0 || npts <= 0) return cudaSuccess;
    const int t = thickness < 1 ? 1 : thickness;
    dim3 grid(8, nsegments);   // the rows of a segment's clipped box are spread over grid.x blocks
    segments_kernel<<<grid, 128, 0, st>>>(ov, pitch, W, H, pts, npts, edges, t,
                                          make_uchar4(rgba[0], rgba[1], rgba[2], rgba[3]));
    return cudaGetLastError();
}

cudaError_t launch_points(uint8_t* ov, int64_t pitch, int W, int H, const int* pts, int npts, int radius,
                          const uint8_t* rgba, cudaStream_t st) {
    if (npts <= 0) return cudaSuccess;
    points_kernel<<<npts, 128, 0, st>>>(ov, pitch, W, H, pts, radius < 0 ? 0 : radius,
                                        make_uchar4(rgba[0], rgba[1], rgba[2], rgba[3]));
    return cudaGetLastError();
}

cudaError_t launch_label_colors(const int* labels, int n, uint8_t* rgb, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    label_colors_kernel<<<(n + 127) / 128, 128, 0, st>>>(labels, n, rgb);
    return cudaGetLastError();
}

}  // namespace mmltk
