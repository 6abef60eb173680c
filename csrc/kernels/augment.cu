// Fused training augmentation + normalisation (sm_100a).
//
// One launch turns a batch of planar RGB images in [0, 1] (uint8 k/255 from the
// loader, or fp32) into the model input: ImageNet-normalised bf16 (or fp32)
// [B, 3, H, W].  Everything between is fused into the same pass: the geometric
// resample (inverse affine, bilinear, lerp towards the 2x2 box average for
// blur, out-of-frame pixels filled with the channel mean), the single-instance
// copy-paste from the donor cache, the colour matrix, gaussian / salt noise and
// the occlusions.  This replaces the reference's parameter kernel, its two image
// kernels and its separate normalisation kernel
// (`src/rfdetr/cuda/gpu_augment_cuda.cu:138-569`) with one pass that reads the
// input once and writes bf16 with 16-byte stores.
//
// Each image's parameters are a 64-float record drawn on the host
// (csrc/host/augment.cpp, same offsets); with no record (null) the kernel only
// normalises.  Each thread produces 8 consecutive pixels of one row for the 3
// channels.  A second kernel warps the target masks with the same records.
#include "common.cuh"

namespace mmltk {

namespace {

enum Rec : int {
    kInv = 0, kFwd = 6, kColor = 12, kColorOff = 21, kNoiseMode = 24, kNoiseStr = 25, kBlur = 26, kOccMode = 27,
    kOccStr = 28, kOccChan = 29, kErase = 30, kAreaScale = 34, kFlags = 35, kPasteSlot = 36, kPasteMode = 37,
    kPasteInv = 38, kNoiseKey = 44, kPasteBox = 45, kRecFloats = 64,
};

__constant__ float kMean[3] = {0.485f, 0.456f, 0.406f};
__constant__ float kInvStd[3] = {1.f / 0.229f, 1.f / 0.224f, 1.f / 0.225f};

// lowbias32 integer finaliser; the host copy in csrc/host/augment.cpp must stay identical.
__device__ __forceinline__ uint32_t hash32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352dU;
    x ^= x >> 15;
    x *= 0x846ca68bU;
    x ^= x >> 16;
    return x;
}
__device__ __forceinline__ float uniform(uint32_t key, uint32_t counter) {
    return float(hash32(key ^ hash32(counter + 0x68e31da4U)) >> 8) * (1.0f / 16777216.0f);
}

template <typename In>
__device__ __forceinline__ float px(const In* p, int64_t i);
template <>
__device__ __forceinline__ float px<uint8_t>(const uint8_t* p, int64_t i) { return float(p[i]) * (1.f / 255.f); }
template <>
__device__ __forceinline__ float px<float>(const float* p, int64_t i) { return p[i]; }

// Bilinear sample (align_corners = false, clamped) of one plane at normalised
// (sx, sy), lerped towards the 2x2 box average by `blur`; outside the frame the
// channel mean.
template <typename In>
__device__ __forceinline__ float sample(const In* plane, int H, int W, float sx, float sy, float blur, int c) {
    if (sx < 0.f || sx > 1.f || sy < 0.f || sy > 1.f) return kMean[c];
    const float fx = fminf(fmaxf(sx * W - 0.5f, 0.f), float(W - 1));
    const float fy = fminf(fmaxf(sy * H - 0.5f, 0.f), float(H - 1));
    const int x0 = int(fx), y0 = int(fy);
    const int x1 = min(W - 1, x0 + 1), y1 = min(H - 1, y0 + 1);
    const float ax = fx - float(x0), ay = fy - float(y0);
    const float v00 = px(plane, int64_t(y0) * W + x0), v01 = px(plane, int64_t(y0) * W + x1);
    const float v10 = px(plane, int64_t(y1) * W + x0), v11 = px(plane, int64_t(y1) * W + x1);
    const float top = fmaf(ax, v01 - v00, v00), bot = fmaf(ax, v11 - v10, v10);
    const float bil = fmaf(ay, bot - top, top);
    const float box = 0.25f * (v00 + v01 + v10 + v11);
    return fmaf(blur, box - bil, bil);
}

__device__ __forceinline__ bool mask_at(const uint8_t* m, int H, int W, float sx, float sy) {
    if (m == nullptr || sx < 0.f || sx > 1.f || sy < 0.f || sy > 1.f) return false;
    const int x = min(W - 1, max(0, __float2int_rn(sx * W - 0.5f)));
    const int y = min(H - 1, max(0, __float2int_rn(sy * H - 0.5f)));
    return m[int64_t(y) * W + x] != 0;
}

// colour, noise, occlusion, clamp and normalisation of one pixel (values in [0, 1] in, normalised out)
__device__ __forceinline__ void effects(float& r, float& g, float& b, const float* R, uint32_t key, int64_t pix,
                                        float nx, float ny) {
    const float r0 = r, g0 = g, b0 = b;
    r = R[kColor + 0] * r0 + R[kColor + 1] * g0 + R[kColor + 2] * b0 + R[kColorOff + 0];
    g = R[kColor + 3] * r0 + R[kColor + 4] * g0 + R[kColor + 5] * b0 + R[kColorOff + 1];
    b = R[kColor + 6] * r0 + R[kColor + 7] * g0 + R[kColor + 8] * b0 + R[kColorOff + 2];
    const int noise = int(R[kNoiseMode]);
    const uint32_t ctr = uint32_t(pix) * 16u;
    if (noise == 1) {
        // Irwin-Hall sum of four uniforms, centred: variance 1/3
        const float sig = 0.06f * R[kNoiseStr];
        float n3[3];
#pragma unroll
        for (int c = 0; c < 3; ++c)
            n3[c] = uniform(key, ctr + 4 * c) + uniform(key, ctr + 4 * c + 1) + uniform(key, ctr + 4 * c + 2) +
                    uniform(key, ctr + 4 * c + 3) - 2.f;
        r = fmaf(sig, n3[0], r);
        g = fmaf(sig, n3[1], g);
        b = fmaf(sig, n3[2], b);
    } else if (noise == 2 && uniform(key, ctr + 12) < 0.02f * R[kNoiseStr]) {
        r = g = b = 1.f;
    }
    const int occ = int(R[kOccMode]);
    bool erase = false;
    if (occ == 2) {
        erase = uniform(key, ctr + 13) < 0.05f * R[kOccStr];
    } else if (occ == 3) {
        erase = nx >= R[kErase + 0] && nx < R[kErase + 2] && ny >= R[kErase + 1] && ny < R[kErase + 3];
    }
    if (erase) {
        r = kMean[0];
        g = kMean[1];
        b = kMean[2];
    } else if (occ == 1) {
        const int c = int(R[kOccChan]);
        const float s = R[kOccStr];
        if (c == 0) r = fmaf(s, kMean[0] - r, r);
        else if (c == 1) g = fmaf(s, kMean[1] - g, g);
        else b = fmaf(s, kMean[2] - b, b);
    }
    r = (fminf(fmaxf(r, 0.f), 1.f) - kMean[0]) * kInvStd[0];
    g = (fminf(fmaxf(g, 0.f), 1.f) - kMean[1]) * kInvStd[1];
    b = (fminf(fmaxf(b, 0.f), 1.f) - kMean[2]) * kInvStd[2];
}

template <typename In>
__device__ __forceinline__ void load_row8(const In* p, float* f);
template <>
__device__ __forceinline__ void load_row8<uint8_t>(const uint8_t* p, float* f) {
    const uint2 raw = *reinterpret_cast<const uint2*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[i] = float((raw.x >> (8 * i)) & 0xffu) * (1.f / 255.f);
        f[4 + i] = float((raw.y >> (8 * i)) & 0xffu) * (1.f / 255.f);
    }
}
template <>
__device__ __forceinline__ void load_row8<float>(const float* p, float* f) {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

template <typename Out>
__device__ __forceinline__ void store_row8(Out* p, const float* f);
template <>
__device__ __forceinline__ void store_row8<__nv_bfloat16>(__nv_bfloat16* p, const float* f) {
    uint4 w;
    w.x = pack_bf16x2(f[0], f[1]);
    w.y = pack_bf16x2(f[2], f[3]);
    w.z = pack_bf16x2(f[4], f[5]);
    w.w = pack_bf16x2(f[6], f[7]);
    *reinterpret_cast<uint4*>(p) = w;
}
template <>
__device__ __forceinline__ void store_row8<float>(float* p, const float* f) {
    *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(f[4], f[5], f[6], f[7]);
}

template <typename In, typename Out>
__global__ void __launch_bounds__(256) augment_kernel(const In* __restrict__ in, Out* __restrict__ out,
                                                      const float* __restrict__ rec, const In* __restrict__ donors,
                                                      const uint8_t* __restrict__ donor_masks, int H, int W) {
    __shared__ float R[kRecFloats];
    const int b = blockIdx.y;
    if (threadIdx.x < kRecFloats) {
        float v;
        if (rec != nullptr) {
            v = rec[int64_t(b) * kRecFloats + threadIdx.x];
        } else {  // identity record: normalisation only
            const int t = threadIdx.x;
            v = (t == kInv || t == kInv + 4 || t == kFwd || t == kFwd + 4 || t == kColor || t == kColor + 4 ||
                 t == kColor + 8 || t == kAreaScale || t == kPasteInv || t == kPasteInv + 4) ? 1.f
                : (t == kPasteSlot ? -1.f : 0.f);
        }
        R[threadIdx.x] = v;
    }
    __syncthreads();
    const int gx = (W + 7) / 8;
    const int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= int64_t(gx) * H) return;
    const int y = int(t / gx), x0 = int(t % gx) * 8;
    const int64_t plane = int64_t(H) * W;
    const In* src = in + int64_t(b) * 3 * plane;
    Out* dst = out + int64_t(b) * 3 * plane;
    const uint32_t key = __float_as_uint(R[kNoiseKey]);
    const bool full = (W % 8 == 0);  // whole 8-pixel group inside the row and 16-byte aligned
    float c3[3][8];
    const bool remap = R[kFlags] != 0.f;
    const float ny = (float(y) + 0.5f) / float(H);
    if (!remap && full) {
#pragma unroll
        for (int c = 0; c < 3; ++c) load_row8(src + c * plane + int64_t(y) * W + x0, c3[c]);
    } else {
        const int slot = int(R[kPasteSlot]);
        const int pmode = int(R[kPasteMode]);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int x = min(x0 + i, W - 1);
            const float nx = (float(x) + 0.5f) / float(W);
            float v[3];
            if (remap) {
                const float sx = R[kInv + 0] * nx + R[kInv + 1] * ny + R[kInv + 2];
                const float sy = R[kInv + 3] * nx + R[kInv + 4] * ny + R[kInv + 5];
#pragma unroll
                for (int c = 0; c < 3; ++c) v[c] = sample(src + c * plane, H, W, sx, sy, R[kBlur], c);
                if (slot >= 0 && donors != nullptr) {
                    const float dx = R[kPasteInv + 0] * nx + R[kPasteInv + 1] * ny + R[kPasteInv + 2];
                    const float dy = R[kPasteInv + 3] * nx + R[kPasteInv + 4] * ny + R[kPasteInv + 5];
                    bool paste = false;
                    if (pmode == 1) {
                        paste = mask_at(donor_masks ? donor_masks + int64_t(slot) * plane : nullptr, H, W, dx, dy);
                    } else if (pmode == 2) {
                        paste = dx >= R[kPasteBox + 0] && dx <= R[kPasteBox + 2] && dy >= R[kPasteBox + 1] &&
                                dy <= R[kPasteBox + 3];
                    }
                    if (paste) {
                        const In* dsrc = donors + int64_t(slot) * 3 * plane;
#pragma unroll
                        for (int c = 0; c < 3; ++c) v[c] = sample(dsrc + c * plane, H, W, dx, dy, R[kBlur], c);
                    }
                }
            } else {
#pragma unroll
                for (int c = 0; c < 3; ++c) v[c] = px(src + c * plane, int64_t(y) * W + x);
            }
#pragma unroll
            for (int c = 0; c < 3; ++c) c3[c][i] = v[c];
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int x = x0 + i;
        effects(c3[0][i], c3[1][i], c3[2][i], R, key, int64_t(y) * W + x, (float(x) + 0.5f) / float(W), ny);
    }
    if (full) {
#pragma unroll
        for (int c = 0; c < 3; ++c) store_row8(dst + c * plane + int64_t(y) * W + x0, c3[c]);
    } else {
        for (int i = 0; i < 8 && x0 + i < W; ++i)
#pragma unroll
            for (int c = 0; c < 3; ++c) dst[c * plane + int64_t(y) * W + x0 + i] = from_f<Out>(c3[c][i]);
    }
}

// rows: [N, 2] int32 = (image, source) with source >= 0 a row of `src`, <= -2 donor slot -(source + 2).
__global__ void __launch_bounds__(256) warp_masks_kernel(const uint8_t* __restrict__ src,
                                                         const uint8_t* __restrict__ donor_masks,
                                                         const int32_t* __restrict__ rows,
                                                         const float* __restrict__ rec, uint8_t* __restrict__ out,
                                                         int H, int W) {
    const int n = blockIdx.y;
    const int b = rows[2 * n], s = rows[2 * n + 1];
    const float* R = rec + int64_t(b) * kRecFloats;
    const int64_t plane = int64_t(H) * W;
    for (int64_t p = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; p < plane; p += int64_t(gridDim.x) * blockDim.x) {
        const int y = int(p / W), x = int(p % W);
        const float nx = (float(x) + 0.5f) / float(W), ny = (float(y) + 0.5f) / float(H);
        const int slot = int(R[kPasteSlot]);
        const float dx = R[kPasteInv + 0] * nx + R[kPasteInv + 1] * ny + R[kPasteInv + 2];
        const float dy = R[kPasteInv + 3] * nx + R[kPasteInv + 4] * ny + R[kPasteInv + 5];
        bool v;
        if (s >= 0) {
            const float sx = R[kInv + 0] * nx + R[kInv + 1] * ny + R[kInv + 2];
            const float sy = R[kInv + 3] * nx + R[kInv + 4] * ny + R[kInv + 5];
            v = mask_at(src + int64_t(s) * plane, H, W, sx, sy);
            if (v && slot >= 0) {  // hidden under the pasted object
                const int pmode = int(R[kPasteMode]);
                if (pmode == 1) v = !mask_at(donor_masks + int64_t(slot) * plane, H, W, dx, dy);
                else v = !(dx >= R[kPasteBox + 0] && dx <= R[kPasteBox + 2] && dy >= R[kPasteBox + 1] && dy <= R[kPasteBox + 3]);
            }
        } else {
            v = mask_at(donor_masks + int64_t(-(s + 2)) * plane, H, W, dx, dy);
        }
        out[int64_t(n) * plane + p] = v ? 1 : 0;
    }
}

}  // namespace

cudaError_t launch_augment(DType out_t, bool in_u8, const void* in, void* out, const float* rec, const void* donors,
                           const uint8_t* donor_masks, int B, int H, int W, cudaStream_t st) {
    if (B == 0) return cudaSuccess;
    const int64_t threads = int64_t((W + 7) / 8) * H;
    const dim3 grid(unsigned((threads + 255) / 256), unsigned(B));
#define MMLTK_AUG(IN, OUT)                                                                                    \
    augment_kernel<IN, OUT><<<grid, 256, 0, st>>>(static_cast<const IN*>(in), static_cast<OUT*>(out), rec, \
                                                  static_cast<const IN*>(donors), donor_masks, H, W)
    if (in_u8 && out_t == DType::kBF16) MMLTK_AUG(uint8_t, __nv_bfloat16);
    else if (in_u8) MMLTK_AUG(uint8_t, float);
    else if (out_t == DType::kBF16) MMLTK_AUG(float, __nv_bfloat16);
    else MMLTK_AUG(float, float);
#undef MMLTK_AUG
    return cudaGetLastError();
}

cudaError_t launch_warp_masks(const uint8_t* src, const uint8_t* donor_masks, const int32_t* rows, const float* rec,
                              uint8_t* out, int N, int H, int W, cudaStream_t st) {
    if (N == 0) return cudaSuccess;
    const int64_t plane = int64_t(H) * W;
    const dim3 grid(unsigned(std::min<int64_t>((plane + 255) / 256, 64)), unsigned(N));
    warp_masks_kernel<<<grid, 256, 0, st>>>(src, donor_masks, rows, rec, out, H, W);
    return cudaGetLastError();
}

}  // namespace mmltk
