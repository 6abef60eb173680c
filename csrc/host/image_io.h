// Minimal PNG codec (8-bit gray / gray+alpha / RGB / RGBA / palette, no
// interlace) on zlib, and CPU image resizing for the dataset compiler.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace mmltk::img {

struct Image {
    int width = 0, height = 0;
    std::vector<uint8_t> rgb;  // interleaved RGB, height * width * 3
};

// Throws std::runtime_error with a reason on unsupported / corrupt files.
Image decode_png_file(const std::string& path);
Image decode_png(const uint8_t* data, size_t size);
// 8-bit RGB (channels 3) or RGBA (4) -> PNG bytes.
std::vector<uint8_t> encode_png(const uint8_t* pixels, int width, int height, int channels);

// Area-averaging (downscale) / bilinear (upscale) resize of interleaved RGB
// into planar float32 [3, H, W] scaled to [0, 1].
void resize_rgb_to_planar(const Image& src, int out_w, int out_h, float* out);
// Nearest-neighbour resize of a binary mask (row-major, 0/1 bytes).
void resize_mask_nearest(const uint8_t* src, int sw, int sh, uint8_t* dst, int dw, int dh);

}  // namespace mmltk::img
