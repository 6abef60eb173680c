#include "image_io.h"

#include <zlib.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <fstream>
#include <stdexcept>

namespace mmltk::img {

namespace {

uint32_t be32(const uint8_t* p) {
    return (uint32_t(p[0]) << 24) | (uint32_t(p[1]) << 16) | (uint32_t(p[2]) << 8) | uint32_t(p[3]);
}

void put_be32(std::vector<uint8_t>& v, uint32_t x) {
    v.push_back(uint8_t(x >> 24));
    v.push_back(uint8_t(x >> 16));
    v.push_back(uint8_t(x >> 8));
    v.push_back(uint8_t(x));
}

uint8_t paeth(int a, int b, int c) {
    const int p = a + b - c;
    const int pa = std::abs(p - a), pb = std::abs(p - b), pc = std::abs(p - c);
    if (pa <= pb && pa <= pc) return uint8_t(a);
    if (pb <= pc) return uint8_t(b);
    return uint8_t(c);
}

}  // namespace

Image decode_png(const uint8_t* d, size_t n) {
    static const uint8_t sig[8] = {137, 80, 78, 71, 13, 10, 26, 10};
    if (n < 8 || std::memcmp(d, sig, 8) != 0) throw std::runtime_error("not a PNG file");
    size_t pos = 8;
    uint32_t w = 0, h = 0;
    int depth = 0, ctype = -1, interlace = 0;
    std::vector<uint8_t> idat, palette;
    while (pos + 8 <= n) {
        const uint32_t len = be32(d + pos);
        const uint8_t* type = d + pos + 4;
        const uint8_t* body = d + pos + 8;
        if (pos + 12 + len > n) throw std::runtime_error("truncated PNG chunk");
        if (!std::memcmp(type, "IHDR", 4)) {
            w = be32(body);
            h = be32(body + 4);
            depth = body[8];
            ctype = body[9];
            interlace = body[12];
        } else if (!std::memcmp(type, "PLTE", 4)) {
            palette.assign(body, body + len);
        } else if (!std::memcmp(type, "IDAT", 4)) {
            idat.insert(idat.end(), body, body + len);
        } else if (!std::memcmp(type, "IEND", 4)) {
            break;
        }
        pos += 12 + len;
    }
    if (w == 0 || h == 0) throw std::runtime_error("PNG without IHDR");
    if (depth != 8) throw std::runtime_error("only 8-bit PNG images are supported");
    if (interlace != 0) throw std::runtime_error("interlaced PNG images are not supported");
    int ch = 0;
    switch (ctype) {
        case 0: ch = 1; break;
        case 2: ch = 3; break;
        case 3: ch = 1; break;
        case 4: ch = 2; break;
        case 6: ch = 4; break;
        default: throw std::runtime_error("unsupported PNG colour type");
    }
    const size_t stride = size_t(w) * ch;
    std::vector<uint8_t> raw((stride + 1) * h);
    uLongf raw_len = static_cast<uLongf>(raw.size());
    if (uncompress(raw.data(), &raw_len, idat.data(), static_cast<uLong>(idat.size())) != Z_OK ||
        raw_len != raw.size())
        throw std::runtime_error("corrupt PNG image data");
    std::vector<uint8_t> px(stride * h);
    for (uint32_t y = 0; y < h; ++y) {
        const uint8_t f = raw[y * (stride + 1)];
        const uint8_t* s = &raw[y * (stride + 1) + 1];
        uint8_t* o = &px[y * stride];
        const uint8_t* up = y ? &px[(y - 1) * stride] : nullptr;
        for (size_t i = 0; i < stride; ++i) {
            const int a = i >= size_t(ch) ? o[i - ch] : 0;
            const int b = up ? up[i] : 0;
            const int c = (up && i >= size_t(ch)) ? up[i - ch] : 0;
            int v = s[i];
            switch (f) {
                case 0: break;
                case 1: v += a; break;
                case 2: v += b; break;
                case 3: v += (a + b) / 2; break;
                case 4: v += paeth(a, b, c); break;
                default: throw std::runtime_error("bad PNG filter");
            }
            o[i] = uint8_t(v);
        }
    }
    Image im;
    im.width = int(w);
    im.height = int(h);
    im.rgb.resize(size_t(w) * h * 3);
    for (size_t p = 0; p < size_t(w) * h; ++p) {
        uint8_t r, g, b;
        if (ctype == 3) {
            const size_t k = size_t(px[p]) * 3;
            if (k + 2 >= palette.size()) throw std::runtime_error("bad PNG palette index");
            r = palette[k];
            g = palette[k + 1];
            b = palette[k + 2];
        } else if (ch <= 2) {
            r = g = b = px[p * ch];
        } else {
            r = px[p * ch];
            g = px[p * ch + 1];
            b = px[p * ch + 2];
        }
        im.rgb[3 * p] = r;
        im.rgb[3 * p + 1] = g;
        im.rgb[3 * p + 2] = b;
    }
    return im;
}

Image decode_png_file(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("cannot open image " + path);
    std::vector<uint8_t> buf((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    try {
        return decode_png(buf.data(), buf.size());
    } catch (const std::exception& e) {
        throw std::runtime_error(path + ": " + e.what());
    }
}

std::vector<uint8_t> encode_png(const uint8_t* pixels, int width, int height, int channels) {
    if (channels != 3 && channels != 4) throw std::runtime_error("encode_png: 3 or 4 channels");
    const size_t stride = size_t(width) * channels;
    std::vector<uint8_t> raw((stride + 1) * height);
    for (int y = 0; y < height; ++y) {
        raw[y * (stride + 1)] = 0;
        std::memcpy(&raw[y * (stride + 1) + 1], pixels + y * stride, stride);
    }
    uLongf zlen = compressBound(static_cast<uLong>(raw.size()));
    std::vector<uint8_t> z(zlen);
    if (compress2(z.data(), &zlen, raw.data(), static_cast<uLong>(raw.size()), 6) != Z_OK)
        throw std::runtime_error("encode_png: deflate failed");
    z.resize(zlen);
    std::vector<uint8_t> out = {137, 80, 78, 71, 13, 10, 26, 10};
    auto chunk = [&](const char* type, const uint8_t* data, size_t len) {
        put_be32(out, uint32_t(len));
        const size_t start = out.size();
        out.insert(out.end(), type, type + 4);
        out.insert(out.end(), data, data + len);
        const uint32_t crc = static_cast<uint32_t>(crc32(0, out.data() + start, static_cast<uInt>(len + 4)));
        put_be32(out, crc);
    };
    uint8_t ihdr[13];
    const uint32_t w = uint32_t(width), h = uint32_t(height);
    const uint8_t hdr[13] = {uint8_t(w >> 24), uint8_t(w >> 16), uint8_t(w >> 8), uint8_t(w),
                             uint8_t(h >> 24), uint8_t(h >> 16), uint8_t(h >> 8), uint8_t(h),
                             8, uint8_t(channels == 4 ? 6 : 2), 0, 0, 0};
    std::memcpy(ihdr, hdr, 13);
    chunk("IHDR", ihdr, 13);
    chunk("IDAT", z.data(), z.size());
    chunk("IEND", nullptr, 0);
    return out;
}

void resize_rgb_to_planar(const Image& src, int ow, int oh, float* out) {
    const int sw = src.width, sh = src.height;
    const size_t plane = size_t(ow) * oh;
    const float sx = float(sw) / ow, sy = float(sh) / oh;
    if (sw == ow && sh == oh) {
        for (size_t p = 0; p < plane; ++p)
            for (int c = 0; c < 3; ++c) out[c * plane + p] = src.rgb[3 * p + c] / 255.f;
        return;
    }
    if (sx >= 1.f && sy >= 1.f) {
        // area averaging: each output pixel is the coverage-weighted mean of its source footprint
        for (int y = 0; y < oh; ++y) {
            const float y0 = y * sy, y1 = (y + 1) * sy;
            for (int x = 0; x < ow; ++x) {
                const float x0 = x * sx, x1 = (x + 1) * sx;
                float acc[3] = {0, 0, 0}, wsum = 0.f;
                for (int yy = int(y0); yy < std::min(sh, int(std::ceil(y1))); ++yy) {
                    const float wy = std::min(y1, float(yy + 1)) - std::max(y0, float(yy));
                    if (wy <= 0) continue;
                    for (int xx = int(x0); xx < std::min(sw, int(std::ceil(x1))); ++xx) {
                        const float wx = std::min(x1, float(xx + 1)) - std::max(x0, float(xx));
                        if (wx <= 0) continue;
                        const float wgt = wx * wy;
                        const uint8_t* p = &src.rgb[3 * (size_t(yy) * sw + xx)];
                        acc[0] += wgt * p[0];
                        acc[1] += wgt * p[1];
                        acc[2] += wgt * p[2];
                        wsum += wgt;
                    }
                }
                for (int c = 0; c < 3; ++c) out[c * plane + size_t(y) * ow + x] = acc[c] / (wsum * 255.f);
            }
        }
        return;
    }
    // bilinear, pixel centres aligned (align_corners = false)
    for (int y = 0; y < oh; ++y) {
        const float fy = std::max(0.f, (y + 0.5f) * sy - 0.5f);
        const int y0 = std::min(int(fy), sh - 1), y1 = std::min(y0 + 1, sh - 1);
        const float ay = fy - y0;
        for (int x = 0; x < ow; ++x) {
            const float fx = std::max(0.f, (x + 0.5f) * sx - 0.5f);
            const int x0 = std::min(int(fx), sw - 1), x1 = std::min(x0 + 1, sw - 1);
            const float ax = fx - x0;
            for (int c = 0; c < 3; ++c) {
                auto at = [&](int yy, int xx) { return float(src.rgb[3 * (size_t(yy) * sw + xx) + c]); };
                const float v = (1 - ay) * ((1 - ax) * at(y0, x0) + ax * at(y0, x1)) +
                                ay * ((1 - ax) * at(y1, x0) + ax * at(y1, x1));
                out[c * plane + size_t(y) * ow + x] = v / 255.f;
            }
        }
    }
}

void resize_mask_nearest(const uint8_t* src, int sw, int sh, uint8_t* dst, int dw, int dh) {
    for (int y = 0; y < dh; ++y) {
        const int sy = std::min(sh - 1, int((y + 0.5f) * sh / dh));
        for (int x = 0; x < dw; ++x) {
            const int sx = std::min(sw - 1, int((x + 0.5f) * sw / dw));
            dst[size_t(y) * dw + x] = src[size_t(sy) * sw + sx];
        }
    }
}

}  // namespace mmltk::img
