#include "augment.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <stdexcept>

namespace mmltk::aug {

namespace {

constexpr float kPi = 3.14159265358979323846f;
constexpr float kPad[4] = {0.5f, 0.5f, 0.25f, 0.25f};

bool group_ok(const Group& g) {
    return std::isfinite(g.p) && std::isfinite(g.lo) && std::isfinite(g.hi) && g.p >= 0.f && g.p <= 1.f &&
           g.lo >= 0.f && g.lo <= g.hi && g.hi <= 1.f;
}

// Sequential draws from one image's stream.
struct Stream {
    uint32_t key, n = 0;
    float next() { return uniform(key, n++); }
    float strength(const Group& g) { return g.lo + (g.hi - g.lo) * next(); }
};

std::array<float, 4> transform_box(const std::array<float, 4>& b, const float* f) {
    float x0 = 1.f, y0 = 1.f, x1 = 0.f, y1 = 0.f;
    for (int c = 0; c < 4; ++c) {
        const float x = (c & 1) ? b[2] : b[0], y = (c & 2) ? b[3] : b[1];
        const float tx = f[0] * x + f[1] * y + f[2], ty = f[3] * x + f[4] * y + f[5];
        x0 = std::min(x0, tx);
        y0 = std::min(y0, ty);
        x1 = std::max(x1, tx);
        y1 = std::max(y1, ty);
    }
    auto c01 = [](float v) { return std::clamp(v, 0.f, 1.f); };
    return {c01(x0), c01(y0), c01(x1), c01(y1)};
}

float area(const std::array<float, 4>& b) { return std::max(0.f, b[2] - b[0]) * std::max(0.f, b[3] - b[1]); }

float overlap(const std::array<float, 4>& a, const std::array<float, 4>& b) {
    return std::max(0.f, std::min(a[2], b[2]) - std::max(a[0], b[0])) *
           std::max(0.f, std::min(a[3], b[3]) - std::max(a[1], b[1]));
}

void identity(std::array<float, kRecFloats>& r) {
    r.fill(0.f);
    r[kInv + 0] = r[kInv + 4] = 1.f;
    r[kFwd + 0] = r[kFwd + 4] = 1.f;
    r[kColor + 0] = r[kColor + 4] = r[kColor + 8] = 1.f;
    r[kAreaScale] = 1.f;
    r[kPasteSlot] = -1.f;
    r[kPasteInv + 0] = r[kPasteInv + 4] = 1.f;
}

}  // namespace

// lowbias32 (C. Wellons, "hash-prospector", public domain): a 32-bit integer
// finaliser with low avalanche bias, cheap on both CPU and GPU (no 64-bit
// multiplies).  The device copy lives in csrc/kernels/augment.cu.
uint32_t hash32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352dU;
    x ^= x >> 15;
    x *= 0x846ca68bU;
    x ^= x >> 16;
    return x;
}

float uniform(uint32_t key, uint32_t counter) {
    return float(hash32(key ^ hash32(counter + 0x68e31da4U)) >> 8) * (1.0f / 16777216.0f);
}

uint32_t image_key(uint64_t seed, int epoch, int rank, uint64_t sequence, uint32_t image) {
    uint32_t k = hash32(uint32_t(seed) ^ 0x1b873593U);
    k = hash32(k ^ uint32_t(seed >> 32));
    k = hash32(k ^ uint32_t(epoch));
    k = hash32(k ^ (uint32_t(rank) * 0x9e3779b9U));
    k = hash32(k ^ uint32_t(sequence));
    k = hash32(k ^ uint32_t(sequence >> 32));
    return hash32(k ^ image);
}

bool Config::valid() const {
    return group_ok(geometry) && group_ok(resize) && group_ok(color) && group_ok(noise) && group_ok(blur) &&
           group_ok(occlusion) && std::isfinite(copy_paste) && copy_paste >= 0.f && copy_paste <= 1.f;
}

Planner::Planner(const Config& cfg, int capacity, int width, int height, bool masks)
    : cfg_(cfg), cap_(capacity), W_(width), H_(height), masks_(masks) {
    if (!cfg_.valid()) throw std::invalid_argument("augmentation: probabilities and strengths must lie in [0, 1]");
    if (capacity <= 0 || width <= 0 || height <= 0) throw std::invalid_argument("augmentation: bad shape");
    donors_.resize(size_t(cap_));
    pending_.resize(size_t(cap_));
    rec_.resize(size_t(cap_));
}

bool Planner::remaps() const {
    return cfg_.enabled && ((cfg_.geometry.p > 0 && cfg_.geometry.hi > 0) || (cfg_.resize.p > 0 && cfg_.resize.hi > 0) ||
                            (cfg_.blur.p > 0 && cfg_.blur.hi > 0) || cfg_.copy_paste > 0);
}

void Planner::plan(const std::vector<uint32_t>& idx, uint64_t seed, int epoch, int rank, uint64_t sequence,
                   float* records) {
    if (int(idx.size()) > cap_) throw std::invalid_argument("augmentation: batch exceeds the planner capacity");
    idx_ = idx;
    for (size_t b = 0; b < idx.size(); ++b) {
        auto& r = rec_[b];
        identity(r);
        pending_[b] = Pending{};
        const uint32_t key = image_key(seed, epoch, rank, sequence, uint32_t(b));
        std::memcpy(&r[kNoiseKey], &key, 4);
        Stream s{key};
        pending_[b].cache_key = hash32(key ^ 0xC0FFEEu);
        if (cfg_.enabled) {
            // geometry: flips, small rotation (scaled to stay inside the frame), then zoom with an offset
            const bool fx = s.next() < cfg_.geometry.p * 0.5f;
            const bool fy = s.next() < cfg_.geometry.p * 0.5f;
            float angle = 0.f;
            if (s.next() < cfg_.geometry.p * 0.35f) {
                const float st = s.strength(cfg_.geometry);
                angle = (2.f * s.next() - 1.f) * (10.f * kPi / 180.f) * st;
            }
            const float c = std::cos(angle), sn = std::sin(angle);
            const float k = 1.f / (std::fabs(c) + std::fabs(sn));
            const float sx = fx ? -1.f : 1.f, sy = fy ? -1.f : 1.f;
            float f[6] = {k * c * sx, -k * sn * sy, 0.f, k * sn * sx, k * c * sy, 0.f};
            f[2] = 0.5f - 0.5f * (f[0] + f[1]);
            f[5] = 0.5f - 0.5f * (f[3] + f[4]);
            if (s.next() < cfg_.resize.p) {
                const float st = s.strength(cfg_.resize);
                const float scale = 1.f + (s.next() < 0.5f ? -0.5f : 0.5f) * st;
                const float dir = scale < 1.f ? 1.f : -1.f, ext = std::fabs(1.f - scale);
                const float ox = s.next() * ext * dir, oy = s.next() * ext * dir;
                for (int i : {0, 1, 3, 4}) f[i] *= scale;
                f[2] = scale * f[2] + ox;
                f[5] = scale * f[5] + oy;
            }
            const float det = f[0] * f[4] - f[1] * f[3], id = 1.f / det;
            const float i00 = f[4] * id, i01 = -f[1] * id, i10 = -f[3] * id, i11 = f[0] * id;
            const float inv[6] = {i00, i01, -(i00 * f[2] + i01 * f[5]), i10, i11, -(i10 * f[2] + i11 * f[5])};
            std::copy(f, f + 6, &r[kFwd]);
            std::copy(inv, inv + 6, &r[kInv]);
            r[kAreaScale] = std::fabs(det);
            const bool ident = f[0] == 1.f && f[1] == 0.f && f[2] == 0.f && f[3] == 0.f && f[4] == 1.f && f[5] == 0.f;
            r[kFlags] = ident ? 0.f : 1.f;

            if (s.next() < cfg_.color.p) {
                const float st = s.strength(cfg_.color);
                const float bright = (2.f * s.next() - 1.f) * 0.15f * st;
                const float contrast = 1.f + (2.f * s.next() - 1.f) * 0.30f * st;
                float sat = 1.f + (2.f * s.next() - 1.f) * 0.30f * st;
                if (s.next() < 0.10f * st) sat = 0.f;  // greyscale
                const float luma[3] = {0.299f, 0.587f, 0.114f};
                for (int o = 0; o < 3; ++o) {
                    for (int i = 0; i < 3; ++i) r[kColor + 3 * o + i] = contrast * ((o == i ? sat : 0.f) + (1.f - sat) * luma[i]);
                    r[kColorOff + o] = 0.5f * (1.f - contrast) + bright;
                }
            }
            if (s.next() < cfg_.noise.p) {
                r[kNoiseMode] = s.next() < 0.5f ? 1.f : 2.f;
                r[kNoiseStr] = s.strength(cfg_.noise);
            }
            if (s.next() < cfg_.blur.p) r[kBlur] = s.strength(cfg_.blur);
            if (s.next() < cfg_.occlusion.p) {
                const float st = s.strength(cfg_.occlusion);
                const int mode = std::min(2, int(s.next() * 3.f)) + 1;
                r[kOccMode] = float(mode);
                r[kOccStr] = st;
                r[kOccChan] = float(std::min(2, int(s.next() * 3.f)));
                if (mode == 3) {
                    const float a = 0.15f * st, aspect = 0.5f + 1.5f * s.next();
                    const float w = std::min(1.f, std::sqrt(a * aspect));
                    const float h = std::min(1.f, a / std::max(w, 1e-6f));
                    const float x0 = s.next() * (1.f - w), y0 = s.next() * (1.f - h);
                    r[kErase + 0] = x0;
                    r[kErase + 1] = y0;
                    r[kErase + 2] = x0 + w;
                    r[kErase + 3] = y0 + h;
                }
            }
            if (r[kBlur] > 0.f) r[kFlags] = 1.f;  // the blur lives in the resampler
            // single-instance copy-paste from the donor cache
            if (cfg_.copy_paste > 0.f && uniform(key, 0xCA57u) < cfg_.copy_paste) {
                const int start = std::min(cap_ - 1, int(uniform(key, 0xCA58u) * float(cap_)));
                int slot = -1;
                for (int q = 0; q < cap_; ++q) {
                    const int cnd = (start + q) % cap_;
                    if (donors_[cnd].valid && donors_[cnd].dataset_index != idx[b]) {
                        slot = cnd;
                        break;
                    }
                }
                if (slot >= 0) {
                    const Donor& d = donors_[slot];
                    const float scale = 0.5f + uniform(key, 0xCA59u);
                    const float dx = uniform(key, 0xCA5Au), dy = uniform(key, 0xCA5Bu);
                    const float tx = dx - scale * 0.5f * (d.box[0] + d.box[2]);
                    const float ty = dy - scale * 0.5f * (d.box[1] + d.box[3]);
                    auto c01 = [](float v) { return std::clamp(v, 0.f, 1.f); };
                    const float ox0 = c01(scale * d.box[0] + tx), oy0 = c01(scale * d.box[1] + ty);
                    const float ox1 = c01(scale * d.box[2] + tx), oy1 = c01(scale * d.box[3] + ty);
                    if (ox1 > ox0 && oy1 > oy0) {
                        const float is = 1.f / scale;
                        r[kPasteSlot] = float(slot);
                        r[kPasteMode] = masks_ ? 1.f : 2.f;
                        const float pinv[6] = {is, 0.f, -tx * is, 0.f, is, -ty * is};
                        std::copy(pinv, pinv + 6, &r[kPasteInv]);
                        std::copy(d.box.begin(), d.box.end(), &r[kPasteBox]);
                        r[kFlags] = 1.f;
                    }
                }
            }
        }
        std::copy(r.begin(), r.end(), records + b * kRecFloats);
    }
}

int64_t Planner::build_targets(const data::Reader& reader, int T, const TargetBuffers& out,
                               std::vector<std::pair<uint32_t, uint32_t>>* mask_sources) {
    const int B = int(idx_.size());
    const float W = float(reader.header().width), H = float(reader.header().height);
    if (int(W) != W_ || int(H) != H_) throw std::invalid_argument("augmentation: dataset size differs from the planner's");
    dropped_ = 0;
    replace_.clear();
    if (mask_sources) mask_sources->clear();
    for (int64_t k = 0; k < int64_t(B) * T; ++k) {
        std::copy(kPad, kPad + 4, out.boxes + 4 * k);
        out.labels[k] = 0;
        out.areas[k] = 0.f;
        if (out.src_rows) out.src_rows[k] = -1;
    }
    for (int b = 0; b < B; ++b) {
        const auto& r = rec_[b];
        const float* fwd = &r[kFwd];
        const int slot = int(r[kPasteSlot]);
        std::array<float, 4> paste_box{};
        float scale = 1.f;
        if (slot >= 0) {
            scale = 1.f / r[kPasteInv];
            const float tx = -r[kPasteInv + 2] * scale, ty = -r[kPasteInv + 5] * scale;
            const auto& d = donors_[slot].box;
            auto c01 = [](float v) { return std::clamp(v, 0.f, 1.f); };
            paste_box = {c01(scale * d[0] + tx), c01(scale * d[1] + ty), c01(scale * d[2] + tx), c01(scale * d[3] + ty)};
        }
        const auto& e = reader.entry(idx_[b]);
        const auto* inst = reader.instances(idx_[b]);
        const int room = T - (slot >= 0 ? 1 : 0);
        int n = 0, retained = 0;
        for (uint32_t k = 0; k < e.num_instances; ++k) {
            const auto& p = inst[k];
            const std::array<float, 4> src{p.x1 / W, p.y1 / H, p.x2 / W, p.y2 / H};
            const auto tb = transform_box(src, fwd);
            const float ta = area(tb);
            const float occ = slot >= 0 ? overlap(tb, paste_box) : 0.f;
            if (ta <= 0.f || occ >= ta || n >= room) {
                ++dropped_;
                continue;
            }
            const int64_t o = int64_t(b) * T + n;
            out.boxes[4 * o + 0] = 0.5f * (tb[0] + tb[2]);
            out.boxes[4 * o + 1] = 0.5f * (tb[1] + tb[3]);
            out.boxes[4 * o + 2] = tb[2] - tb[0];
            out.boxes[4 * o + 3] = tb[3] - tb[1];
            out.labels[o] = p.class_id;
            float src_area = float(p.x2 - p.x1) * float(p.y2 - p.y1);
            int64_t row = -1;
            if (masks_) {
                if (p.rle_pairs) {
                    double a = 0;
                    for (int q = 0; q < p.rle_pairs; ++q) a += reader.rle()[p.rle_offset + q].length;
                    src_area = float(a);
                }
                row = mask_sources ? int64_t(mask_sources->size()) : -1;
                if (mask_sources) mask_sources->emplace_back(idx_[b], k);
                if (out.src_rows) out.src_rows[o] = int32_t(row);
            }
            out.areas[o] = src_area * r[kAreaScale] * std::max(0.f, 1.f - occ / ta);
            // donor reservoir: every retained instance is equally likely to become the donor
            ++retained;
            if (uniform(pending_[b].cache_key, uint32_t(retained)) * float(retained) < 1.f) {
                pending_[b].src_row = row;
                pending_[b].donor = Donor{true, int64_t(p.class_id), idx_[b], src_area, src};
            }
            ++n;
        }
        if (slot >= 0) {
            const Donor& d = donors_[slot];
            const int64_t o = int64_t(b) * T + n;
            out.boxes[4 * o + 0] = 0.5f * (paste_box[0] + paste_box[2]);
            out.boxes[4 * o + 1] = 0.5f * (paste_box[1] + paste_box[3]);
            out.boxes[4 * o + 2] = paste_box[2] - paste_box[0];
            out.boxes[4 * o + 3] = paste_box[3] - paste_box[1];
            out.labels[o] = d.label;
            const float clip = std::min(1.f, area(paste_box) / (std::max(area(d.box), 1e-12f) * scale * scale));
            out.areas[o] = d.area * scale * scale * clip;
            if (out.src_rows) out.src_rows[o] = -(slot + 2);
            ++n;
        }
        out.counts[b] = n;
        if (cfg_.enabled && cfg_.copy_paste > 0.f && pending_[b].donor.valid) replace_.emplace_back(b, pending_[b].src_row);
    }
    return mask_sources ? int64_t(mask_sources->size()) : 0;
}

void Planner::commit_donors() {
    for (const auto& [b, row] : replace_) donors_[b] = pending_[b].donor;
    replace_.clear();
}

}  // namespace mmltk::aug
