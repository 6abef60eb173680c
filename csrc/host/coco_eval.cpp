#include "coco_eval.h"

#include <algorithm>
#include <stdexcept>

namespace mmltk::eval {

namespace {

constexpr uint16_t kAllBits = (1u << kThresholds) - 1;

// thresholds 0.50 + 0.05 t, as the float comparison IoU >= t uses
float threshold(int t) { return float(0.5 + 0.05 * t); }

uint16_t eligible(float iou) {
    uint16_t b = 0;
    for (int t = 0; t < kThresholds; ++t)
        if (iou >= threshold(t)) b |= uint16_t(1u << t);
    return b;
}

float box_iou(const float* a, const float* b) {
    const float iw = std::max(0.f, std::min(a[2], b[2]) - std::max(a[0], b[0]));
    const float ih = std::max(0.f, std::min(a[3], b[3]) - std::max(a[1], b[1]));
    const float inter = iw * ih;
    const float ua = std::max(0.f, a[2] - a[0]) * std::max(0.f, a[3] - a[1]) +
                     std::max(0.f, b[2] - b[0]) * std::max(0.f, b[3] - b[1]) - inter;
    return ua <= 0.f ? 0.f : inter / ua;
}

struct Cand {
    float iou;
    uint32_t gt;       // index within this image+category's ground truth
    uint32_t ordinal;  // annotation ordinal (tie break)
    uint16_t bits;
};

// greedy per-threshold matching of one image+category; preds sorted by score (desc)
template <typename IoU>
void match_group(const std::vector<uint32_t>& preds, const std::vector<uint32_t>& gt_ordinals, IoU&& iou,
                 const float* scores, uint32_t image, uint16_t cat, std::vector<Match>& out) {
    std::vector<uint16_t> open(gt_ordinals.size(), kAllBits);
    std::vector<Cand> cands;
    for (uint32_t p : preds) {
        cands.clear();
        for (uint32_t g = 0; g < gt_ordinals.size(); ++g) {
            const float v = iou(p, g);
            if (v >= threshold(0)) cands.push_back({v, g, gt_ordinals[g], eligible(v)});
        }
        std::sort(cands.begin(), cands.end(), [](const Cand& a, const Cand& b) {
            return a.iou > b.iou || (a.iou == b.iou && a.ordinal < b.ordinal);
        });
        uint16_t got = 0;
        for (const Cand& c : cands) {
            const uint16_t take = open[c.gt] & c.bits & uint16_t(~got);
            if (!take) continue;
            got |= take;
            open[c.gt] &= uint16_t(~take);
            if (got == kAllBits) break;
        }
        out.push_back({scores[p], image, p, cat, got});
    }
}

Metric reduce(std::vector<std::vector<Match>> by_cat, const std::vector<uint64_t>& gt_total) {
    Metric m;
    std::array<double, kThresholds> sums{};
    int cats = 0;
    std::vector<double> prec;
    for (size_t c = 0; c < by_cat.size(); ++c) {
        if (gt_total[c] == 0) continue;
        ++cats;
        auto& v = by_cat[c];
        std::sort(v.begin(), v.end(), [](const Match& a, const Match& b) {
            if (a.score != b.score) return a.score > b.score;
            if (a.image != b.image) return a.image < b.image;
            return a.ordinal < b.ordinal;
        });
        prec.resize(v.size());
        for (int t = 0; t < kThresholds; ++t) {
            std::array<size_t, 101> at;
            at.fill(v.size());
            size_t next = 0, tp = 0;
            for (size_t i = 0; i < v.size(); ++i) {
                tp += (v[i].bits >> t) & 1u;
                prec[i] = double(tp) / double(i + 1);
                const double recall = double(tp) / double(gt_total[c]);
                while (next < 101 && recall >= double(next) * 0.01) at[next++] = i;
            }
            for (size_t i = v.size(); i > 1; --i) prec[i - 2] = std::max(prec[i - 2], prec[i - 1]);
            double ap = 0;
            for (size_t i : at)
                if (i < v.size()) ap += prec[i];
            sums[t] += ap / 101.0;
        }
    }
    if (cats == 0) return m;
    double all = 0;
    for (int t = 0; t < kThresholds; ++t) {
        m.per_threshold[t] = sums[t] / cats;
        all += m.per_threshold[t];
    }
    m.ap = all / kThresholds;
    m.ap50 = m.per_threshold[0];
    m.ap75 = m.per_threshold[5];
    return m;
}

}  // namespace

std::vector<std::pair<uint32_t, uint32_t>> encode_runs(const uint8_t* m, size_t n, uint64_t* area) {
    std::vector<std::pair<uint32_t, uint32_t>> runs;
    uint64_t a = 0;
    size_t i = 0;
    while (i < n) {
        if (!m[i]) {
            ++i;
            continue;
        }
        size_t j = i;
        while (j < n && m[j]) ++j;
        runs.emplace_back(uint32_t(i), uint32_t(j - i));
        a += j - i;
        i = j;
    }
    if (area) *area = a;
    return runs;
}

uint64_t runs_intersection(const std::vector<std::pair<uint32_t, uint32_t>>& a, const data::RLEPair* b, size_t nb) {
    uint64_t inter = 0;
    size_t i = 0, j = 0;
    while (i < a.size() && j < nb) {
        const uint64_t a0 = a[i].first, a1 = a0 + a[i].second;
        const uint64_t b0 = b[j].start, b1 = b0 + b[j].length;
        const uint64_t lo = std::max(a0, b0), hi = std::min(a1, b1);
        if (hi > lo) inter += hi - lo;
        if (a1 < b1) ++i;
        else ++j;
    }
    return inter;
}

Evaluator::Evaluator(const data::Reader& reader, bool masks, int max_dets)
    : reader_(reader), masks_(masks), max_dets_(max_dets) {
    if (max_dets <= 0) throw std::invalid_argument("evaluator: max_dets must be positive");
    W_ = int(reader.header().width);
    H_ = int(reader.header().height);
    C_ = int(reader.header().num_classes);
    gt_total_.assign(size_t(C_), 0);
    for (uint32_t i = 0; i < reader.num_images(); ++i) {
        const auto* p = reader.instances(i);
        for (uint32_t k = 0; k < reader.entry(i).num_instances; ++k)
            if (p[k].class_id < C_) ++gt_total_[p[k].class_id];
    }
    box_by_cat_.resize(size_t(C_));
    if (masks_) mask_by_cat_.resize(size_t(C_));
}

void Evaluator::add_image(uint32_t image, const float* scores, const int64_t* labels, const float* boxes, int n,
                          const uint8_t* masks) {
    if (image >= reader_.num_images()) throw std::out_of_range("evaluator: image index");
    const auto& e = reader_.entry(image);
    const auto* gt = reader_.instances(image);
    // predictions per category (first max_dets valid ones), score-sorted
    std::vector<std::vector<uint32_t>> by_cat(static_cast<size_t>(C_));
    std::vector<std::array<float, 4>> pb(size_t(std::max(n, 0)));
    int kept = 0;
    for (int i = 0; i < n && kept < max_dets_; ++i) {
        const int64_t l = labels[i];
        if (l < 0 || l >= C_) continue;
        const float* b = boxes + 4 * i;
        pb[i] = {std::min(b[0], b[2]), std::min(b[1], b[3]), std::max(b[0], b[2]), std::max(b[1], b[3])};
        by_cat[size_t(l)].push_back(uint32_t(i));
        ++kept;
    }
    for (auto& v : by_cat)
        std::stable_sort(v.begin(), v.end(), [&](uint32_t a, uint32_t b) { return scores[a] > scores[b]; });
    std::vector<std::vector<uint32_t>> gt_by_cat(static_cast<size_t>(C_));
    for (uint32_t k = 0; k < e.num_instances; ++k)
        if (gt[k].class_id < C_) gt_by_cat[gt[k].class_id].push_back(k);

    std::vector<Match> box_out, mask_out;
    const size_t plane = size_t(W_) * H_;
    std::vector<std::vector<std::pair<uint32_t, uint32_t>>> pruns;
    std::vector<uint64_t> parea;
    if (masks_ && masks) {
        pruns.resize(size_t(n));
        parea.resize(size_t(n));
    }
    for (int c = 0; c < C_; ++c) {
        const auto& preds = by_cat[size_t(c)];
        if (preds.empty()) continue;
        const auto& gts = gt_by_cat[size_t(c)];
        std::vector<uint32_t> ord(gts.begin(), gts.end());
        std::vector<std::array<float, 4>> gb(gts.size());
        for (size_t g = 0; g < gts.size(); ++g) {
            const auto& q = gt[gts[g]];
            gb[g] = {float(q.x1), float(q.y1), float(q.x2), float(q.y2)};
        }
        match_group(preds, ord, [&](uint32_t p, uint32_t g) { return box_iou(pb[p].data(), gb[g].data()); }, scores,
                    image, uint16_t(c), box_out);
        if (masks_ && masks) {
            for (uint32_t p : preds)
                if (pruns[p].empty() && parea[p] == 0)
                    pruns[p] = encode_runs(masks + size_t(p) * plane, plane, &parea[p]);
            std::vector<uint64_t> garea(gts.size(), 0);
            for (size_t g = 0; g < gts.size(); ++g) {
                const auto& q = gt[gts[g]];
                for (int r = 0; r < q.rle_pairs; ++r) garea[g] += reader_.rle()[q.rle_offset + r].length;
            }
            match_group(preds, ord,
                        [&](uint32_t p, uint32_t g) {
                            const auto& q = gt[gts[g]];
                            const uint64_t inter = runs_intersection(pruns[p], reader_.rle() + q.rle_offset, q.rle_pairs);
                            const uint64_t uni = parea[p] + garea[g] - inter;
                            return uni == 0 ? 0.f : float(double(inter) / double(uni));
                        },
                        scores, image, uint16_t(c), mask_out);
        }
    }
    std::lock_guard<std::mutex> lk(mu_);
    for (const auto& m : box_out) box_by_cat_[m.category].push_back(m);
    for (const auto& m : mask_out) mask_by_cat_[m.category].push_back(m);
    ++images_seen_;
}

Metric Evaluator::summarize(bool mask) const {
    std::lock_guard<std::mutex> lk(mu_);
    if (mask && !masks_) throw std::logic_error("evaluator: built without masks");
    return reduce(mask ? mask_by_cat_ : box_by_cat_, gt_total_);
}

size_t Evaluator::num_matches(bool mask) const {
    std::lock_guard<std::mutex> lk(mu_);
    size_t n = 0;
    for (const auto& v : mask ? mask_by_cat_ : box_by_cat_) n += v.size();
    return n;
}

std::vector<double> Evaluator::export_matches(bool mask) const {
    std::lock_guard<std::mutex> lk(mu_);
    std::vector<double> out;
    for (const auto& v : mask ? mask_by_cat_ : box_by_cat_)
        for (const auto& m : v) {
            out.push_back(m.score);
            out.push_back(m.image);
            out.push_back(m.ordinal);
            out.push_back(m.category);
            out.push_back(m.bits);
        }
    return out;
}

void Evaluator::import_matches(bool mask, const double* rows, size_t n) {
    std::lock_guard<std::mutex> lk(mu_);
    auto& dst = mask ? mask_by_cat_ : box_by_cat_;
    if (mask && !masks_) throw std::logic_error("evaluator: built without masks");
    for (size_t i = 0; i < n; ++i) {
        const double* r = rows + 5 * i;
        const auto c = uint16_t(r[3]);
        if (c >= dst.size()) throw std::out_of_range("evaluator: imported category");
        dst[c].push_back({float(r[0]), uint32_t(r[1]), uint32_t(r[2]), c, uint16_t(r[4])});
    }
}

}  // namespace mmltk::eval
