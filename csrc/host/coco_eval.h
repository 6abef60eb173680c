// COCO-style detection / instance-segmentation evaluator over a compiled
// dataset's ground truth.
//
// Metric definition (reference `src/rfdetr/inference/evaluator.cpp:260-460,1438-1490`,
// `include/mmltk/rfdetr/evaluation.h`): IoU thresholds 0.50:0.05:0.95; per
// image, each category's predictions are matched greedily in descending score
// order, each taking -- independently for every threshold -- the unmatched
// ground truth with the highest IoU at or above that threshold (ties: lower
// annotation ordinal); per category, all images' matches sorted by score give
// the precision envelope, sampled at 101 recall points (r = 0, 0.01, ..., 1;
// the first prediction reaching recall r); AP = mean over thresholds of the
// mean over categories that have ground truth; AP50 / AP75 the 0.50 / 0.75
// columns.  No area ranges, no crowd regions.  At most `max_dets` predictions
// per image are kept, in the order given (the post-processor's score order).
//
// Design: per-image matching is independent and is what costs; `add_image`
// can be called from several threads (it only takes a lock to append the
// compact match records), and the records can be exported / imported so that
// ranks evaluate disjoint image shards and one reduction sees them all.
#pragma once

#include <array>
#include <cstdint>
#include <mutex>
#include <vector>

#include "dataset.h"

namespace mmltk::eval {

constexpr int kThresholds = 10;

struct Match {
    float score;
    uint32_t image;       // dataset index
    uint32_t ordinal;     // prediction position within its image
    uint16_t category;
    uint16_t bits;        // bit t: matched at threshold t
};

struct Metric {
    double ap = 0, ap50 = 0, ap75 = 0;
    std::array<double, kThresholds> per_threshold{};
};

class Evaluator {
   public:
    Evaluator(const data::Reader& reader, bool masks, int max_dets);

    // scores [n], labels [n] (category index == compiled class id), boxes [n, 4]
    // xyxy pixels of the compiled image; masks: [n, H, W] binary (or null).
    void add_image(uint32_t image, const float* scores, const int64_t* labels, const float* boxes, int n,
                   const uint8_t* masks);

    Metric summarize(bool mask) const;
    size_t num_images() const { return images_seen_; }
    size_t num_matches(bool mask) const;

    // Compact records, for cross-rank reduction: [n, 5] doubles
    // (score, image, ordinal, category, bits).
    std::vector<double> export_matches(bool mask) const;
    void import_matches(bool mask, const double* rows, size_t n);

   private:
    const data::Reader& reader_;
    bool masks_;
    int max_dets_;
    int W_, H_, C_;
    std::vector<uint64_t> gt_total_;  // per category
    mutable std::mutex mu_;
    std::vector<std::vector<Match>> box_by_cat_, mask_by_cat_;
    size_t images_seen_ = 0;
};

// run-length helpers (row-major, (start, length) runs)
std::vector<std::pair<uint32_t, uint32_t>> encode_runs(const uint8_t* mask, size_t pixels, uint64_t* area);
uint64_t runs_intersection(const std::vector<std::pair<uint32_t, uint32_t>>& a, const data::RLEPair* b, size_t nb);

}  // namespace mmltk::eval
