// Host side of the fused training augmentation: per-image plans and the
// augmented detection targets.
//
// Behaviour follows the reference's GPU augmenter and target builder
// (`src/rfdetr/gpu_augment.cpp:29-133,213-544`, `src/rfdetr/cuda/gpu_augment_cuda.cu:181-309`,
// `src/rfdetr/target_builder.cpp:338-615`): the same augmentation groups,
// probabilities, strength ranges and effect formulas, the same box transform
// and drop rules and the same single-instance copy-paste with a rolling donor
// cache.  The design differs: every random draw of a batch is made HERE, once,
// into a fixed 64-float record per image which is the only thing the device
// kernel reads (the reference draws the same numbers twice, on the host for the
// targets and again in a device kernel for the pixels).  The device then needs
// only a per-pixel noise key.  Random numbers come from a 32-bit counter hash
// (the `lowbias32` integer finaliser) keyed by (seed, epoch, rank, sequence,
// image), so plans are reproducible across runs and ranks get distinct streams.
#pragma once

#include <array>
#include <cstdint>
#include <vector>

#include "dataset.h"

namespace mmltk::aug {

struct Group {
    float p = 0.5f, lo = 0.05f, hi = 0.5f;
};

struct Config {
    bool enabled = false;
    Group geometry, resize, color, noise, blur, occlusion;
    float copy_paste = 0.5f;
    bool valid() const;
};

// Layout of one image's record (floats).  The kernel (csrc/kernels/augment.cu)
// reads the same offsets.
enum Rec : int {
    kInv = 0,          // 6: output (normalised) -> source (normalised) affine
    kFwd = 6,          // 6: source -> output affine (boxes)
    kColor = 12,       // 9: 3x3 colour matrix (row = output channel)
    kColorOff = 21,    // 3
    kNoiseMode = 24,   // 0 none, 1 gaussian, 2 salt
    kNoiseStr = 25,
    kBlur = 26,        // lerp weight of the 2x2 box average over bilinear
    kOccMode = 27,     // 0 none, 1 channel fade, 2 pixel drop, 3 rectangle erase
    kOccStr = 28,
    kOccChan = 29,
    kErase = 30,       // 4: x0 y0 x1 y1 (normalised)
    kAreaScale = 34,
    kFlags = 35,       // bit 0: geometry is not the identity (remap path)
    kPasteSlot = 36,   // donor slot or -1
    kPasteMode = 37,   // 1 donor mask, 2 donor box
    kPasteInv = 38,    // 6: output -> donor source affine
    kNoiseKey = 44,    // uint32 bits of the per-image noise key
    kPasteBox = 45,    // 4: donor source box (normalised xyxy)
    kRecFloats = 64,
};

struct Donor {
    bool valid = false;
    int64_t label = -1;
    uint32_t dataset_index = 0;
    float area = 0.f;
    std::array<float, 4> box{};
};

// Output of build_targets (caller-owned buffers, sized by the caller):
//  boxes [B, T, 4] cxcywh (padding slots get (0.5,0.5,0.25,0.25)), labels [B, T],
//  counts [B], areas [B, T] (pixels of the output image), and for masks
//  src_rows [B, T] (row into the source-mask upload, -1 for a pasted instance).
struct TargetBuffers {
    float* boxes;
    int64_t* labels;
    int32_t* counts;
    float* areas;
    int32_t* src_rows;  // may be null (no masks)
};

class Planner {
   public:
    Planner(const Config& cfg, int capacity, int width, int height, bool masks);

    // Draws the plans of one batch into `records` ([n, kRecFloats]).
    void plan(const std::vector<uint32_t>& dataset_indices, uint64_t seed, int epoch, int rank, uint64_t sequence,
              float* records);

    // Augmented padded targets for the batch last planned (plan() must come
    // first; with augmentation disabled, plan() writes identity records).
    // Returns the number of instances whose source masks are needed, and fills
    // `mask_sources` with (dataset_index, instance) pairs in upload order.
    int64_t build_targets(const data::Reader& reader, int slots, const TargetBuffers& out,
                          std::vector<std::pair<uint32_t, uint32_t>>* mask_sources);

    // Donor-cache replacements selected by the last build_targets:
    // (slot == image position, source-mask row or -1).  The caller copies the
    // input image (and mask row) into the slot after the augmentation kernel.
    const std::vector<std::pair<int, int64_t>>& replacements() const { return replace_; }
    // Commits the replacements' metadata (call after queueing the copies).
    void commit_donors();

    int dropped() const { return dropped_; }
    const Config& config() const { return cfg_; }
    bool remaps() const;

   private:
    Config cfg_;
    int cap_, W_, H_;
    bool masks_;
    std::vector<Donor> donors_;
    struct Pending {
        uint32_t cache_key = 0;
        int64_t src_row = -1;
        Donor donor;
    };
    std::vector<Pending> pending_;
    std::vector<uint32_t> idx_;
    std::vector<std::array<float, kRecFloats>> rec_;
    std::vector<std::pair<int, int64_t>> replace_;
    int dropped_ = 0;
};

uint32_t hash32(uint32_t x);
float uniform(uint32_t key, uint32_t counter);
uint32_t image_key(uint64_t seed, int epoch, int rank, uint64_t sequence, uint32_t image);

}  // namespace mmltk::aug
