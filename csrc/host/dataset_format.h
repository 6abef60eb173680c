// Compiled dataset file format (".bin").
//
// The on-disk layout is the reference's format, byte for byte, so files
// compiled by either tool load in the other (`include/compiled_format.h:9-61`
// of the reference: FileHeader 8328 B, ImageEntry 24 B, PackedInstance 16 B,
// RLEPair 8 B, magic 0x464153544C445232, version 4, <= 256 classes):
//
//   [FileHeader][ImageEntry x num_images][PackedInstance x total]
//   [pad to 4 KiB][pixels: num_images x image_stride bytes][RLEPair x total]
//
// Pixels are float32, planar RGB, in [0, 1], image_stride = 3*W*H*4 bytes.
// Boxes are xyxy in target-image pixels; masks are row-major (start, length)
// runs over the W*H target grid.  The reference's compiler sources are not
// part of its snapshot, so the offsets are defined here as: ImageEntry.
// pixel_offset = absolute file offset of the image's pixels, label_offset =
// index of the image's first PackedInstance, label_bytes = 16 * num_instances,
// PackedInstance.mask_rle_offset = index of its first RLEPair.
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>

namespace mmltk::data {

constexpr uint64_t kMagic = 0x464153544C445232ULL;
constexpr uint32_t kVersion = 4;
constexpr uint32_t kMaxClasses = 256;
constexpr size_t kPage = 4096;

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) & ~(a - 1); }

#pragma pack(push, 1)
struct PackedInstance {
    uint8_t class_id;
    uint8_t pad;
    int16_t x1, y1, x2, y2;
    uint32_t rle_offset;
    uint16_t rle_pairs;
};
struct ImageEntry {
    uint64_t pixel_offset;
    uint32_t label_offset;
    uint16_t num_instances;
    uint16_t pad;
    uint32_t label_bytes;
    uint32_t reserved;
};
struct FileHeader {
    uint64_t magic;
    uint32_t version;
    uint32_t num_images;
    uint32_t width;
    uint32_t height;
    uint32_t channels;
    uint32_t num_classes;
    uint64_t index_offset;
    uint64_t label_offset;
    uint64_t pixel_offset;
    uint64_t rle_offset;
    uint64_t total_size;
    uint64_t image_stride;
    std::array<std::array<char, 32>, kMaxClasses> class_names;
    std::array<uint8_t, 56> reserved;
};
struct RLEPair {
    uint32_t start;
    uint32_t length;
};
#pragma pack(pop)

static_assert(sizeof(PackedInstance) == 16, "PackedInstance layout");
static_assert(sizeof(ImageEntry) == 24, "ImageEntry layout");
static_assert(sizeof(FileHeader) == 8328, "FileHeader layout");
static_assert(sizeof(RLEPair) == 8, "RLEPair layout");

}  // namespace mmltk::data
