// Dataset compiler, memory-mapped reader and prefetching batch loader for the
// compiled ".bin" format (dataset_format.h).
//
// Counterparts of the reference's DatasetCompiler / DatasetLoader
// (`include/dataset_compiler.h:18-129`, `include/dataset_loader.h:10-78`,
// format spec `README.md:293-360`).  Their .cpp sources are not part of the
// reference snapshot; behaviour follows the headers and the README:
//  * compiler: images are decoded, resized to the target size and stored as
//    float32 planar RGB in [0, 1]; boxes are scaled; masks are resized
//    (nearest) and re-encoded as runs; instances left empty by the resize are
//    dropped and counted;
//  * loader: mmap, seeded per-epoch shuffle, batches sharded over ranks
//    (batch b goes to rank b % count, every rank gets the same number),
//    worker threads gather into caller-owned (pinned) slots ahead of use,
//    lease-style next / release.
#pragma once

#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <deque>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "dataset_format.h"

namespace mmltk::data {

struct CompileInput {
    std::vector<std::string> image_paths;
    std::vector<int32_t> counts;          // instances per image
    std::vector<uint8_t> classes;         // [total]
    std::vector<float> boxes;             // [total, 4] xyxy, source pixels
    std::vector<int64_t> rle_begin;       // [total] index into rle (pairs)
    std::vector<int64_t> rle_count;       // [total]
    std::vector<uint32_t> rle;            // [2 * pairs] (start, length) on the source grid
    std::vector<std::string> class_names;
    int width = 432, height = 432;
    int workers = 0;
};

struct CompileStats {
    uint64_t images = 0, instances = 0, dropped_instances = 0, rle_pairs = 0, bytes = 0;
};

CompileStats compile_dataset(const CompileInput& in, const std::string& out_path);

class Reader {
   public:
    explicit Reader(const std::string& path);
    ~Reader();
    Reader(const Reader&) = delete;
    Reader& operator=(const Reader&) = delete;

    const FileHeader& header() const { return *hdr_; }
    uint32_t num_images() const { return hdr_->num_images; }
    const ImageEntry& entry(uint32_t i) const { return index_[i]; }
    const float* pixels(uint32_t i) const {
        return reinterpret_cast<const float*>(base_ + index_[i].pixel_offset);
    }
    const PackedInstance* instances(uint32_t i) const { return labels_ + index_[i].label_offset; }
    const RLEPair* rle() const { return rle_; }
    uint64_t total_instances() const { return n_labels_; }
    uint64_t total_rle_pairs() const { return n_rle_; }

   private:
    int fd_ = -1;
    size_t size_ = 0;
    const uint8_t* base_ = nullptr;
    const FileHeader* hdr_ = nullptr;
    const ImageEntry* index_ = nullptr;
    const PackedInstance* labels_ = nullptr;
    const RLEPair* rle_ = nullptr;
    uint64_t n_labels_ = 0, n_rle_ = 0;
};

// Prefetching batch loader.  Slots are caller-owned host buffers (pinned by
// the caller) of `slot_bytes` each, filled with `batch` images as float32 or
// bf16 planar RGB, or as uint8 (round(255 x)): the compiled pixels are k/255,
// so uint8 is exact and moves a quarter of the fp32 bytes host -> device.
class Loader {
   public:
    struct Config {
        std::string path;
        int batch = 8;
        bool shuffle = true;
        uint64_t seed = 42;
        int shard_rank = 0, shard_count = 1;
        bool drop_last = false;
        int workers = 4;
        int format = 0;  // 0 fp32, 1 bf16, 2 uint8
        std::vector<int> cpus;   // CPUs of the producer thread (empty: not pinned)
    };
    Loader(const Config& cfg, std::vector<void*> slots, size_t slot_bytes);
    ~Loader();

    void begin_epoch(uint64_t epoch);
    // batches this rank yields per epoch (the same for every epoch and rank)
    size_t num_batches() const {
        const size_t n = reader_.num_images(), b = size_t(cfg_.batch);
        const size_t all = cfg_.drop_last ? n / b : (n + b - 1) / b;
        return cfg_.shard_count == 1 ? all : all / size_t(cfg_.shard_count);
    }
    // Blocks until the next batch is in a slot.  Returns false at epoch end.
    bool next(int& slot, std::vector<uint32_t>& indices);
    void release(int slot);
    Reader& reader() { return reader_; }
    const Config& config() const { return cfg_; }

   private:
    void producer();
    void fill(int slot, const std::vector<uint32_t>& idx);

    Config cfg_;
    Reader reader_;
    std::vector<void*> slots_;
    size_t slot_bytes_;
    std::vector<std::vector<uint32_t>> batches_;
    std::mutex mu_;
    std::condition_variable cv_;
    std::deque<int> free_, ready_;
    std::vector<std::vector<uint32_t>> slot_idx_;
    size_t next_batch_ = 0, consumed_ = 0;
    uint64_t generation_ = 0;
    bool stop_ = false;
    std::thread thread_;
};

}  // namespace mmltk::data
