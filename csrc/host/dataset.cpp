#include "dataset.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <random>
#include <stdexcept>

#include "image_io.h"
#include "exec_policy.h"
#include "worker_pool.h"

namespace mmltk::data {

namespace {

uint16_t f2bf(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    const uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;  // round to nearest even
    return static_cast<uint16_t>(u >> 16);
}

void pwrite_all(int fd, const void* buf, size_t n, off_t off) {
    const uint8_t* p = static_cast<const uint8_t*>(buf);
    while (n > 0) {
        const ssize_t w = ::pwrite(fd, p, n, off);
        if (w <= 0) throw std::runtime_error("dataset compiler: write failed");
        p += w;
        n -= size_t(w);
        off += w;
    }
}

struct ImageLabels {
    std::vector<PackedInstance> inst;
    std::vector<RLEPair> rle;
    uint64_t dropped = 0;
};

// Resize one image's instances to the target grid: boxes scaled (clamped),
// masks decoded on the source grid, resized nearest, re-encoded.
ImageLabels prepare_labels(const CompileInput& in, size_t img, int64_t first, int sw, int sh) {
    ImageLabels out;
    const int tw = in.width, th = in.height;
    const float sx = float(tw) / sw, sy = float(th) / sh;
    std::vector<uint8_t> src, dst(size_t(tw) * th);
    for (int k = 0; k < in.counts[img]; ++k) {
        const int64_t j = first + k;
        const float* b = &in.boxes[4 * j];
        PackedInstance p{};
        p.class_id = in.classes[j];
        p.x1 = int16_t(std::clamp(std::lround(b[0] * sx), 0L, long(tw)));
        p.y1 = int16_t(std::clamp(std::lround(b[1] * sy), 0L, long(th)));
        p.x2 = int16_t(std::clamp(std::lround(b[2] * sx), 0L, long(tw)));
        p.y2 = int16_t(std::clamp(std::lround(b[3] * sy), 0L, long(th)));
        p.rle_offset = 0;
        p.rle_pairs = 0;
        const int64_t nr = in.rle_count[j];
        if (nr > 0) {
            src.assign(size_t(sw) * sh, 0);
            const uint32_t* r = &in.rle[2 * in.rle_begin[j]];
            for (int64_t q = 0; q < nr; ++q) {
                const uint64_t s = r[2 * q], l = r[2 * q + 1];
                for (uint64_t t = s; t < std::min<uint64_t>(s + l, src.size()); ++t) src[t] = 1;
            }
            img::resize_mask_nearest(src.data(), sw, sh, dst.data(), tw, th);
            const uint32_t first_pair = uint32_t(out.rle.size());
            size_t t = 0, n = dst.size();
            int minx = tw, miny = th, maxx = -1, maxy = -1;
            while (t < n) {
                if (!dst[t]) {
                    ++t;
                    continue;
                }
                const size_t s = t;
                while (t < n && dst[t]) {
                    const int x = int(t % tw), y = int(t / tw);
                    minx = std::min(minx, x);
                    maxx = std::max(maxx, x);
                    miny = std::min(miny, y);
                    maxy = std::max(maxy, y);
                    ++t;
                }
                out.rle.push_back({uint32_t(s), uint32_t(t - s)});
            }
            if (maxx < 0) {  // the mask vanished at the target resolution
                out.rle.resize(first_pair);
                ++out.dropped;
                continue;
            }
            p.rle_offset = first_pair;
            p.rle_pairs = uint16_t(std::min<size_t>(out.rle.size() - first_pair, 65535));
        }
        if (p.x2 <= p.x1 || p.y2 <= p.y1) {
            ++out.dropped;
            if (p.rle_pairs) out.rle.resize(p.rle_offset);
            continue;
        }
        out.inst.push_back(p);
    }
    return out;
}

}  // namespace

CompileStats compile_dataset(const CompileInput& in, const std::string& out_path) {
    const size_t N = in.image_paths.size();
    if (in.counts.size() != N) throw std::runtime_error("compile: one count per image expected");
    if (in.class_names.size() > kMaxClasses) throw std::runtime_error("compile: at most 256 classes");
    std::vector<int64_t> first(N + 1, 0);
    for (size_t i = 0; i < N; ++i) first[i + 1] = first[i] + in.counts[i];
    WorkerPool pool(in.workers > 0 ? in.workers : std::max(1u, std::min(16u, std::thread::hardware_concurrency())));
    // phase 1: labels (needs each source image's size)
    std::vector<ImageLabels> labels(N);
    std::vector<std::string> errors(N);
    pool.parallel_for(int64_t(N), [&](int64_t i) {
        try {
            const img::Image im = img::decode_png_file(in.image_paths[i]);
            labels[i] = prepare_labels(in, size_t(i), first[i], im.width, im.height);
        } catch (const std::exception& e) {
            errors[i] = e.what();
        }
    });
    for (auto& e : errors)
        if (!e.empty()) throw std::runtime_error("dataset compiler: " + e);
    // layout
    FileHeader h{};
    h.magic = kMagic;
    h.version = kVersion;
    h.num_images = uint32_t(N);
    h.width = uint32_t(in.width);
    h.height = uint32_t(in.height);
    h.channels = 3;
    h.num_classes = uint32_t(in.class_names.size());
    for (size_t c = 0; c < in.class_names.size(); ++c) {
        std::memset(h.class_names[c].data(), 0, 32);
        std::memcpy(h.class_names[c].data(), in.class_names[c].data(), std::min<size_t>(31, in.class_names[c].size()));
    }
    h.image_stride = uint64_t(3) * in.width * in.height * sizeof(float);
    uint64_t n_inst = 0, n_rle = 0, dropped = 0;
    for (auto& l : labels) {
        n_inst += l.inst.size();
        n_rle += l.rle.size();
        dropped += l.dropped;
    }
    h.index_offset = sizeof(FileHeader);
    h.label_offset = h.index_offset + N * sizeof(ImageEntry);
    h.pixel_offset = align_up(h.label_offset + n_inst * sizeof(PackedInstance), kPage);
    h.rle_offset = h.pixel_offset + N * h.image_stride;
    h.total_size = h.rle_offset + n_rle * sizeof(RLEPair);
    std::vector<ImageEntry> index(N);
    std::vector<PackedInstance> all_inst;
    std::vector<RLEPair> all_rle;
    all_inst.reserve(n_inst);
    all_rle.reserve(n_rle);
    for (size_t i = 0; i < N; ++i) {
        ImageEntry& e = index[i];
        e.pixel_offset = h.pixel_offset + i * h.image_stride;
        e.label_offset = uint32_t(all_inst.size());
        e.num_instances = uint16_t(labels[i].inst.size());
        e.label_bytes = uint32_t(labels[i].inst.size() * sizeof(PackedInstance));
        const uint32_t rbase = uint32_t(all_rle.size());
        for (auto p : labels[i].inst) {
            if (p.rle_pairs) p.rle_offset += rbase;
            all_inst.push_back(p);
        }
        all_rle.insert(all_rle.end(), labels[i].rle.begin(), labels[i].rle.end());
    }
    const std::string tmp = out_path + ".tmp";
    const int fd = ::open(tmp.c_str(), O_CREAT | O_TRUNC | O_RDWR, 0644);
    if (fd < 0) throw std::runtime_error("dataset compiler: cannot create " + tmp);
    try {
        if (::ftruncate(fd, off_t(h.total_size)) != 0) throw std::runtime_error("dataset compiler: ftruncate failed");
        pwrite_all(fd, &h, sizeof(h), 0);
        pwrite_all(fd, index.data(), index.size() * sizeof(ImageEntry), off_t(h.index_offset));
        if (!all_inst.empty())
            pwrite_all(fd, all_inst.data(), all_inst.size() * sizeof(PackedInstance), off_t(h.label_offset));
        if (!all_rle.empty()) pwrite_all(fd, all_rle.data(), all_rle.size() * sizeof(RLEPair), off_t(h.rle_offset));
        // phase 2: pixels, decoded and resized in parallel, written at their offsets
        pool.parallel_for(int64_t(N), [&](int64_t i) {
            try {
                const img::Image im = img::decode_png_file(in.image_paths[i]);
                std::vector<float> px(size_t(3) * in.width * in.height);
                img::resize_rgb_to_planar(im, in.width, in.height, px.data());
                pwrite_all(fd, px.data(), px.size() * sizeof(float), off_t(index[i].pixel_offset));
            } catch (const std::exception& e) {
                errors[i] = e.what();
            }
        });
        for (auto& e : errors)
            if (!e.empty()) throw std::runtime_error("dataset compiler: " + e);
        ::fsync(fd);
        ::close(fd);
    } catch (...) {
        ::close(fd);
        ::unlink(tmp.c_str());
        throw;
    }
    if (::rename(tmp.c_str(), out_path.c_str()) != 0) throw std::runtime_error("dataset compiler: rename failed");
    CompileStats st;
    st.images = N;
    st.instances = n_inst;
    st.dropped_instances = dropped;
    st.rle_pairs = n_rle;
    st.bytes = h.total_size;
    return st;
}

// ---------------------------------------------------------------- reader
Reader::Reader(const std::string& path) {
    fd_ = ::open(path.c_str(), O_RDONLY);
    if (fd_ < 0) throw std::runtime_error("cannot open compiled dataset " + path);
    struct stat sb;
    if (::fstat(fd_, &sb) != 0) throw std::runtime_error("cannot stat " + path);
    size_ = size_t(sb.st_size);
    if (size_ < sizeof(FileHeader)) throw std::runtime_error(path + ": too small for a compiled dataset");
    void* m = ::mmap(nullptr, size_, PROT_READ, MAP_SHARED, fd_, 0);
    if (m == MAP_FAILED) throw std::runtime_error("mmap failed for " + path);
    base_ = static_cast<const uint8_t*>(m);
    hdr_ = reinterpret_cast<const FileHeader*>(base_);
    if (hdr_->magic != kMagic) throw std::runtime_error(path + ": bad magic (not a compiled dataset)");
    if (hdr_->version != kVersion) throw std::runtime_error(path + ": unsupported format version");
    if (hdr_->total_size > size_) throw std::runtime_error(path + ": truncated file");
    index_ = reinterpret_cast<const ImageEntry*>(base_ + hdr_->index_offset);
    labels_ = reinterpret_cast<const PackedInstance*>(base_ + hdr_->label_offset);
    rle_ = reinterpret_cast<const RLEPair*>(base_ + hdr_->rle_offset);
    n_rle_ = (hdr_->total_size - hdr_->rle_offset) / sizeof(RLEPair);
    n_labels_ = 0;
    for (uint32_t i = 0; i < hdr_->num_images; ++i) n_labels_ += index_[i].num_instances;
    ::madvise(m, size_, MADV_WILLNEED);
}

Reader::~Reader() {
    if (base_) ::munmap(const_cast<uint8_t*>(base_), size_);
    if (fd_ >= 0) ::close(fd_);
}

// ---------------------------------------------------------------- loader
Loader::Loader(const Config& cfg, std::vector<void*> slots, size_t slot_bytes)
    : cfg_(cfg), reader_(cfg.path), slots_(std::move(slots)), slot_bytes_(slot_bytes) {
    const size_t need = size_t(cfg_.batch) * reader_.header().image_stride / (cfg_.format == 1 ? 2 : cfg_.format == 2 ? 4 : 1);
    if (slot_bytes_ < need) throw std::runtime_error("loader: slot buffers are too small for one batch");
    if (slots_.empty()) throw std::runtime_error("loader: at least one slot buffer is needed");
    if (cfg_.shard_count < 1 || cfg_.shard_rank < 0 || cfg_.shard_rank >= cfg_.shard_count)
        throw std::runtime_error("loader: bad shard rank / count");
    slot_idx_.resize(slots_.size());
    thread_ = std::thread([this] { producer(); });
}

Loader::~Loader() {
    {
        std::lock_guard<std::mutex> lk(mu_);
        stop_ = true;
    }
    cv_.notify_all();
    thread_.join();
}

void Loader::begin_epoch(uint64_t epoch) {
    std::unique_lock<std::mutex> lk(mu_);
    const uint32_t n = reader_.num_images();
    std::vector<uint32_t> order(n);
    for (uint32_t i = 0; i < n; ++i) order[i] = i;
    if (cfg_.shuffle) {
        std::mt19937_64 rng(cfg_.seed * 1000003ull + epoch);
        for (uint32_t i = n; i > 1; --i) std::swap(order[i - 1], order[rng() % i]);
    }
    std::vector<std::vector<uint32_t>> all;
    for (uint32_t s = 0; s < n; s += uint32_t(cfg_.batch)) {
        const uint32_t e = std::min<uint32_t>(n, s + uint32_t(cfg_.batch));
        if (cfg_.drop_last && e - s < uint32_t(cfg_.batch)) break;
        all.emplace_back(order.begin() + s, order.begin() + e);
    }
    // every rank gets the same number of batches (lockstep DDP)
    const size_t per_rank = all.size() / size_t(cfg_.shard_count);
    batches_.clear();
    for (size_t b = 0; b < per_rank; ++b) batches_.push_back(all[b * cfg_.shard_count + cfg_.shard_rank]);
    if (cfg_.shard_count == 1) batches_ = all;
    // reset the pipeline
    free_.clear();
    ready_.clear();
    for (size_t s = 0; s < slots_.size(); ++s) free_.push_back(int(s));
    next_batch_ = 0;
    consumed_ = 0;
    ++generation_;
    lk.unlock();
    cv_.notify_all();
}

void Loader::fill(int slot, const std::vector<uint32_t>& idx) {
    const size_t stride = reader_.header().image_stride;
    const size_t floats = stride / sizeof(float);
    // images of one batch are gathered in parallel on the shared worker pool
    WorkerPool::global().parallel_for(int64_t(idx.size()), [&](int64_t k) {
        const float* src = reader_.pixels(idx[k]);
        if (cfg_.format == 1) {
            uint16_t* dst = static_cast<uint16_t*>(slots_[slot]) + k * floats;
            for (size_t i = 0; i < floats; ++i) dst[i] = f2bf(src[i]);
        } else if (cfg_.format == 2) {
            uint8_t* dst = static_cast<uint8_t*>(slots_[slot]) + k * floats;
            for (size_t i = 0; i < floats; ++i) dst[i] = uint8_t(std::lrintf(std::min(1.f, std::max(0.f, src[i])) * 255.f));
        } else {
            std::memcpy(static_cast<uint8_t*>(slots_[slot]) + k * stride, src, stride);
        }
    });
}

void Loader::producer() {
    if (!cfg_.cpus.empty()) set_thread_affinity(cfg_.cpus);
    while (true) {
        int slot = -1;
        std::vector<uint32_t> idx;
        uint64_t gen;
        {
            std::unique_lock<std::mutex> lk(mu_);
            cv_.wait(lk, [this] { return stop_ || (!free_.empty() && next_batch_ < batches_.size()); });
            if (stop_) return;
            slot = free_.front();
            free_.pop_front();
            idx = batches_[next_batch_++];
            gen = generation_;
        }
        fill(slot, idx);
        {
            std::lock_guard<std::mutex> lk(mu_);
            if (gen != generation_) continue;  // epoch restarted meanwhile: slot was reset
            slot_idx_[slot] = idx;
            ready_.push_back(slot);
        }
        cv_.notify_all();
    }
}

bool Loader::next(int& slot, std::vector<uint32_t>& indices) {
    std::unique_lock<std::mutex> lk(mu_);
    if (consumed_ >= batches_.size()) return false;
    cv_.wait(lk, [this] { return stop_ || !ready_.empty(); });
    if (stop_) return false;
    slot = ready_.front();
    ready_.pop_front();
    indices = slot_idx_[slot];
    ++consumed_;
    return true;
}

void Loader::release(int slot) {
    {
        std::lock_guard<std::mutex> lk(mu_);
        free_.push_back(slot);
    }
    cv_.notify_all();
}

}  // namespace mmltk::data
