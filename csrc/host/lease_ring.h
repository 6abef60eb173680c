// Latest-frame lease ring for live pipelines (counterpart of the reference's
// lease rings in `src/live/*`): a fixed set of slots moves between a producer
// (capture) and a consumer (analysis) without copies.
//
//  * producer: acquire_write() -> a slot no one holds (the oldest published
//    frame that the consumer has not taken is recycled: live analysis wants the
//    newest frame, not every frame), then publish(slot, seq);
//  * consumer: acquire_latest(timeout) -> the newest published slot (older
//    published ones are dropped and counted), release(slot) when done.
// A slot is in exactly one state: free, writing, published or leased.
#pragma once

#include <condition_variable>
#include <cstdint>
#include <mutex>
#include <vector>

namespace mmltk::live {

class LeaseRing {
   public:
    explicit LeaseRing(int slots);
    // -1 if every slot is writing or leased
    int acquire_write();
    void publish(int slot, uint64_t seq);
    // -1 on timeout or after close(); seq of the frame in *seq
    int acquire_latest(double timeout_s, uint64_t* seq);
    void release(int slot);
    void close();
    uint64_t dropped() const;
    uint64_t published() const;
    int slots() const { return int(state_.size()); }

   private:
    enum State : uint8_t { kFree, kWriting, kPublished, kLeased };
    mutable std::mutex mu_;
    std::condition_variable cv_;
    std::vector<State> state_;
    std::vector<uint64_t> seq_;
    uint64_t dropped_ = 0, published_ = 0;
    bool closed_ = false;
};

}  // namespace mmltk::live
