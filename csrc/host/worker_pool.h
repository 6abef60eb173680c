// Fixed-size worker pool with optional CPU pinning and a blocking
// parallel_for (counterpart of the reference's `WorkerPool`,
// `include/worker_pool.h:17-94`): nested parallel_for calls from a worker run
// inline instead of deadlocking.
#pragma once

#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <functional>
#include <future>
#include <mutex>
#include <queue>
#include <string>
#include <thread>
#include <vector>

namespace mmltk {

std::vector<int> parse_cpuset(const std::string& spec);   // "0-3,8,10-11"
std::string format_cpuset(const std::vector<int>& cpus);
bool pin_current_thread(int cpu);

class WorkerPool {
   public:
    explicit WorkerPool(int threads, std::vector<int> cpus = {});
    ~WorkerPool();
    WorkerPool(const WorkerPool&) = delete;
    WorkerPool& operator=(const WorkerPool&) = delete;

    int size() const { return static_cast<int>(workers_.size()); }
    std::future<void> enqueue(std::function<void()> fn);
    // Runs fn(i) for i in [0, n); blocks until done.  Called from inside a
    // worker it runs inline.
    void parallel_for(int64_t n, const std::function<void(int64_t)>& fn);

    // Re-pins the workers (each before its next task): worker i -> cpus[i % size].
    void set_affinity(std::vector<int> cpus);

    // The process-wide pool (the loader's gather threads, the batch LSAP, the evaluator).
    static WorkerPool& global();
    // Size and CPUs of the global pool: the size applies only if the pool does not exist
    // yet, the CPUs always.  Returns the pool's size.
    static int configure_global(int threads, std::vector<int> cpus);

   private:
    void loop(int index);
    std::vector<std::thread> workers_;
    std::vector<int> cpus_;
    uint64_t pin_gen_ = 0;
    std::queue<std::packaged_task<void()>> tasks_;
    std::mutex mu_;
    std::condition_variable cv_;
    bool stop_ = false;
};

}  // namespace mmltk
