#include "worker_pool.h"

#include <pthread.h>
#include <sched.h>

#include <algorithm>
#include <sstream>

namespace mmltk {

namespace {
thread_local bool t_in_worker = false;
}

std::vector<int> parse_cpuset(const std::string& spec) {
    std::vector<int> out;
    std::stringstream ss(spec);
    std::string item;
    while (std::getline(ss, item, ',')) {
        if (item.empty()) continue;
        const auto dash = item.find('-');
        if (dash == std::string::npos) {
            out.push_back(std::stoi(item));
        } else {
            const int a = std::stoi(item.substr(0, dash));
            const int b = std::stoi(item.substr(dash + 1));
            if (b < a) throw std::invalid_argument("bad cpuset range: " + item);
            for (int c = a; c <= b; ++c) out.push_back(c);
        }
    }
    std::sort(out.begin(), out.end());
    out.erase(std::unique(out.begin(), out.end()), out.end());
    return out;
}

std::string format_cpuset(const std::vector<int>& cpus) {
    std::vector<int> c(cpus);
    std::sort(c.begin(), c.end());
    std::string out;
    for (size_t i = 0; i < c.size();) {
        size_t j = i;
        while (j + 1 < c.size() && c[j + 1] == c[j] + 1) ++j;
        if (!out.empty()) out += ",";
        out += std::to_string(c[i]);
        if (j > i) out += "-" + std::to_string(c[j]);
        i = j + 1;
    }
    return out;
}

bool pin_current_thread(int cpu) {
    cpu_set_t set;
    CPU_ZERO(&set);
    CPU_SET(cpu, &set);
    return pthread_setaffinity_np(pthread_self(), sizeof(set), &set) == 0;
}

WorkerPool::WorkerPool(int threads, std::vector<int> cpus) : cpus_(std::move(cpus)) {
    threads = std::max(1, threads);
    for (int i = 0; i < threads; ++i) workers_.emplace_back([this, i] { loop(i); });
}

WorkerPool::~WorkerPool() {
    {
        std::lock_guard<std::mutex> lk(mu_);
        stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
}

void WorkerPool::loop(int index) {
    t_in_worker = true;
    uint64_t pinned = 0;   // generation of cpus_ this thread is pinned to (0: never pinned)
    {
        std::lock_guard<std::mutex> lk(mu_);
        if (!cpus_.empty()) {
            pin_current_thread(cpus_[static_cast<size_t>(index) % cpus_.size()]);
            pinned = pin_gen_;
        }
    }
    while (true) {
        std::packaged_task<void()> task;
        {
            std::unique_lock<std::mutex> lk(mu_);
            cv_.wait(lk, [this] { return stop_ || !tasks_.empty(); });
            if (stop_ && tasks_.empty()) return;
            task = std::move(tasks_.front());
            tasks_.pop();
            if (pinned != pin_gen_ && !cpus_.empty()) {
                pin_current_thread(cpus_[static_cast<size_t>(index) % cpus_.size()]);
                pinned = pin_gen_;
            }
        }
        task();
    }
}

void WorkerPool::set_affinity(std::vector<int> cpus) {
    std::lock_guard<std::mutex> lk(mu_);
    cpus_ = std::move(cpus);
    ++pin_gen_;
}

std::future<void> WorkerPool::enqueue(std::function<void()> fn) {
    std::packaged_task<void()> task(std::move(fn));
    auto fut = task.get_future();
    {
        std::lock_guard<std::mutex> lk(mu_);
        tasks_.push(std::move(task));
    }
    cv_.notify_one();
    return fut;
}

void WorkerPool::parallel_for(int64_t n, const std::function<void(int64_t)>& fn) {
    if (n <= 0) return;
    if (t_in_worker || n == 1 || size() == 1) {
        for (int64_t i = 0; i < n; ++i) fn(i);
        return;
    }
    const int64_t chunks = std::min<int64_t>(n, size());
    std::atomic<int64_t> next{0};
    std::vector<std::future<void>> futs;
    futs.reserve(static_cast<size_t>(chunks));
    for (int64_t c = 0; c < chunks; ++c) {
        futs.push_back(enqueue([&] {
            for (int64_t i = next.fetch_add(1); i < n; i = next.fetch_add(1)) fn(i);
        }));
    }
    for (auto& f : futs) f.get();
}

namespace {
std::mutex g_pool_mu;
WorkerPool* g_pool = nullptr;   // created once, never destroyed (lives until process exit)
}  // namespace

WorkerPool& WorkerPool::global() {
    std::lock_guard<std::mutex> lk(g_pool_mu);
    if (g_pool == nullptr) g_pool = new WorkerPool(std::max(1u, std::min(16u, std::thread::hardware_concurrency())));
    return *g_pool;
}

int WorkerPool::configure_global(int threads, std::vector<int> cpus) {
    std::lock_guard<std::mutex> lk(g_pool_mu);
    if (g_pool == nullptr) {
        const int n = threads > 0 ? threads : static_cast<int>(std::max(1u, std::min(16u, std::thread::hardware_concurrency())));
        g_pool = new WorkerPool(n, std::move(cpus));
    } else if (!cpus.empty()) {
        g_pool->set_affinity(std::move(cpus));
    }
    return g_pool->size();
}

}  // namespace mmltk
