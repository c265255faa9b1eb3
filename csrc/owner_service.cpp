#include "owner_service.h"
#include "trace.h"

#include <chrono>
#include <cstdio>
#include <stdexcept>
#include <thread>

#if defined(__x86_64__)
#include <immintrin.h>
#endif

namespace engram {

namespace {
inline void cpu_relax() {
#if defined(__x86_64__)
    _mm_pause();
#endif
}
} // namespace

void OwnerService::start(OwnerServiceConfig config, Launcher launcher, std::function<void()> thread_init) {
    if (thread_.joinable())
        throw std::runtime_error("owner service already started");
    if (config.headers == nullptr || config.serve.size() != config.world || config.layers == 0)
        throw std::runtime_error("owner service configuration");
    config_ = std::move(config);
    launcher_ = std::move(launcher);
    thread_init_ = std::move(thread_init);
    completed_.assign(size_t(config_.world) * config_.layers, 0);
    // Start from the epochs already published, so a service restarted on a live
    // mailbox does not replay old requests.
    for (uint32_t r = 0; r < config_.world; ++r)
        for (uint32_t l = 0; l < config_.layers; ++l)
            completed_[r * config_.layers + l] =
                __atomic_load_n(&config_.headers[size_t(r) * config_.layers + l].ready, __ATOMIC_ACQUIRE);
    stop_.store(false);
    thread_ = std::thread([this] { loop(); });
}

void OwnerService::fail(const std::string &what) {
    {
        std::lock_guard<std::mutex> lock(error_mutex_);
        if (error_.empty())
            error_ = what;
    }
    stop_.store(true);
    std::fprintf(stderr, "engram owner service (rank %u): %s\n", config_.rank, what.c_str());
}

void OwnerService::loop() {
    try {
        if (thread_init_)
            thread_init_();
    } catch (const std::exception &e) {
        fail(std::string("thread init: ") + e.what());
        return;
    }
    const auto &c = config_;
    std::vector<PushTask> batch;
    batch.reserve(size_t(c.world) * c.layers);
    auto last_work = std::chrono::steady_clock::now();
    try {
        while (!stop_.load(std::memory_order_relaxed)) {
            batch.clear();
            for (uint32_t r = 0; r < c.world; ++r) {
                if (!c.serve[r])
                    continue;
                for (uint32_t l = 0; l < c.layers; ++l) {
                    const MailboxHeader *h = c.headers + size_t(r) * c.layers + l;
                    const uint64_t epoch = __atomic_load_n(&h->ready, __ATOMIC_ACQUIRE);
                    uint64_t &done = completed_[size_t(r) * c.layers + l];
                    if (epoch == done)
                        continue;
                    // A jump forward is legal: the owner's hook kernels serve
                    // requests too, and a requester publishes a layer's next
                    // epoch only after every owner released the previous one,
                    // so the epochs in between are complete.  Going back is not.
                    if (epoch < done)
                        throw std::runtime_error("mailbox sequence went backwards: requester " + std::to_string(r) +
                                                 " layer " + std::to_string(l) + " epoch " + std::to_string(epoch) +
                                                 " after " + std::to_string(done));
                    if (epoch > done + 1)
                        skipped_.fetch_add(epoch - done - 1, std::memory_order_relaxed);
                    const uint32_t rows = __atomic_load_n(&h->rows, __ATOMIC_RELAXED);
                    const uint32_t layer = __atomic_load_n(&h->layer, __ATOMIC_RELAXED);
                    const uint32_t requester = __atomic_load_n(&h->requester, __ATOMIC_RELAXED);
                    if (rows == 0 || rows > c.capacity || layer != l || requester != r)
                        throw std::runtime_error("mailbox bounds: requester " + std::to_string(r) + " layer " +
                                                 std::to_string(l) + " rows " + std::to_string(rows));
                    PushTask t{};
                    t.requester = r;
                    t.layer = l;
                    t.rows = rows;
                    t.epoch = epoch;
                    t.channels = __atomic_load_n(&h->channels, __ATOMIC_RELAXED);
                    batch.push_back(t);
                    done = epoch;
                    rows_.fetch_add(rows, std::memory_order_relaxed);
                }
            }
            if (!batch.empty()) {
                requests_.fetch_add(batch.size(), std::memory_order_relaxed);
                batches_.fetch_add(1, std::memory_order_relaxed);
                const auto t0 = std::chrono::steady_clock::now();
                {
                    TraceRange trace("engram/owner_push");
                    launcher_(batch);
                }
                last_work = std::chrono::steady_clock::now();
                const uint64_t us = uint64_t(
                    std::chrono::duration_cast<std::chrono::microseconds>(last_work - t0).count());
                if (us > max_launch_us_.load(std::memory_order_relaxed))
                    max_launch_us_.store(us, std::memory_order_relaxed);
                continue;
            }
            const auto idle = std::chrono::steady_clock::now() - last_work;
            if (idle < std::chrono::microseconds(c.idle_spin_us)) {
                for (int i = 0; i < 64; ++i)
                    cpu_relax();
            } else {
                std::this_thread::sleep_for(std::chrono::microseconds(c.nap_us));
            }
        }
    } catch (const std::exception &e) {
        fail(e.what());
    }
}

void OwnerService::stop_and_join() noexcept {
    stop_.store(true);
    if (thread_.joinable())
        thread_.join();
}

void OwnerService::check() {
    std::lock_guard<std::mutex> lock(error_mutex_);
    if (!error_.empty())
        throw std::runtime_error("owner service failed: " + error_);
}

std::string OwnerService::error() {
    std::lock_guard<std::mutex> lock(error_mutex_);
    return error_;
}

uint64_t OwnerService::completed(uint32_t requester, uint32_t layer) const {
    if (requester >= config_.world || layer >= config_.layers || completed_.empty())
        return 0;
    return completed_[size_t(requester) * config_.layers + layer];
}

} // namespace engram
