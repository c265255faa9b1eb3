// Owner service: the host-route trigger.
//
// Parity: `OwnerServices` (sge_write/csrc/owner_service.hpp:15-111).  One
// thread per owner (not per requester): it polls every [requester][layer]
// mailbox header in this rank's host shard with acquire loads, checks the
// epoch sequence and bounds, and hands each sweep's new requests as one batch
// to a launcher, which enqueues a single push kernel on the owner's stream.
// The GPU then moves the rows and publishes the done flags itself, so the
// thread never waits for data.  The first error is latched and stops the
// service; the runtime re-raises it on the next fetch or hook.
#pragma once

#include "kernels/params.h"

#include <atomic>
#include <cstdint>
#include <functional>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace engram {

struct OwnerServiceConfig {
    uint32_t world = 0, layers = 0, capacity = 0, rank = 0;
    const MailboxHeader *headers = nullptr;  // [world][layers] in this rank's host shard
    std::vector<uint8_t> serve;              // serve[r] != 0: requester r uses the host route to me
    uint32_t idle_spin_us = 20000;           // busy-poll this long after the last request, then nap
    uint32_t nap_us = 50;
};

class OwnerService {
  public:
    using Launcher = std::function<void(const std::vector<PushTask> &)>;

    OwnerService() = default;
    ~OwnerService() { stop_and_join(); }
    OwnerService(const OwnerService &) = delete;
    OwnerService &operator=(const OwnerService &) = delete;

    void start(OwnerServiceConfig config, Launcher launcher, std::function<void()> thread_init = {});
    void stop_and_join() noexcept;
    // Throws the latched error, if any.
    void check();
    bool running() const { return thread_.joinable() && !stop_.load(); }
    std::string error();
    uint64_t requests() const { return requests_.load(); }
    uint64_t rows() const { return rows_.load(); }
    uint64_t batches() const { return batches_.load(); }
    // Epochs the owner's hook kernels finished before this thread saw them.
    uint64_t skipped() const { return skipped_.load(); }
    // Longest time one launcher call took (host side), in microseconds.
    uint64_t max_launch_us() const { return max_launch_us_.load(); }
    // Epoch this service last accepted from (requester, layer).
    uint64_t completed(uint32_t requester, uint32_t layer) const;

  private:
    void loop();
    void fail(const std::string &what);

    OwnerServiceConfig config_;
    Launcher launcher_;
    std::function<void()> thread_init_;
    std::vector<uint64_t> completed_;
    std::atomic<bool> stop_{false};
    std::atomic<uint64_t> requests_{0}, rows_{0}, batches_{0}, max_launch_us_{0}, skipped_{0};
    std::mutex error_mutex_;
    std::string error_;
    std::thread thread_;
};

} // namespace engram
