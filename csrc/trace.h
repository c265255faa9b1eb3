// NVTX ranges around host submission steps: fetch issue, hook wait, write,
// owner-service launches.  NVTX 3 is header-only: with no profiler attached a
// range costs one call through a no-op pointer.  Off unless enabled
// (ENGRAM_NVTX=1 at set_config, or set_nvtx()).
#pragma once

#include <nvtx3/nvToolsExt.h>

#include <atomic>

namespace engram {

inline std::atomic<bool> &nvtx_enabled() {
    static std::atomic<bool> on{false};
    return on;
}

class TraceRange {
  public:
    explicit TraceRange(const char *name) : on_(nvtx_enabled().load(std::memory_order_relaxed)) {
        if (on_)
            nvtxRangePushA(name);
    }
    ~TraceRange() {
        if (on_)
            nvtxRangePop();
    }
    TraceRange(const TraceRange &) = delete;
    TraceRange &operator=(const TraceRange &) = delete;

  private:
    bool on_;
};

} // namespace engram
