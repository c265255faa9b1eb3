// engram_route_pack_noalloc: an allocation-free entry point to the per-owner
// request pack.
//
// This entry point has no counterpart in the reference; it exists for callers
// that cannot allocate GPU memory on their own: code running while a stream is
// being captured into a CUDA Graph (cudaMalloc is not allowed there), plugins
// that run inside a host framework which owns every device allocation through
// its own pool, and plain C callers that link this library without torch and
// its caching allocator.  The caller passes the indices and the two outputs;
// the kernel's scratch (per-(layer, owner) slot cursors and per-layer arrival
// counters, plus an unused epoch block the kernel signature needs) lives in a
// file-scope device array of fixed size, `kNoAllocScratchBytes` (32 KiB),
// which every GPU that loads this library keeps until the process exits.
//
// Limits: at most 32 layers and 64 owners (the array holds exactly that);
// larger requests are rejected with an error message and nothing runs.
//
// Set-up: the first call on a device (with that device current) looks up the
// device address of the array with cudaGetSymbolAddress and caches it; make
// that first call before any stream capture.  Host code never passes the
// array's host-side name to a kernel, only the looked-up device address.
//
// Sharing: every call on a device uses the same array and it keeps the last
// call's contents.  The entry point clears the cursors and counters on the
// caller's stream before the kernel, so calls ordered on one stream (or
// otherwise serialised) are correct; calls that overlap on the GPU, e.g. on
// two unsynchronised streams, race on the array and give wrong results.
//
// The entry point calls no allocating routine: no cudaMalloc, no cudaFree, no
// torch allocation; only cudaGetSymbolAddress (once per device),
// cudaMemsetAsync on the array, and the kernel launch.
#include "params.h"

#include <cstdio>
#include <cstring>
#include <mutex>

namespace {

constexpr size_t kNoAllocScratchBytes = 32 * 1024;
constexpr int kNoAllocMaxDevices = 64;

// cursors [32 x 64] u32 (8 KiB) | arrivals [32] u32 | epochs [32 x 64] u64 (16 KiB)
static __device__ __align__(256) unsigned char g_route_pack_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mutex;
void *g_scratch_address[kNoAllocMaxDevices] = {};

void set_message(char *err, size_t err_len, const char *text) {
    if (err != nullptr && err_len > 0) {
        std::strncpy(err, text, err_len - 1);
        err[err_len - 1] = '\0';
    }
}

// Looks up this device's scratch address once; returns nullptr on failure.
void *scratch_for_current_device(char *err, size_t err_len) {
    int device = -1;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kNoAllocMaxDevices) {
        set_message(err, err_len, "engram_route_pack_noalloc: no usable current CUDA device");
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (g_scratch_address[device] == nullptr) {
        void *ptr = nullptr;
        const cudaError_t rc = cudaGetSymbolAddress(&ptr, g_route_pack_scratch);
        if (rc != cudaSuccess || ptr == nullptr) {
            char text[256];
            std::snprintf(text, sizeof(text), "engram_route_pack_noalloc: cudaGetSymbolAddress failed: %s",
                          cudaGetErrorString(rc));
            set_message(err, err_len, text);
            return nullptr;
        }
        g_scratch_address[device] = ptr;
    }
    return g_scratch_address[device];
}

} // namespace

// Packs the non-padding requests of `indices` ([layers, tokens * ept] int32 on
// the current device) per owner, exactly as the route_pack op does:
//   packed[o][l][i] = (position << 32) | (table_base[l] + x % entries[l])
// for i < counts[l][o], where owner o = x / entries[l] and owners_host[o] != 0.
// `packed` is int64 [world][layers][capacity], `counts` int32 [layers][world];
// `entries_host` and `owners_host` are host arrays of length layers / world.
// Returns 0 on success; otherwise a nonzero code and a message in `err`.
extern "C" int engram_route_pack_noalloc(const int32_t *indices, uint32_t layers, uint32_t tokens, uint32_t ept,
                                         const uint32_t *entries_host, uint32_t world, const uint8_t *owners_host,
                                         int64_t *packed, uint32_t capacity, int32_t *counts, cudaStream_t stream,
                                         char *err, size_t err_len) {
    using namespace engram;
    if (layers == 0 || layers > uint32_t(kMaxLayers) || world == 0 || world > uint32_t(kMaxRanks)) {
        set_message(err, err_len,
                    "engram_route_pack_noalloc: layers must be in [1, 32] and world in [1, 64] "
                    "(the fixed scratch array holds no more)");
        return 1;
    }
    const uint64_t rows = uint64_t(tokens) * ept;
    if (rows > capacity || rows * layers >= (1ull << 32)) {
        set_message(err, err_len, "engram_route_pack_noalloc: tokens * ept exceeds capacity or 32-bit indexing");
        return 2;
    }
    if ((rows > 0 && indices == nullptr) || packed == nullptr || counts == nullptr || entries_host == nullptr ||
        owners_host == nullptr) {
        set_message(err, err_len, "engram_route_pack_noalloc: null pointer argument");
        return 3;
    }
    unsigned char *scratch = static_cast<unsigned char *>(scratch_for_current_device(err, err_len));
    if (scratch == nullptr)
        return 4;

    const size_t lw = size_t(kMaxLayers) * kMaxRanks;
    DispatchParams d{};
    d.cursors = reinterpret_cast<uint32_t *>(scratch);
    d.layer_arrivals = d.cursors + lw;
    d.epochs = reinterpret_cast<uint64_t *>(scratch + 16 * 1024);
    d.totals = reinterpret_cast<uint32_t *>(counts);
    d.error = ErrorSink{nullptr, nullptr};
    uint32_t at = 0;
    for (uint32_t l = 0; l < layers; ++l) {
        if (entries_host[l] == 0 || uint64_t(entries_host[l]) * world > 0x7FFFFFFFull) {
            set_message(err, err_len, "engram_route_pack_noalloc: entries must be positive and world*entries < 2^31");
            return 5;
        }
        d.layer.entries[l] = entries_host[l];
        d.layer.table_bases[l] = at;
        at += entries_host[l];
    }
    for (uint32_t o = 0; o < world; ++o)
        d.inbox_base[o] =
            owners_host[o] ? reinterpret_cast<uint64_t>(packed) + uint64_t(o) * layers * capacity * 8ull : 0;
    d.indices = indices;
    d.layers = layers;
    d.rows = uint32_t(rows);
    d.capacity = capacity;
    d.world = world;
    d.rank = 0;
    d.channels = 1;
    d.tile_rows = 4096;

    // The array keeps the previous call's state: the cursors and arrival
    // counters the kernel relies on must start at zero.
    cudaError_t rc = cudaMemsetAsync(scratch, 0, (lw + kMaxLayers) * sizeof(uint32_t), stream);
    if (rc == cudaSuccess && rows == 0)
        rc = cudaMemsetAsync(counts, 0, size_t(layers) * world * sizeof(int32_t), stream);
    if (rc == cudaSuccess && rows > 0)
        rc = launch_dispatch(d, stream);
    if (rc != cudaSuccess) {
        char text[256];
        std::snprintf(text, sizeof(text), "engram_route_pack_noalloc: %s", cudaGetErrorString(rc));
        set_message(err, err_len, text);
        return 6;
    }
    return 0;
}
