// engram_route_pack_noalloc: an allocation-free entry point to the per-owner
// request pack.  The contract (what it computes, limits, set-up, sharing and
// the callers it is for) is declared in engram_noalloc.h; this file defines it
// against that declaration.
//
// It has no counterpart in the reference.  Its callers cannot allocate GPU
// memory themselves (CUDA Graph stream capture, plugins whose host framework
// owns all device memory, C callers without torch's allocator), so the
// dispatch kernel's scratch lives in a file-scope device array of
// ENGRAM_NOALLOC_SCRATCH_BYTES that every GPU loading the library keeps until
// exit.  Host code never hands the array's host-side name to a kernel: the
// first call on a device looks up its device address with
// cudaGetSymbolAddress (that device current) and caches it.
#include "engram_noalloc.h"
#include "params.h"

#include <cstdio>
#include <cstring>
#include <mutex>

namespace {

constexpr size_t kNoAllocScratchBytes = ENGRAM_NOALLOC_SCRATCH_BYTES;
static_assert(ENGRAM_NOALLOC_MAX_LAYERS == engram::kMaxLayers && ENGRAM_NOALLOC_MAX_OWNERS == engram::kMaxRanks,
              "header limits follow the kernel's tables");
constexpr int kNoAllocMaxDevices = 64;

// cursors [32 x 64] u32 (8 KiB) | arrivals [32] u32 | epochs [32 x 64] u64 (16 KiB, at 16 KiB)
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

extern "C" int engram_route_pack_noalloc(const int32_t *indices, uint32_t layers, uint32_t tokens, uint32_t ept,
                                         const uint32_t *entries_host, uint32_t world, const uint8_t *owners_host,
                                         int64_t *packed, uint32_t capacity, int32_t *counts, cudaStream_t stream,
                                         char *err, size_t err_len) {
    using namespace engram;
    if (layers == 0 || layers > uint32_t(kMaxLayers) || world == 0 || world > uint32_t(kMaxRanks)) {
        set_message(err, err_len,
                    "engram_route_pack_noalloc: layers must be in [1, 32] and world in [1, 64] "
                    "(the fixed scratch array holds no more)");
        return ENGRAM_NOALLOC_BAD_SHAPE;
    }
    const uint64_t rows = uint64_t(tokens) * ept;
    if (rows > capacity || rows * layers >= (1ull << 32)) {
        set_message(err, err_len, "engram_route_pack_noalloc: tokens * ept exceeds capacity or 32-bit indexing");
        return ENGRAM_NOALLOC_BAD_ROWS;
    }
    if ((rows > 0 && indices == nullptr) || packed == nullptr || counts == nullptr || entries_host == nullptr ||
        owners_host == nullptr) {
        set_message(err, err_len, "engram_route_pack_noalloc: null pointer argument");
        return ENGRAM_NOALLOC_NULL_ARG;
    }
    unsigned char *scratch = static_cast<unsigned char *>(scratch_for_current_device(err, err_len));
    if (scratch == nullptr)
        return ENGRAM_NOALLOC_NO_DEVICE;

    const size_t lw = size_t(kMaxLayers) * kMaxRanks;
    DispatchParams d{};
    d.cursors = reinterpret_cast<uint32_t *>(scratch);
    d.layer_arrivals = d.cursors + lw;
    d.epochs = reinterpret_cast<uint64_t *>(scratch + 16 * 1024);
    d.totals = reinterpret_cast<uint32_t *>(counts);
    d.error = ErrorSink{nullptr, nullptr};
    // Table bases are 32-bit in the packed entries: the running sum is kept in
    // 64 bits and rejected before it could wrap.
    uint64_t at = 0;
    for (uint32_t l = 0; l < layers; ++l) {
        if (entries_host[l] == 0 || uint64_t(entries_host[l]) * world > 0x7FFFFFFFull) {
            set_message(err, err_len, "engram_route_pack_noalloc: entries must be positive and world*entries < 2^31");
            return ENGRAM_NOALLOC_BAD_ENTRIES;
        }
        if (at + entries_host[l] > 0xFFFFFFFFull) {
            set_message(err, err_len, "engram_route_pack_noalloc: the sum of entries over layers exceeds 2^32 - 1");
            return ENGRAM_NOALLOC_BAD_ENTRIES;
        }
        d.layer.entries[l] = entries_host[l];
        d.layer.table_bases[l] = uint32_t(at);
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
        return ENGRAM_NOALLOC_CUDA_ERROR;
    }
    return 0;
}
