// Request deduplication around the gather (sm_100a).
//
// Skewed request streams (e.g. Zipf over the vocabulary) ask for the same rows
// many times per fetch: with s = 1.1 over 4M rows and 98K requests per layer,
// only ~27% of the requests are distinct, and every duplicate pulls the same
// 256 bytes over NVLink from the same hot owner and the same L2 line there.
// This file removes the duplicates before the transfer:
//
//   dedup_kernel   inserts every direct-route request (layer, row) into an
//                  epoch-tagged open-addressing table and elects the smallest
//                  item of each key as its first occurrence;
//   (gather)       moves only first occurrences (GatherParams::dedup);
//   expand_kernel  copies each duplicate from its first occurrence's output
//                  row (local HBM), then, in its last CTA, advances the epoch
//                  and posts the unique/total counts to host-mapped memory.
//
// The table is never cleared: a key written in an older fetch carries an older
// epoch and reads as empty.  Lanes of a warp that hold the same key are merged
// with match.any first, so a hot key costs one probe per warp, not per lane.
// No reference counterpart: the reference moves every request.
#include "params.h"
#include "ptx.cuh"

namespace engram {

namespace {

constexpr int kDedupThreads = 256;
constexpr uint32_t kEpochMask = (1u << 28) - 1;

__device__ __forceinline__ uint32_t current_epoch(const uint32_t *state) {
    const uint32_t e = (state[0] + 1) & kEpochMask;
    return e == 0 ? 1 : e;
}

// MurmurHash3's 64-bit finaliser (Appleby) to spread keys over the table.
__device__ __forceinline__ uint32_t mix(uint64_t k) {
    k ^= k >> 33;
    k *= 0xff51afd7ed558ccdull;
    k ^= k >> 33;
    k *= 0xc4ceb9fe1a85ec53ull;
    k ^= k >> 33;
    return uint32_t(k);
}

__global__ void __launch_bounds__(kDedupThreads) dedup_kernel(const __grid_constant__ DedupParams p) {
    __shared__ uint32_t s_uniques, s_items;
    if (threadIdx.x == 0)
        s_uniques = s_items = 0;
    __syncthreads();
    const uint32_t epoch = current_epoch(p.state);
    const uint32_t lane = threadIdx.x % 32;
    const uint32_t total = p.layers * p.rows;
    const uint32_t stride = gridDim.x * blockDim.x;
    // Every lane of a warp runs the same number of iterations (warp-collective ops).
    const uint32_t first = blockIdx.x * blockDim.x + (threadIdx.x & ~31u);
    for (uint32_t base = first; base < total; base += stride) {
        const uint32_t item = base + lane;
        uint64_t key = 0;
        if (item < total) {
            const uint32_t layer = item / p.rows;
            const int32_t x = __ldg(p.indices + item);
            if (x >= 0) {
                const uint32_t owner = uint32_t(x) / p.layer.entries[layer];
                // Replicated hot rows are local reads: nothing to save.
                if (owner < p.world && p.direct_base[owner] != 0 && uint32_t(x) >= p.layer.hot_rows[layer])
                    key = (uint64_t(epoch) << 36) | (uint64_t(layer) << 31) | uint32_t(x);
            }
        }
        const uint32_t same = __match_any_sync(0xFFFFFFFFu, key);
        const uint32_t leader = __ffs(same) - 1;
        uint32_t slot = kDedupNone;
        bool inserted = false;
        if (key != 0 && lane == leader) {
            uint32_t h = mix(key) & p.table_mask;
            for (uint32_t probe = 0; probe <= p.table_mask; ++probe, h = (h + 1) & p.table_mask) {
                unsigned long long *k = reinterpret_cast<unsigned long long *>(p.keys + h);
                unsigned long long cur = *reinterpret_cast<volatile unsigned long long *>(k);
                if (cur == key) {
                    slot = h;
                    break;
                }
                if ((cur >> 36) == epoch)
                    continue;  // taken by another key of this fetch
                const unsigned long long old = atomicCAS(k, cur, key);
                if (old == cur) {
                    slot = h;
                    inserted = true;
                    break;
                }
                if (old == key) {
                    slot = h;
                    break;
                }
                if ((old >> 36) != epoch) {  // raced with a stale value; retry this slot
                    h = (h - 1) & p.table_mask;
                    continue;
                }
            }
            if (slot != kDedupNone) {
                // The leader holds the group's smallest item (items grow with the lane).
                unsigned long long *v = reinterpret_cast<unsigned long long *>(p.vals + slot);
                const unsigned long long mine = (uint64_t(epoch) << 32) | (0xFFFFFFFFu - item);
                const unsigned long long seen = *reinterpret_cast<volatile unsigned long long *>(v);
                if (seen < mine)
                    atomicMax(v, mine);
            }
        }
        slot = __shfl_sync(0xFFFFFFFFu, slot, leader);
        if (item < total)
            p.slots[item] = key != 0 ? slot : kDedupNone;
        const uint32_t news = __popc(__ballot_sync(0xFFFFFFFFu, inserted));
        const uint32_t counted = __popc(__ballot_sync(0xFFFFFFFFu, key != 0 && slot != kDedupNone));
        if (lane == 0 && (news | counted)) {
            atomicAdd(&s_uniques, news);
            atomicAdd(&s_items, counted);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && (s_uniques | s_items)) {
        atomicAdd(p.state + 1, s_uniques);
        atomicAdd(p.state + 2, s_items);
    }
}

__global__ void __launch_bounds__(kDedupThreads) expand_kernel(const __grid_constant__ DedupParams p) {
    __shared__ uint32_t s_last;
    const uint32_t epoch = current_epoch(p.state);
    constexpr uint32_t kLanesPerRow = 16;
    const uint32_t total = p.layers * p.rows;
    const uint32_t vectors = p.row_bytes / 16;
    const uint32_t sub = threadIdx.x / kLanesPerRow, vlane = threadIdx.x % kLanesPerRow;
    const uint32_t rows_per_step = kDedupThreads / kLanesPerRow;
    for (uint32_t item0 = blockIdx.x * rows_per_step; item0 < total; item0 += gridDim.x * rows_per_step) {
        const uint32_t item = item0 + sub;
        if (item >= total)
            continue;
        const uint32_t slot = p.slots[item];
        if (slot == kDedupNone)
            continue;
        const uint64_t v = p.vals[slot];
        const uint32_t leader = 0xFFFFFFFFu - uint32_t(v);
        if ((v >> 32) != epoch || leader == item || leader >= total)
            continue;
        const uint32_t layer = item / p.rows;
        const uint8_t *src = p.output + (uint64_t(layer) * p.capacity + (leader - layer * p.rows)) * p.row_bytes;
        uint8_t *dst = p.output + (uint64_t(layer) * p.capacity + (item - layer * p.rows)) * p.row_bytes;
        for (uint32_t c = vlane; c < vectors; c += kLanesPerRow)
            st_v4(dst + uint64_t(c) * 16, ld_v4(src + uint64_t(c) * 16));
    }
    // The last CTA closes the epoch: later fetches see this one's keys as stale.
    __syncthreads();
    if (threadIdx.x == 0) {
        s_last = atom_add_acq_rel_gpu(p.state + 3, 1u) == gridDim.x - 1;
        if (s_last) {
            const uint32_t uniques = p.state[1], items = p.state[2];
            p.state[0] = epoch;
            p.state[1] = 0;
            p.state[2] = 0;
            p.state[3] = 0;
            if (p.host_stats != nullptr) {
                st_relaxed_sys_u32(p.host_stats + 0, uniques);
                st_relaxed_sys_u32(p.host_stats + 1, items);
                st_release_sys_u32(p.host_stats + 2, epoch);
            }
        }
    }
}

} // namespace

cudaError_t launch_dedup(const DedupParams &p, int num_sms, cudaStream_t stream) {
    const uint32_t total = p.layers * p.rows;
    if (total == 0)
        return cudaSuccess;
    uint32_t blocks = (total + kDedupThreads - 1) / kDedupThreads;
    const uint32_t cap = uint32_t(num_sms) * 4;
    blocks = blocks < cap ? blocks : cap;
    dedup_kernel<<<blocks, kDedupThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_expand(const DedupParams &p, int num_sms, cudaStream_t stream) {
    const uint32_t total = p.layers * p.rows;
    if (total == 0)
        return cudaSuccess;
    const uint32_t rows_per_block = kDedupThreads / 16;
    uint32_t blocks = (total + rows_per_block - 1) / rows_per_block;
    const uint32_t cap = uint32_t(num_sms) * 4;
    blocks = blocks < cap ? blocks : cap;
    expand_kernel<<<blocks, kDedupThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

} // namespace engram
