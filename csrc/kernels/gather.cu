// Requester-side gather (sm_100a): the hot kernel of every fetch.
//
// Parity: the reference's direct-read paths, `engram_fetch.cuh:70-101` (READ,
// EGM rows) + `:223-269` (scale warps) and `gpu_request.cu:214-270`
// (`issue_egm`, WRITE).  Differences by design:
//   * the source of a direct row is the owner's HBM mirror reached through
//     NVLink 5 / NVSwitch, this rank's own shard, or this rank's replica of
//     the hot id prefix; never host memory of another rank;
//   * two variants, picked per buffer (ENGRAM_GATHER_KERNEL=auto|simt|bulk):
//       - SIMT (the default, "auto" and "simt"): each warp owns an equal
//         contiguous range of rows; one lane resolves each row and LPR lanes
//         move it with 32-byte (or 16-byte) vector loads and stores, UNROLL
//         rows in flight per lane.  Rows from a peer's HBM mirror are plain
//         per-thread loads through the NVLink mapping;
//       - TMA ring (only with ENGRAM_GATHER_KERNEL=bulk): one `cp.async.bulk`
//         (global -> shared, completing on an mbarrier) per row into an
//         8-stage shared ring; a consumer warp streams finished stages to the
//         final positions; two scale warps copy each tile's FP8 scales using
//         the indices the producer left in the stage.  For rows on the
//         peer-HBM route its bulk copies read the peer's memory, which the
//         project's north star rules out for the default path, so it is an
//         opt-in for comparison;
//   * indices may sit in pinned host memory: both variants stage them ahead
//     with cp.async, so the PCIe latency overlaps the row copies;
//   * route tables, layer geometry and strides are kernel parameters
//     (__grid_constant__), so CUDA Graph replays carry them;
//   * an out-of-range index is recorded in the error record and zero-filled,
//     and every barrier wait is bounded; nothing traps.
// The bulk copies are plain (non-multicast) loads; multicast never appears here.
#include <type_traits>

#include "params.h"
#include "ptx.cuh"

namespace engram {

namespace {

constexpr int kSimtThreads = 512;
constexpr int kBulkTile = 32;           // rows per stage: one producer lane per row
constexpr int kBulkThreads = 128;       // producer warp, consumer warp, 2 scale warps
constexpr uint32_t kStageTargetBytes = 64 * 1024;
constexpr uint64_t kPipelineTimeoutNs = 2000000000ull;
constexpr uint32_t kIndexDepth = 8;     // tiles of indices in flight per producer
constexpr uint32_t kIndexAhead = 4;     // SIMT: steps of indices in flight per warp

struct StageMeta {
    uint32_t layer, start, count, direct_mask, zero_mask, pad[3];
};

__device__ __forceinline__ void load_tables(const GatherParams &p, uint64_t *s_direct, uint64_t *s_sf,
                                            uint32_t *s_entries, uint32_t *s_tbase, uint32_t *s_sfbase,
                                            uint32_t *s_hot, uint32_t *s_hotbase) {
    for (uint32_t i = threadIdx.x; i < p.world; i += blockDim.x) {
        s_direct[i] = p.direct_base[i];
        s_sf[i] = p.sf_base[i];
    }
    for (uint32_t i = threadIdx.x; i < p.layers; i += blockDim.x) {
        s_entries[i] = p.layer.entries[i];
        s_tbase[i] = p.layer.table_bases[i];
        s_sfbase[i] = p.layer.sf_bases[i];
        s_hot[i] = p.layer.hot_rows[i];
        s_hotbase[i] = p.layer.hot_bases[i];
    }
}

// ------------------------------------------------------------- TMA variant
__global__ void __launch_bounds__(kBulkThreads) gather_bulk_kernel(const __grid_constant__ GatherParams p,
                                                                   uint32_t tiles_per_layer, uint32_t tiles_per_cta,
                                                                   uint32_t stages) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t s_direct[kMaxRanks], s_sf[kMaxRanks];
    __shared__ uint32_t s_entries[kMaxLayers], s_tbase[kMaxLayers], s_sfbase[kMaxLayers];
    __shared__ uint32_t s_hot[kMaxLayers], s_hotbase[kMaxLayers];
    __shared__ int32_t s_index[kIndexDepth * kBulkTile];
    const uint32_t stage_bytes = kBulkTile * p.row_bytes;
    uint8_t *data = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + size_t(stages) * stage_bytes);
    uint64_t *empty = full + stages;
    StageMeta *meta = reinterpret_cast<StageMeta *>(empty + stages);
    int32_t *stage_x = reinterpret_cast<int32_t *>(meta + stages);  // each stage's indices, for the scale warps

    load_tables(p, s_direct, s_sf, s_entries, s_tbase, s_sfbase, s_hot, s_hotbase);
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < stages; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, p.packs > 0 ? 2 : 1);  // consumer (+ the tile's scale warp)
        }
        fence_mbar_init();
    }
    __syncthreads();

    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t total_tiles = p.layers * tiles_per_layer;
    const uint32_t t0 = blockIdx.x * tiles_per_cta;
    const uint32_t t1 = min(t0 + tiles_per_cta, total_tiles);

    const uint32_t epoch = p.dedup ? dedup_epoch(p.dedup_state) : 0;
    if (warp == 0) {
        // Producer: classify the tile's rows and issue one bulk copy per direct
        // row.  Indices arrive through a kIndexDepth-tile cp.async ring, so
        // address generation never waits on a dependent global load.
        auto index_of = [&](uint32_t t, uint32_t &layer, uint32_t &start, uint32_t &count) {
            layer = t / tiles_per_layer;
            start = (t - layer * tiles_per_layer) * kBulkTile;
            count = min(uint32_t(kBulkTile), p.rows - start);
        };
        auto prefetch = [&](uint32_t t, uint32_t slot) {
            if (t < t1) {
                uint32_t l, st, c;
                index_of(t, l, st, c);
                if (lane < c)
                    cp_async_4(s_index + slot * kBulkTile + lane, p.indices + l * p.rows + st + lane);
            }
            cp_async_commit();  // one group per tile, empty past the end
        };
#pragma unroll
        for (uint32_t d = 0; d < kIndexDepth; ++d)
            prefetch(t0 + d, d);
        for (uint32_t t = t0, k = 0; t < t1; ++t, ++k) {
            const uint32_t stage = k % stages, phase = k / stages;
            const uint32_t slot = k % kIndexDepth;
            uint32_t layer, start, count;
            index_of(t, layer, start, count);
            cp_async_wait<kIndexDepth - 1>();  // tile k's indices have landed
            const int32_t x = lane < count ? s_index[slot * kBulkTile + lane] : -1;
            prefetch(t + kIndexDepth, slot);
            if (k >= stages && !mbar_wait(empty + stage, (phase - 1) & 1, kPipelineTimeoutNs)) {
                if (lane == 0)
                    report_error(p.error, kPipelineTimeout, layer, 0, t, 0);
                break;
            }
            const uint8_t *src = nullptr;
            bool zero = false;
            if (lane < count) {
                if (x < 0) {
                    zero = true;
                } else {
                    const uint32_t n = s_entries[layer];
                    const uint32_t owner = uint32_t(x) / n;
                    if (owner >= p.world) {
                        zero = true;
                        report_error(p.error, kIndexOutOfRange, layer, owner, uint64_t(x), 0);
                    } else if (uint32_t(x) < s_hot[layer]) {
                        src = reinterpret_cast<const uint8_t *>(p.hot_base) +
                              (uint64_t(s_hotbase[layer]) + uint32_t(x)) * p.row_bytes;
                    } else if (s_direct[owner] != 0 &&
                               !(p.dedup && dedup_duplicate(p, layer * p.rows + start + lane, epoch))) {
                        const uint64_t row = uint64_t(s_tbase[layer]) + (uint32_t(x) - owner * n);
                        src = reinterpret_cast<const uint8_t *>(s_direct[owner]) + row * p.row_bytes;
                    }
                }
            }
            const uint32_t direct_mask = __ballot_sync(0xFFFFFFFFu, src != nullptr);
            const uint32_t zero_mask = __ballot_sync(0xFFFFFFFFu, zero);
            stage_x[stage * kBulkTile + lane] = x;
            __syncwarp();  // the lanes' index stores precede lane 0's releasing arrive
            if (lane == 0) {
                meta[stage] = StageMeta{layer, start, count, direct_mask, zero_mask, {0, 0, 0}};
                mbar_arrive_expect_tx(full + stage, __popc(direct_mask) * p.row_bytes);
            }
            __syncwarp();
            if (src != nullptr)
                bulk_load(data + size_t(stage) * stage_bytes + size_t(lane) * p.row_bytes, src, p.row_bytes,
                          full + stage);
        }
        cp_async_wait<0>();
    } else if (warp == 1) {
        // Consumer: stream each finished stage to the output.
        const uint32_t vectors = p.row_bytes / 16;
        const uint32_t lpr = vectors < 32 ? vectors : 32;
        const uint32_t rps = 32 / lpr;
        const uint32_t sub = lane / lpr, vl = lane % lpr;
        for (uint32_t t = t0, k = 0; t < t1; ++t, ++k) {
            const uint32_t stage = k % stages, phase = k / stages;
            if (!mbar_wait(full + stage, phase & 1, kPipelineTimeoutNs)) {
                if (lane == 0)
                    report_error(p.error, kPipelineTimeout, 0, 1, t, 0);
                break;
            }
            const StageMeta m = meta[stage];
            const uint32_t live = m.direct_mask | m.zero_mask;
            uint8_t *dst = p.output + (uint64_t(m.layer) * p.capacity + m.start) * p.row_bytes;
            const uint8_t *src = data + size_t(stage) * stage_bytes;
            if (sub < rps) {
                for (uint32_t v = vl; v < vectors; v += lpr) {
                    for (uint32_t r0 = sub; r0 < m.count; r0 += rps * 4) {
                        Vec16 val[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const uint32_t r = r0 + u * rps;
                            val[u] = Vec16{0, 0, 0, 0};
                            if (r < m.count && ((m.direct_mask >> r) & 1u))
                                val[u] = ld_shared_v4(src + size_t(r) * p.row_bytes + v * 16);
                        }
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const uint32_t r = r0 + u * rps;
                            if (r < m.count && ((live >> r) & 1u))
                                st_v4(dst + size_t(r) * p.row_bytes + v * 16, val[u]);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive(empty + stage);
        }
    } else if (p.packs > 0) {
        // Scale warps: warp 2 + j takes the CTA's tiles k = j, j + 2, ...  It
        // reads the tile's indices from the stage (never a second read from
        // global or pinned host memory), copies each row's scales and then
        // releases the stage together with the consumer.
        constexpr uint32_t kSfWarps = kBulkThreads / 32 - 2;
        const uint32_t j = warp - 2;
        for (uint32_t t = t0 + j, k = j; t < t1; t += kSfWarps, k += kSfWarps) {
            const uint32_t stage = k % stages, phase = k / stages;
            if (!mbar_wait(full + stage, phase & 1, kPipelineTimeoutNs)) {
                if (lane == 0)
                    report_error(p.error, kPipelineTimeout, 0, 2 + j, t, 0);
                break;
            }
            const StageMeta m = meta[stage];
            const int32_t x = stage_x[stage * kBulkTile + lane];
            __syncwarp();
            if (lane < m.count) {
                const uint32_t r = m.start + lane;
                const uint32_t token = r / p.ept, slot = r - token * p.ept;
                float *out = p.sf_output + uint64_t(m.layer) * p.sf_layer_stride + uint64_t(token) * p.sf_token_stride +
                             uint64_t(slot) * p.packs * p.sf_hidden_stride;
                const float *src = nullptr;
                if (x >= 0) {
                    const uint32_t span = s_entries[m.layer] * p.sf_shard_div;
                    const uint32_t shard = uint32_t(x) / span;
                    if (shard < p.world && s_sf[shard] != 0)
                        src = reinterpret_cast<const float *>(s_sf[shard]) + s_sfbase[m.layer] +
                              uint64_t(uint32_t(x) - shard * span) * p.packs;
                }
                uint32_t q = 0;
                for (; q + 2 <= p.packs; q += 2) {
                    const float v0 = src != nullptr ? __ldg(src + q) : 0.0f;
                    const float v1 = src != nullptr ? __ldg(src + q + 1) : 0.0f;
                    out[uint64_t(q) * p.sf_hidden_stride] = v0;
                    out[uint64_t(q + 1) * p.sf_hidden_stride] = v1;
                }
                if (q < p.packs)
                    out[uint64_t(q) * p.sf_hidden_stride] = src != nullptr ? __ldg(src + q) : 0.0f;
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive(empty + stage);
        }
    }
}

// ------------------------------------------------------------ SIMT variant
// A warp walks its items 32 at a time (one step).  Lane l resolves the step's
// item l once (owner, source, destination, scales) and the copy loop hands the
// 16-byte vectors of each row to LPR lanes with two shuffles per row, so the
// per-row integer work is done by one lane instead of LPR lanes.  The next
// kIndexAhead steps' indices are loaded before this step's rows, hiding that latency.
template <int LPR, int VPL, int UNROLL, int VB = 16, bool L2HINT = false>
__global__ void __launch_bounds__(kSimtThreads, 2) gather_simt_kernel(const __grid_constant__ GatherParams p) {
    using V = typename std::conditional<L2HINT, RowVec32L2, RowVec<VB>>::type;
    __shared__ uint64_t s_direct[kMaxRanks], s_sf[kMaxRanks];
    __shared__ int32_t s_index[kSimtThreads / 32][kIndexAhead * 32];
    __shared__ uint32_t s_entries[kMaxLayers], s_tbase[kMaxLayers], s_sfbase[kMaxLayers];
    __shared__ uint32_t s_hot[kMaxLayers], s_hotbase[kMaxLayers];
    load_tables(p, s_direct, s_sf, s_entries, s_tbase, s_sfbase, s_hot, s_hotbase);
    __syncthreads();

    constexpr uint32_t kRowsPerStep = 32 / LPR;
    constexpr uint32_t kMaxPacksInFlight = 4;
    const uint32_t lane = threadIdx.x % 32;
    const uint32_t sub = lane / LPR, vlane = lane % LPR;
    const uint32_t vectors = p.row_bytes / VB;
    const uint32_t total = p.layers * p.rows;
    const uint32_t warp_id = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const uint32_t warps = gridDim.x * (blockDim.x / 32);
    // Work split.  Contiguous (default): warp w owns items [lo, hi), an equal
    // share of all items, so no warp runs a whole 32-row group more than
    // another (with 4736 warps and 6144 groups, a group stride leaves some
    // warps two groups and others one).  Strided: warp w owns groups
    // w, w + warps, ...  Step k covers items base(k) + lane.
    uint32_t lo, hi, step_stride, steps;
    if (p.strided) {
        lo = warp_id * 32;
        hi = total;
        step_stride = warps * 32;
        steps = lo < total ? (total - lo + step_stride - 1) / step_stride : 0;
    } else {
        const uint32_t share = (total + warps - 1) / warps;
        lo = min(warp_id * share, total);
        hi = min(lo + share, total);
        step_stride = 32;
        steps = (hi - lo + 31) / 32;
    }

    const uint32_t epoch = p.dedup ? dedup_epoch(p.dedup_state) : 0;
    // The indices of this warp's next kIndexAhead steps are in flight at
    // once, copied by cp.async into a per-warp shared ring.  Their completion
    // is tracked apart from the row loads' registers, so a row copy never
    // waits on a later step's index (a PCIe round trip when the indices sit
    // in pinned host memory).  Each lane reads back only what it copied.
    int32_t *ring = s_index[threadIdx.x / 32];
#pragma unroll
    for (uint32_t a = 0; a < kIndexAhead; ++a) {
        const uint32_t item = lo + a * step_stride + lane;
        if (a < steps && item < hi)
            cp_async_4(ring + a * 32 + lane, p.indices + item);
        else
            *reinterpret_cast<volatile int32_t *>(ring + a * 32 + lane) = -1;
        cp_async_commit();
    }
    for (uint32_t k = 0; k < steps; ++k) {
        const uint32_t base = lo + k * step_stride;
        const uint32_t item = base + lane;
        const uint32_t live = min(32u, hi - base);  // items of this step
        cp_async_wait<kIndexAhead - 1>();  // step k has landed
        int32_t *slot_x = ring + (k % kIndexAhead) * 32 + lane;
        const int32_t x = *reinterpret_cast<volatile int32_t *>(slot_x);
        // Resolve this lane's item; its scale loads are issued now and stored
        // after the rows, so their latency overlaps the row copies.
        uint64_t src = 0, dst = 0;  // src == 0 && dst != 0: zero row; dst == 0: not ours
        float *sf_out = nullptr;
        const float *sf_src = nullptr;
        float sf_val[kMaxPacksInFlight];
        if (item < hi) {
            const uint32_t layer = item / p.rows;
            const uint32_t at = item - layer * p.rows;
            dst = reinterpret_cast<uint64_t>(p.output) + (uint64_t(layer) * p.capacity + at) * p.row_bytes;
            if (x >= 0) {
                const uint32_t n = s_entries[layer];
                const uint32_t owner = uint32_t(x) / n;
                if (owner >= p.world) {
                    report_error(p.error, kIndexOutOfRange, layer, owner, uint64_t(x), 0);
                } else if (uint32_t(x) < s_hot[layer]) {  // replicated hot row: local copy
                    src = p.hot_base + (uint64_t(s_hotbase[layer]) + uint32_t(x)) * p.row_bytes;
                } else if (s_direct[owner] != 0) {
                    if (p.dedup && dedup_duplicate(p, item, epoch))
                        dst = 0;  // a repeat: copied from its first occurrence after the gather
                    else
                        src = s_direct[owner] + (uint64_t(s_tbase[layer]) + (uint32_t(x) - owner * n)) * p.row_bytes;
                } else {
                    dst = 0;  // host route: the owner pushes this row
                }
            }
            if (p.packs > 0) {
                const uint32_t token = at / p.ept, slot = at - token * p.ept;
                sf_out = p.sf_output + uint64_t(layer) * p.sf_layer_stride + uint64_t(token) * p.sf_token_stride +
                         uint64_t(slot) * p.packs * p.sf_hidden_stride;
                if (x >= 0) {
                    const uint32_t span = s_entries[layer] * p.sf_shard_div;
                    const uint32_t shard = uint32_t(x) / span;
                    if (shard < p.world && s_sf[shard] != 0)
                        sf_src = reinterpret_cast<const float *>(s_sf[shard]) + s_sfbase[layer] +
                                 uint64_t(uint32_t(x) - shard * span) * p.packs;
                }
#pragma unroll
                for (uint32_t k = 0; k < kMaxPacksInFlight; ++k)
                    sf_val[k] = (sf_src != nullptr && k < p.packs) ? __ldg(sf_src + k) : 0.0f;
            }
        }
        // Refill the slot with step k + kIndexAhead (x is consumed above).
        {
            const uint32_t next = k + kIndexAhead;
            const uint32_t nitem = lo + next * step_stride + lane;
            if (next < steps && nitem < hi)
                cp_async_4(slot_x, p.indices + nitem);
            else
                *reinterpret_cast<volatile int32_t *>(slot_x) = -1;
            cp_async_commit();
        }
        // Copy the step's rows: UNROLL row-steps x VPL vectors in flight per lane.
        for (uint32_t r0 = 0; r0 < live; r0 += kRowsPerStep * UNROLL) {
            uint64_t rs[UNROLL], rd[UNROLL];
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) {
                const uint32_t r = r0 + u * kRowsPerStep + sub;
                rs[u] = __shfl_sync(0xFFFFFFFFu, src, r % 32);
                rd[u] = __shfl_sync(0xFFFFFFFFu, dst, r % 32);
                if (r >= live)  // past this step's items (and no lane-wrapped repeats)
                    rs[u] = rd[u] = 0;
            }
            for (uint32_t chunk = 0; chunk < vectors; chunk += LPR * VPL) {
                typename V::T buf[UNROLL][VPL];
#pragma unroll
                for (int u = 0; u < UNROLL; ++u)
#pragma unroll
                    for (int k = 0; k < VPL; ++k) {
                        const uint32_t v = chunk + vlane + k * LPR;
                        buf[u][k] = V::zero();
                        if (rs[u] != 0 && v < vectors)
                            buf[u][k] = V::load(reinterpret_cast<const uint8_t *>(rs[u]) + uint64_t(v) * VB);
                    }
#pragma unroll
                for (int u = 0; u < UNROLL; ++u)
#pragma unroll
                    for (int k = 0; k < VPL; ++k) {
                        const uint32_t v = chunk + vlane + k * LPR;
                        if (rd[u] != 0 && v < vectors)
                            V::store(reinterpret_cast<uint8_t *>(rd[u]) + uint64_t(v) * VB, buf[u][k]);
                    }
            }
        }
        if (sf_out != nullptr) {
#pragma unroll
            for (uint32_t k = 0; k < kMaxPacksInFlight; ++k)
                if (k < p.packs)
                    sf_out[uint64_t(k) * p.sf_hidden_stride] = sf_val[k];
            for (uint32_t k = kMaxPacksInFlight; k < p.packs; ++k)
                sf_out[uint64_t(k) * p.sf_hidden_stride] = sf_src != nullptr ? __ldg(sf_src + k) : 0.0f;
        }
    }
}

template <int LPR, int VPL, int UNROLL, int VB = 16, bool L2HINT = false>
cudaError_t launch_simt(const GatherParams &p, int num_sms, cudaStream_t stream) {
    const uint32_t total = p.layers * p.rows;
    const uint32_t warps = kSimtThreads / 32;
    // Small batches are spread over more SMs (down to 4 items per warp) so
    // their latency is one round of row loads; large ones fill the grid cap.
    constexpr uint32_t kMinItemsPerWarp = 4;
    const uint32_t per_block = p.strided ? warps * 32 : warps * kMinItemsPerWarp;
    uint32_t blocks = (total + per_block - 1) / per_block;
    const uint32_t cap = uint32_t(num_sms) * (p.ctas_per_sm ? p.ctas_per_sm : 2);
    blocks = blocks < cap ? blocks : cap;
    if (blocks == 0)
        return cudaSuccess;
    gather_simt_kernel<LPR, VPL, UNROLL, VB, L2HINT><<<blocks, kSimtThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_simt_any(const GatherParams &p, int num_sms, cudaStream_t stream) {
    const uint32_t vectors = p.row_bytes / 16;
    // 256-bit vectors: 32-byte multiples of 128 bytes and more (8 lanes per
    // 256-byte row); the 16-byte kernels serve every other row size.
    if (p.vector_bytes == 32 && p.row_bytes % 32 == 0 && vectors >= 8) {
        if (p.l2_prefetch && vectors <= 16)
            return launch_simt<8, 1, 4, 32, true>(p, num_sms, stream);
        if (vectors <= 16)
            return launch_simt<8, 1, 4, 32>(p, num_sms, stream);
        if (vectors <= 32)
            return launch_simt<16, 1, 4, 32>(p, num_sms, stream);
        return launch_simt<32, 1, 4, 32>(p, num_sms, stream);
    }
    if (vectors <= 2)
        return launch_simt<2, 1, 4>(p, num_sms, stream);
    if (vectors <= 4)
        return launch_simt<4, 1, 4>(p, num_sms, stream);
    if (vectors <= 8)
        return launch_simt<4, 2, 4>(p, num_sms, stream);
    if (vectors <= 16) {
        if (p.unroll == 2)
            return launch_simt<8, 2, 2>(p, num_sms, stream);
        if (p.unroll == 8)
            return launch_simt<8, 2, 8>(p, num_sms, stream);
        if (p.unroll == 1)
            return launch_simt<16, 1, 4>(p, num_sms, stream);
        return launch_simt<8, 2, 4>(p, num_sms, stream);
    }
    if (vectors <= 32)
        return launch_simt<16, 2, 4>(p, num_sms, stream);
    return launch_simt<32, 2, 4>(p, num_sms, stream);
}

cudaError_t launch_bulk(const GatherParams &p, int num_sms, cudaStream_t stream) {
    const uint32_t stage_bytes = kBulkTile * p.row_bytes;
    uint32_t stages = kStageTargetBytes / stage_bytes;
    stages = stages < 2 ? 2 : (stages > 8 ? 8 : stages);
    const size_t smem =
        size_t(stages) * stage_bytes + size_t(stages) * (16 + sizeof(StageMeta) + kBulkTile * sizeof(int32_t));
    static size_t configured = 0;
    if (smem > configured) {
        cudaError_t rc =
            cudaFuncSetAttribute(gather_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        if (rc != cudaSuccess)
            return rc;
        configured = smem;
    }
    int per_sm = 0;
    cudaError_t rc = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gather_bulk_kernel, kBulkThreads, smem);
    if (rc != cudaSuccess)
        return rc;
    per_sm = per_sm < 1 ? 1 : per_sm;
    const uint32_t tiles_per_layer = (p.rows + kBulkTile - 1) / kBulkTile;
    const uint32_t total_tiles = tiles_per_layer * p.layers;
    uint32_t grid = uint32_t(num_sms) * uint32_t(per_sm);
    grid = grid < total_tiles ? grid : total_tiles;
    const uint32_t tiles_per_cta = (total_tiles + grid - 1) / grid;
    grid = (total_tiles + tiles_per_cta - 1) / tiles_per_cta;
    gather_bulk_kernel<<<grid, kBulkThreads, smem, stream>>>(p, tiles_per_layer, tiles_per_cta, stages);
    return cudaGetLastError();
}

} // namespace

cudaError_t launch_gather(const GatherParams &p, int num_sms, cudaStream_t stream) {
    if (p.layers == 0 || p.rows == 0)
        return cudaSuccess;
    // The ring needs two stages of 32 rows; larger rows use the SIMT kernel.
    if (p.variant == kGatherSimt || p.row_bytes > 2048)
        return launch_simt_any(p, num_sms, stream);
    return launch_bulk(p, num_sms, stream);
}

} // namespace engram
