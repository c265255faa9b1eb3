// Requester-side gather (sm_100a): the hot kernel of the peer-HBM route.
//
// Parity: the reference's direct-read paths, `engram_fetch.cuh:70-101` (READ,
// EGM rows) + `:223-269` (scale warps) and `gpu_request.cu:214-270`
// (`issue_egm`, WRITE).  Differences by design:
//   * the source of a direct row is the owner's HBM mirror reached through
//     NVLink 5 / NVSwitch (or this rank's own shard), not host memory over C2C;
//   * route tables, layer geometry and strides are kernel parameters
//     (__grid_constant__), so CUDA Graph replays carry them without any
//     device-side metadata upload;
//   * every lane keeps several independent 16-byte loads in flight (UNROLL
//     rows per lane) so that ~10 MB of requests are outstanding GPU-wide, far
//     above the NVLink bandwidth-delay product, and stores go straight to the
//     final [tokens, hidden*ept] position (no reorder pass);
//   * an out-of-range index is recorded in the error record and zero-filled
//     instead of trapping.
// Loads from peer memory are plain per-thread vector loads: no TMA and no
// cluster multicast touches another GPU's memory.
#include "params.h"
#include "ptx.cuh"

namespace engram {

namespace {

constexpr int kGatherThreads = 512;

template <int LPR, int VPL, int UNROLL>
__global__ void __launch_bounds__(kGatherThreads, 2) gather_kernel(const __grid_constant__ GatherParams p) {
    __shared__ uint64_t s_direct[kMaxRanks];
    __shared__ uint64_t s_sf[kMaxRanks];
    __shared__ uint32_t s_entries[kMaxLayers], s_tbase[kMaxLayers], s_sfbase[kMaxLayers];
    for (uint32_t i = threadIdx.x; i < p.world; i += blockDim.x) {
        s_direct[i] = p.direct_base[i];
        s_sf[i] = p.sf_base[i];
    }
    for (uint32_t i = threadIdx.x; i < p.layers; i += blockDim.x) {
        s_entries[i] = p.layer.entries[i];
        s_tbase[i] = p.layer.table_bases[i];
        s_sfbase[i] = p.layer.sf_bases[i];
    }
    __syncthreads();

    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t num_warps = blockDim.x / 32;
    const uint32_t row_warps = num_warps - p.sf_warps;
    const uint64_t total = uint64_t(p.layers) * p.rows;

    if (warp < row_warps) {
        constexpr uint32_t kRowsPerStep = 32 / LPR;
        constexpr uint32_t kRowsPerIter = kRowsPerStep * UNROLL;
        const uint32_t sub = lane / LPR, vlane = lane % LPR;
        const uint32_t vectors = p.row_bytes / 16;
        const uint64_t first = (uint64_t(blockIdx.x) * row_warps + warp) * kRowsPerIter;
        const uint64_t stride = uint64_t(gridDim.x) * row_warps * kRowsPerIter;
        for (uint64_t base = first; base < total; base += stride) {
            const uint8_t *src[UNROLL];
            uint8_t *dst[UNROLL];
            bool zero[UNROLL];
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) {
                const uint64_t item = base + u * kRowsPerStep + sub;
                src[u] = nullptr;
                dst[u] = nullptr;
                zero[u] = false;
                if (item < total) {
                    const uint32_t layer = uint32_t(item / p.rows);
                    const uint32_t at = uint32_t(item - uint64_t(layer) * p.rows);
                    const int32_t x = __ldg(p.indices + item);
                    dst[u] = p.output + (uint64_t(layer) * p.capacity + at) * p.row_bytes;
                    if (x < 0) {
                        zero[u] = true;
                    } else {
                        const uint32_t n = s_entries[layer];
                        const uint32_t owner = uint32_t(x) / n;
                        if (owner >= p.world) {
                            zero[u] = true;
                            if (vlane == 0)
                                report_error(p.error, kIndexOutOfRange, layer, owner, uint64_t(x), 0);
                        } else if (s_direct[owner] != 0) {
                            const uint64_t row = uint64_t(s_tbase[layer]) + (uint32_t(x) - owner * n);
                            src[u] = reinterpret_cast<const uint8_t *>(s_direct[owner]) + row * p.row_bytes;
                        } else {
                            dst[u] = nullptr;  // host route: the owner pushes this row
                        }
                    }
                }
            }
            for (uint32_t chunk = 0; chunk < vectors; chunk += LPR * VPL) {
                Vec16 buf[UNROLL][VPL];
#pragma unroll
                for (int u = 0; u < UNROLL; ++u)
#pragma unroll
                    for (int k = 0; k < VPL; ++k) {
                        const uint32_t v = chunk + vlane + k * LPR;
                        if (src[u] != nullptr && v < vectors)
                            buf[u][k] = ld_nc_na_v4(src[u] + uint64_t(v) * 16);
                    }
#pragma unroll
                for (int u = 0; u < UNROLL; ++u)
#pragma unroll
                    for (int k = 0; k < VPL; ++k) {
                        const uint32_t v = chunk + vlane + k * LPR;
                        if (dst[u] == nullptr || v >= vectors)
                            continue;
                        if (zero[u])
                            st_v4(dst[u] + uint64_t(v) * 16, Vec16{0, 0, 0, 0});
                        else if (src[u] != nullptr)
                            st_v4(dst[u] + uint64_t(v) * 16, buf[u][k]);
                    }
            }
        }
    } else if (p.packs > 0) {
        // Scale warps: one (layer, row) item per lane; for the column-major
        // layout consecutive lanes take consecutive tokens of one entry slot so
        // the strided output is written coalesced.
        const uint32_t sf_lane = (warp - row_warps) * 32 + lane;
        const uint64_t first = uint64_t(blockIdx.x) * p.sf_warps * 32 + sf_lane;
        const uint64_t stride = uint64_t(gridDim.x) * p.sf_warps * 32;
        for (uint64_t item = first; item < total; item += stride) {
            const uint32_t layer = uint32_t(item / p.rows);
            const uint32_t r = uint32_t(item - uint64_t(layer) * p.rows);
            uint32_t token, slot;
            if (p.col_major_sf) {
                slot = r / p.tokens;
                token = r - slot * p.tokens;
            } else {
                token = r / p.ept;
                slot = r - token * p.ept;
            }
            const uint32_t at = token * p.ept + slot;
            const int32_t x = __ldg(p.indices + uint64_t(layer) * p.rows + at);
            float *out = p.sf_output + uint64_t(layer) * p.sf_layer_stride + uint64_t(token) * p.sf_token_stride +
                         uint64_t(slot) * p.packs * p.sf_hidden_stride;
            const float *src = nullptr;
            if (x >= 0) {
                const uint32_t span = s_entries[layer] * p.sf_shard_div;
                const uint32_t shard = uint32_t(x) / span;
                if (shard < p.world && s_sf[shard] != 0)
                    src = reinterpret_cast<const float *>(s_sf[shard]) + s_sfbase[layer] +
                          uint64_t(uint32_t(x) - shard * span) * p.packs;
            }
            for (uint32_t k = 0; k < p.packs; ++k)
                out[uint64_t(k) * p.sf_hidden_stride] = src != nullptr ? __ldg(src + k) : 0.0f;
        }
    }
}

template <int LPR, int VPL, int UNROLL>
cudaError_t launch_variant(const GatherParams &p, int num_sms, cudaStream_t stream) {
    const uint32_t warps = kGatherThreads / 32;
    const uint32_t row_warps = warps - p.sf_warps;
    const uint64_t total = uint64_t(p.layers) * p.rows;
    const uint64_t per_block = uint64_t(row_warps) * (32 / LPR) * UNROLL;
    uint64_t blocks = (total + per_block - 1) / per_block;
    blocks = blocks < uint64_t(num_sms) * 2 ? blocks : uint64_t(num_sms) * 2;
    if (blocks == 0)
        return cudaSuccess;
    gather_kernel<LPR, VPL, UNROLL><<<unsigned(blocks), kGatherThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

} // namespace

cudaError_t launch_gather(const GatherParams &p, int num_sms, cudaStream_t stream) {
    if (p.layers == 0 || p.rows == 0)
        return cudaSuccess;
    const uint32_t vectors = p.row_bytes / 16;
    if (vectors <= 4)
        return launch_variant<4, 1, 4>(p, num_sms, stream);
    if (vectors <= 8)
        return launch_variant<8, 1, 4>(p, num_sms, stream);
    if (vectors <= 16)
        return launch_variant<16, 1, 4>(p, num_sms, stream);
    if (vectors <= 32)
        return launch_variant<32, 1, 4>(p, num_sms, stream);
    if (vectors <= 64)
        return launch_variant<32, 2, 2>(p, num_sms, stream);
    return launch_variant<32, 4, 1>(p, num_sms, stream);
}

} // namespace engram
