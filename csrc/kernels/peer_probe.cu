// Peer-memory probe for random rows (sm_100a): the NVLink envelope that the
// Engram gather and owner push live in, measured with the access patterns they
// can use.  Every launch moves `rows` rows of `row_bytes` between this GPU and
// its peers in an all-to-all pattern (row i belongs to a pseudo-random remote
// peer and a pseudo-random table row; push destinations are pseudo-random
// output rows), so it reproduces the traffic of a uniform fetch without the
// gather's bookkeeping.
//
// Mechanisms (ProbeMode):
//   pull_v4 / pull_v8   requester SMs load 16 / 32 bytes per lane from the
//                       peer's table and store locally (registers in flight)
//   pull_ldgsts         16-byte cp.async (global -> shared, no registers held)
//                       into a per-warp ring, then shared -> local output
//   push_v4 / push_v8   owner SMs load local rows and store 16 / 32 bytes per
//                       lane into the peer's output
//   push_bulk           owner SMs bulk-load local rows into shared memory and
//                       bulk-store each row into the peer's output
//                       (cp.async.bulk shared -> global; a store, never a load,
//                       touches peer memory)
//   push_seq_v8         32-byte stores of random local rows into consecutive
//                       rows of each peer's output (a staging-buffer pattern)
//   pull_seq_v8         32-byte loads of consecutive peer rows (streaming)
//   pull_v8_l2          32-byte loads with the .L2::256B prefetch-size hint
// Even CTAs run `mode_even`, odd CTAs `mode_odd`, so one launch can also
// measure pull and push sharing the links.  Diagnostics only: it overwrites
// output regions and runs between fetches.  No reference counterpart.
#include "params.h"
#include "ptx.cuh"

namespace engram {

namespace {

constexpr int kProbeThreads = 256;
constexpr uint32_t kProbeWarps = kProbeThreads / 32;
constexpr uint32_t kRingBytesPerWarp = 8192;
constexpr uint64_t kProbeWaitNs = 2000000000ull;

__device__ __forceinline__ uint32_t mix32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7FEB352Du;
    x ^= x >> 15;
    x *= 0x846CA68Bu;
    x ^= x >> 16;
    return x;
}

struct RowPlan {
    const uint8_t *src;
    uint8_t *dst;
};

__device__ __forceinline__ RowPlan plan_row(const PeerProbeParams &p, uint32_t i, bool push, bool seq = false) {
    const uint32_t h = mix32(i * 2654435761u + p.seed);
    uint32_t peer = p.rank;
    if (seq) {
        // Row i goes to (or comes from) peer i % (world - 1) at its row
        // i / (world - 1): consecutive rows per peer, every peer busy.
        const uint32_t others = p.world > 1 ? p.world - 1 : 1;
        const uint32_t q = i / others;
        if (p.world > 1)
            peer = (p.rank + 1 + i % others) % p.world;
        RowPlan r;
        if (push) {
            r.src = p.local_table + uint64_t(mix32(h ^ 0x9E3779B9u) % p.table_rows) * p.row_bytes;
            r.dst = reinterpret_cast<uint8_t *>(p.peer_out[peer]) + uint64_t(q % p.out_rows) * p.row_bytes;
        } else {
            r.src = reinterpret_cast<const uint8_t *>(p.peer_table[peer]) + uint64_t(q % p.table_rows) * p.row_bytes;
            r.dst = p.local_out + uint64_t(i % p.out_rows) * p.row_bytes;
        }
        return r;
    }
    if (p.world > 1)
        peer = (p.rank + 1 + h % (p.world - 1)) % p.world;
    const uint64_t trow = mix32(h ^ 0x9E3779B9u) % p.table_rows;
    RowPlan r;
    if (push) {
        const uint64_t orow = mix32(h ^ 0x85EBCA6Bu) % p.out_rows;
        r.src = p.local_table + trow * p.row_bytes;
        r.dst = reinterpret_cast<uint8_t *>(p.peer_out[peer]) + orow * p.row_bytes;
    } else {
        r.src = reinterpret_cast<const uint8_t *>(p.peer_table[peer]) + trow * p.row_bytes;
        r.dst = p.local_out + uint64_t(i % p.out_rows) * p.row_bytes;
    }
    return r;
}

// Register path: LPR lanes per row, BYTES per lane per access, UNROLL row
// groups in flight per lane.
template <int BYTES, int UNROLL, bool L2HINT = false>
__device__ void run_regs(const PeerProbeParams &p, bool push, uint32_t lo, uint32_t hi, uint32_t warp, uint32_t warps,
                         bool seq = false) {
    const uint32_t lane = threadIdx.x % 32;
    const uint32_t lpr = min(32u, p.row_bytes / BYTES);
    const uint32_t rps = 32 / lpr;  // rows per warp access
    const uint32_t sub = lane / lpr, vl = lane % lpr;
    const uint32_t per_lane = p.row_bytes / (BYTES * lpr);
    for (uint32_t base = lo + warp * rps * UNROLL; base < hi; base += warps * rps * UNROLL) {
        RowPlan rp[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            const uint32_t i = base + u * rps + sub;
            rp[u] = i < hi && sub < rps ? plan_row(p, i, push, seq) : RowPlan{nullptr, nullptr};
        }
        for (uint32_t c = 0; c < per_lane; ++c) {
            const uint32_t off = (c * lpr + vl) * BYTES;
            if constexpr (BYTES == 16) {
                Vec16 v[UNROLL];
#pragma unroll
                for (int u = 0; u < UNROLL; ++u)
                    if (rp[u].src)
                        v[u] = ld_nc_na_v4(rp[u].src + off);
#pragma unroll
                for (int u = 0; u < UNROLL; ++u)
                    if (rp[u].src)
                        st_v4(rp[u].dst + off, v[u]);
            } else {
                Vec32 v[UNROLL];
#pragma unroll
                for (int u = 0; u < UNROLL; ++u)
                    if (rp[u].src)
                        v[u] = L2HINT ? ld_nc_na_l2_256_v8(rp[u].src + off) : ld_nc_na_v8(rp[u].src + off);
#pragma unroll
                for (int u = 0; u < UNROLL; ++u)
                    if (rp[u].src)
                        st_v8(rp[u].dst + off, v[u]);
            }
        }
    }
}

__device__ __forceinline__ void cp_async_16(void *dst_smem, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst_smem)), "l"(src) : "memory");
}

// LDGSTS ring: one warp access moves 2 rows (16 lanes x 16 B each); a stage
// is one such access; kStages stages in flight per warp.
__device__ void run_ldgsts(const PeerProbeParams &p, uint8_t *ring, uint32_t lo, uint32_t hi, uint32_t warp,
                           uint32_t warps) {
    constexpr uint32_t kStages = kRingBytesPerWarp / 512;
    const uint32_t lane = threadIdx.x % 32;
    const uint32_t sub = lane / 16, vl = lane % 16;
    // Steps of 2 rows owned by this warp: i = lo + (warp + k * warps) * 2 + sub.
    const uint32_t pairs = (hi - lo + 1) / 2;
    const uint32_t steps = warp < pairs ? (pairs - warp + warps - 1) / warps : 0;
    uint8_t *dsts[kStages];
    for (uint32_t k = 0; k < steps + kStages - 1; ++k) {
        if (k < steps) {
            const uint32_t i = lo + (warp + k * warps) * 2 + sub;
            uint8_t *slot = ring + (k % kStages) * 512 + lane * 16;
            uint8_t *dst = nullptr;
            if (i < hi) {
                const RowPlan rp = plan_row(p, i, false);
                cp_async_16(slot, rp.src + vl * 16);
                dst = rp.dst + vl * 16;
            }
            dsts[k % kStages] = dst;
        }
        cp_async_commit();
        if (k + 1 >= kStages) {
            const uint32_t j = k + 1 - kStages;  // stage to drain
            cp_async_wait<kStages - 1>();
            uint8_t *dst = dsts[j % kStages];
            if (dst != nullptr)
                st_v4(dst, ld_shared_v4(ring + (j % kStages) * 512 + lane * 16));
        }
    }
    cp_async_wait<0>();
}

__device__ __forceinline__ void bulk_store(void *dst_global, const void *src_smem, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst_global),
                 "r"(smem_addr(src_smem)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Bulk push: a stage is 8 rows; lanes 0-7 each bulk-load one local row into
// the stage (completing on the stage's mbarrier) and then bulk-store it into
// the peer's output.  kStages stages per warp.
__device__ bool run_push_bulk(const PeerProbeParams &p, uint8_t *ring, uint64_t *bars, uint32_t lo, uint32_t hi,
                              uint32_t warp, uint32_t warps) {
    constexpr uint32_t kRowsPerStage = 8;
    const uint32_t stage_bytes = kRowsPerStage * p.row_bytes;
    const uint32_t stages = kRingBytesPerWarp / stage_bytes;
    const uint32_t lane = threadIdx.x % 32;
    if (lane < stages)
        mbar_init(bars + lane, 1);
    fence_mbar_init();
    __syncwarp();
    const uint32_t groups = (hi - lo + kRowsPerStage - 1) / kRowsPerStage;
    const uint32_t steps = warp < groups ? (groups - warp + warps - 1) / warps : 0;
    bool ok = true;
    // Issue loads for stage k, store stage k - (stages - 1): loads of later
    // stages overlap stores of earlier ones.
    uint8_t *dst_of[8] = {};
    for (uint32_t k = 0; k < steps + stages - 1 && ok; ++k) {
        if (k < steps) {
            const uint32_t s = k % stages;
            if (k >= stages) {
                // The bulk stores of this stage's previous use must have read
                // shared memory before it is overwritten.
                if (lane < kRowsPerStage)
                    bulk_wait_read<0>();
                __syncwarp();
            }
            const uint32_t i = lo + (warp + k * warps) * kRowsPerStage + lane;
            const bool live = lane < kRowsPerStage && i < hi;
            RowPlan rp{nullptr, nullptr};
            if (live)
                rp = plan_row(p, i, true);
            const uint32_t n = __popc(__ballot_sync(0xFFFFFFFFu, live));
            if (lane == 0)
                mbar_arrive_expect_tx(bars + s, n * p.row_bytes);
            __syncwarp();
            if (live)
                bulk_load(ring + s * stage_bytes + lane * p.row_bytes, rp.src, p.row_bytes, bars + s);
            if (lane < kRowsPerStage)
                dst_of[s] = live ? rp.dst : nullptr;
        }
        if (k + 1 >= stages) {
            const uint32_t j = k + 1 - stages;
            const uint32_t s = j % stages;
            if (!mbar_wait(bars + s, (j / stages) & 1, kProbeWaitNs)) {
                ok = false;
                break;
            }
            if (lane < kRowsPerStage && dst_of[s] != nullptr) {
                bulk_store(dst_of[s], ring + s * stage_bytes + lane * p.row_bytes, p.row_bytes);
                bulk_commit();
            }
        }
    }
    if (lane < kRowsPerStage)
        bulk_wait_read<0>();
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    return ok;
}

__global__ void __launch_bounds__(kProbeThreads) peer_probe_kernel(const __grid_constant__ PeerProbeParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t warp_in_cta = threadIdx.x / 32;
    uint8_t *ring = smem + warp_in_cta * kRingBytesPerWarp;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kProbeWarps * kRingBytesPerWarp) + warp_in_cta * 8;
    // CTA parity picks the mode; each parity class splits its share of rows.
    const bool odd = blockIdx.x & 1;
    const uint32_t mode = odd ? p.mode_odd : p.mode_even;
    const uint32_t ctas_even = (gridDim.x + 1) / 2, ctas_odd = gridDim.x / 2;
    const uint32_t split = p.mode_even == p.mode_odd || ctas_odd == 0 ? p.rows : uint32_t(uint64_t(p.rows) * p.even_share_pct / 100);
    uint32_t lo, hi, cta, ctas;
    if (p.mode_even == p.mode_odd || ctas_odd == 0) {
        lo = 0, hi = p.rows, cta = blockIdx.x, ctas = gridDim.x;
    } else if (!odd) {
        lo = 0, hi = split, cta = blockIdx.x / 2, ctas = ctas_even;
    } else {
        lo = split, hi = p.rows, cta = blockIdx.x / 2, ctas = ctas_odd;
    }
    const uint32_t warp = cta * kProbeWarps + warp_in_cta, warps = ctas * kProbeWarps;
    bool ok = true;
    switch (mode) {
    case kProbePullV4:
        run_regs<16, 4>(p, false, lo, hi, warp, warps);
        break;
    case kProbePullV4Deep:
        run_regs<16, 8>(p, false, lo, hi, warp, warps);
        break;
    case kProbePullV8:
        run_regs<32, 4>(p, false, lo, hi, warp, warps);
        break;
    case kProbePullLdgsts:
        run_ldgsts(p, ring, lo, hi, warp, warps);
        break;
    case kProbePushV4:
        run_regs<16, 4>(p, true, lo, hi, warp, warps);
        break;
    case kProbePushV8:
        run_regs<32, 4>(p, true, lo, hi, warp, warps);
        break;
    case kProbePushBulk:
        ok = run_push_bulk(p, ring, bars, lo, hi, warp, warps);
        break;
    case kProbePushSeqV8:
        run_regs<32, 4>(p, true, lo, hi, warp, warps, true);
        break;
    case kProbePullSeqV8:
        run_regs<32, 4>(p, false, lo, hi, warp, warps, true);
        break;
    case kProbePullV8L2:
        run_regs<32, 4, true>(p, false, lo, hi, warp, warps);
        break;
    default:
        break;
    }
    if (!ok && (threadIdx.x % 32) == 0)
        report_error(p.error, kPipelineTimeout, 0, mode, warp, 0);
}

} // namespace

cudaError_t launch_peer_probe(const PeerProbeParams &p, int blocks, cudaStream_t stream) {
    if (blocks <= 0 || p.rows == 0)
        return cudaSuccess;
    const size_t smem = size_t(kProbeWarps) * kRingBytesPerWarp + kProbeWarps * 8 * sizeof(uint64_t);
    static bool configured = false;
    if (!configured) {
        cudaError_t rc =
            cudaFuncSetAttribute(peer_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        if (rc != cudaSuccess)
            return rc;
        configured = true;
    }
    peer_probe_kernel<<<blocks, kProbeThreads, smem, stream>>>(p);
    return cudaGetLastError();
}

} // namespace engram
