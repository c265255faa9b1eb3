// Host-route exchange kernels (sm_100a): dispatch, owner push and hook wait.
//
// Parity with the reference's SGE-WRITE data plane:
//   dispatch  <- `route_counts`/`route_prefix`/`route_pack`/`send_requests`
//                and the fused `pack_send_egm` (gpu_request.cu:8-172, 275-333)
//   push      <- the owner CPU thread + RDMA WRITE (owner_service.hpp:30-81,
//                rdma.hpp:133-167)
//   hook wait <- `finish_layer` (gpu_request.cu:337-372)
// B200 design:
//   * dispatch is one kernel: warp-aggregated atomics (match.any) reserve inbox
//     slots per owner and each (row, position) pair is stored straight into the
//     owner's HBM inbox through NVLink; the last CTA of a layer publishes the
//     mailbox headers with st.release.sys.  Packing order does not matter
//     because every entry carries its final output position.
//   * the owner's GPU reads the rows from its host-pinned shard zero-copy and
//     stores them through NVLink directly into the requester's final output
//     positions, so the hook has nothing to scatter.
//   * per-(layer, owner) epochs advance only for non-empty requests, so empty
//     layers and idle owners keep requester and owner sequences aligned under
//     CUDA Graph replay (gpu_request.cu:47-50, 128-130).
//   * every wait is bounded by the global timer and reports through the error
//     record; nothing traps.
#include "params.h"
#include "ptx.cuh"

namespace engram {

namespace {

constexpr int kDispatchThreads = 256;
constexpr int kPushThreads = 256;
constexpr int kPushLanesPerRow = 16;

__global__ void __launch_bounds__(kDispatchThreads) dispatch_kernel(const __grid_constant__ DispatchParams p) {
    __shared__ uint32_t s_last;
    const uint32_t layer = blockIdx.y;
    const uint32_t n = p.layer.entries[layer];
    const uint32_t tbase = p.layer.table_bases[layer];
    const uint32_t lo = blockIdx.x * p.tile_rows;
    const uint32_t hi = min(lo + p.tile_rows, p.rows);
    const uint32_t lane = threadIdx.x % 32;
    const int32_t *idx = p.indices + uint64_t(layer) * p.rows;

    for (uint32_t base = lo; base < hi; base += blockDim.x) {
        const uint32_t at = base + threadIdx.x;
        const int32_t x = at < hi ? __ldg(idx + at) : -1;
        uint32_t owner = p.world;
        if (x >= 0) {
            owner = uint32_t(x) / n;
            if (owner >= p.world) {
                report_error(p.error, kIndexOutOfRange, layer, owner, uint64_t(x), 0);
                owner = p.world;
            }
        }
        const bool host = owner < p.world && p.inbox_base[owner] != 0;
        const uint32_t key = host ? owner : 0xFFFFFFFFu;
        const uint32_t peers = __match_any_sync(0xFFFFFFFFu, key);
        if (host) {
            const uint32_t leader = __ffs(peers) - 1;
            uint32_t slot = 0;
            if (lane == leader)
                slot = atomicAdd(p.cursors + layer * p.world + owner, __popc(peers));
            slot = __shfl_sync(peers, slot, leader) + __popc(peers & ((1u << lane) - 1));
            if (slot < p.capacity) {
                const uint64_t entry = (uint64_t(at) << 32) | uint64_t(tbase + (uint32_t(x) - owner * n));
                auto *inbox = reinterpret_cast<uint64_t *>(p.inbox_base[owner]);
                inbox[(uint64_t(p.rank) * p.layers + layer) * p.capacity + slot] = entry;
            } else {
                report_error(p.error, kInboxOverflow, layer, owner, slot, p.capacity);
            }
        }
    }
    // Publish this CTA's peer stores system-wide before arriving.
    fence_sc_sys();
    __syncthreads();
    if (threadIdx.x == 0)
        s_last = atom_add_acq_rel_gpu(p.layer_arrivals + layer, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last)
        return;
    fence_acq_rel_gpu();
    for (uint32_t owner = threadIdx.x; owner < p.world; owner += blockDim.x) {
        const uint32_t slot = layer * p.world + owner;
        const uint32_t count = atomicExch(p.cursors + slot, 0u);
        p.totals[slot] = count;
        if (count == 0 || p.header_base[owner] == 0)
            continue;
        const uint64_t epoch = p.epochs[slot] + 1;
        p.epochs[slot] = epoch;
        auto *header = reinterpret_cast<MailboxHeader *>(p.header_base[owner]) +
                       (uint64_t(p.rank) * p.layers + layer);
        st_relaxed_sys_u32(&header->rows, min(count, p.capacity));
        st_relaxed_sys_u32(&header->layer, layer);
        st_relaxed_sys_u32(&header->requester, p.rank);
        st_relaxed_sys_u32(&header->channels, p.channels);
        st_release_sys_u64(&header->ready, epoch);
    }
    if (threadIdx.x == 0)
        p.layer_arrivals[layer] = 0;
}

__global__ void __launch_bounds__(kPushThreads) push_kernel(const __grid_constant__ PushParams p) {
    __shared__ uint32_t s_last;
    // Locate this block's task (blocks are laid out task after task).
    uint32_t t = 0;
    while (t + 1 < p.num_tasks && p.tasks[t + 1].first_block <= blockIdx.x)
        ++t;
    const PushTask task = p.tasks[t];
    const uint32_t block_in_task = blockIdx.x - task.first_block;
    const uint32_t lo = block_in_task * task.rows_per_block;
    const uint32_t hi = min(lo + task.rows_per_block, task.rows);
    const uint32_t task_blocks = (task.rows + task.rows_per_block - 1) / task.rows_per_block;

    const uint64_t *inbox = p.inbox + (uint64_t(task.requester) * p.layers + task.layer) * p.capacity;
    uint8_t *out = reinterpret_cast<uint8_t *>(p.out_base[task.requester]) +
                   uint64_t(task.layer) * p.capacity * p.row_bytes;
    const uint32_t vectors = p.row_bytes / 16;
    constexpr uint32_t kRowsPerStep = kPushThreads / kPushLanesPerRow;
    constexpr int kUnroll = 4;
    const uint32_t sub = threadIdx.x / kPushLanesPerRow, vlane = threadIdx.x % kPushLanesPerRow;

    for (uint32_t base = lo; base < hi; base += kRowsPerStep * kUnroll) {
        const uint8_t *src[kUnroll];
        uint8_t *dst[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const uint32_t i = base + u * kRowsPerStep + sub;
            src[u] = nullptr;
            dst[u] = nullptr;
            if (i < hi) {
                const uint64_t entry = __ldcg(reinterpret_cast<const unsigned long long *>(inbox) + i);
                const uint32_t row = uint32_t(entry), pos = uint32_t(entry >> 32);
                if (row < p.table_rows && pos < p.capacity) {
                    src[u] = p.table + uint64_t(row) * p.row_bytes;
                    dst[u] = out + uint64_t(pos) * p.row_bytes;
                } else if (vlane == 0) {
                    report_error(p.error, kPushBounds, task.layer, task.requester, entry, p.table_rows);
                }
            }
        }
        for (uint32_t chunk = 0; chunk < vectors; chunk += kPushLanesPerRow) {
            Vec16 buf[kUnroll];
            const uint32_t v = chunk + vlane;
#pragma unroll
            for (int u = 0; u < kUnroll; ++u)
                if (src[u] != nullptr && v < vectors)
                    buf[u] = ld_nc_na_v4(src[u] + uint64_t(v) * 16);
#pragma unroll
            for (int u = 0; u < kUnroll; ++u)
                if (dst[u] != nullptr && v < vectors)
                    st_v4(dst[u] + uint64_t(v) * 16, buf[u]);
        }
    }
    // The last block of the task releases the requester's done flag after every
    // block's peer stores are visible system-wide.
    fence_sc_sys();
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t *counter = p.arrivals + uint64_t(task.requester) * p.layers + task.layer;
        s_last = atom_add_acq_rel_gpu(counter, 1u) == task_blocks - 1;
        if (s_last) {
            *counter = 0;
            fence_sc_sys();
            auto *done = reinterpret_cast<uint64_t *>(p.done_base[task.requester]) +
                         (uint64_t(task.layer) * p.world + p.rank);
            st_release_sys_u64(done, task.epoch);
        }
    }
}

__global__ void hook_wait_kernel(const __grid_constant__ HookParams p) {
    for (uint32_t owner = threadIdx.x; owner < p.world; owner += blockDim.x) {
        const uint32_t slot = p.layer * p.world + owner;
        if (p.totals[slot] == 0)
            continue;
        const uint64_t expected = p.epochs[slot];
        bool timed_out = false;
        const uint64_t seen = wait_flag_eq(p.done + slot, expected, p.timeout_ns, &timed_out);
        if (timed_out)
            report_error(p.error, kWaitTimeout, p.layer, owner, seen, expected);
    }
}

__global__ void wait_probe_kernel(const uint64_t *flag, uint64_t expected, uint64_t timeout_ns, ErrorSink error) {
    if (threadIdx.x != 0)
        return;
    bool timed_out = false;
    const uint64_t seen = wait_flag_eq(flag, expected, timeout_ns, &timed_out);
    if (timed_out)
        report_error(error, kWaitTimeout, 0, 0, seen, expected);
}

// Streaming 16-byte copy used to measure the peer-memory envelope (pull: the
// source is a peer mapping; push: the destination is).
__global__ void __launch_bounds__(512) stream_copy_kernel(const Vec16 *src, Vec16 *dst, uint64_t vectors) {
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    for (; i + 3 * stride < vectors; i += 4 * stride) {
        Vec16 a = ld_nc_na_v4(src + i), b = ld_nc_na_v4(src + i + stride), c = ld_nc_na_v4(src + i + 2 * stride),
              d = ld_nc_na_v4(src + i + 3 * stride);
        st_v4(dst + i, a);
        st_v4(dst + i + stride, b);
        st_v4(dst + i + 2 * stride, c);
        st_v4(dst + i + 3 * stride, d);
    }
    for (; i < vectors; i += stride)
        st_v4(dst + i, ld_nc_na_v4(src + i));
}

} // namespace

cudaError_t launch_stream_copy(const void *src, void *dst, uint64_t bytes, int blocks, cudaStream_t stream) {
    stream_copy_kernel<<<blocks, 512, 0, stream>>>(static_cast<const Vec16 *>(src), static_cast<Vec16 *>(dst),
                                                   bytes / 16);
    return cudaGetLastError();
}

cudaError_t launch_dispatch(const DispatchParams &p, cudaStream_t stream) {
    if (p.rows == 0 || p.layers == 0)
        return cudaSuccess;
    dim3 grid((p.rows + p.tile_rows - 1) / p.tile_rows, p.layers);
    dispatch_kernel<<<grid, kDispatchThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_push(const PushParams &p, int blocks, cudaStream_t stream) {
    if (blocks <= 0 || p.num_tasks == 0)
        return cudaSuccess;
    push_kernel<<<blocks, kPushThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_hook_wait(const HookParams &p, cudaStream_t stream) {
    hook_wait_kernel<<<1, 64, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_wait_probe(const uint64_t *flag, uint64_t expected, uint64_t timeout_ns, ErrorSink error,
                              cudaStream_t stream) {
    wait_probe_kernel<<<1, 32, 0, stream>>>(flag, expected, timeout_ns, error);
    return cudaGetLastError();
}

} // namespace engram
