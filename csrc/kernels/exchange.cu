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
//   * the owner's GPU reads the rows from its host-pinned shard zero-copy (or
//     from its HBM mirror when it keeps one) and
//     stores them through NVLink directly into the requester's final output
//     positions, so the hook has nothing to scatter.  A request is split into
//     chunks (512 rows by default) claimed by fetch-and-add, so push kernels launched by the owner's
//     CPU service and the owner's own hook kernels (which serve while they
//     wait) share the work and no GPU spins on work only another launch does.
//   * ids of a replicated hot prefix are never dispatched: the requester's
//     gather reads them from its replica.
//   * per-(layer, owner) epochs advance only for non-empty requests, so empty
//     layers and idle owners keep requester and owner sequences aligned under
//     CUDA Graph replay (gpu_request.cu:47-50, 128-130).
//   * every wait is bounded by the global timer and a poll count, and reports
//     through the error record; nothing traps.
#include "params.h"
#include "ptx.cuh"

namespace engram {

namespace {

constexpr int kDispatchThreads = 256;
constexpr int kPushThreads = 256;
constexpr int kPushLanesPerRow = 16;
constexpr uint32_t kSkipRow = 0xFFFFFFFFu;  // a staged entry that failed its bounds check

__global__ void __launch_bounds__(kDispatchThreads) dispatch_kernel(const __grid_constant__ DispatchParams p) {
    __shared__ uint32_t s_last;
    const uint32_t layer = blockIdx.y;
    const uint32_t n = p.layer.entries[layer];
    const uint32_t tbase = p.layer.table_bases[layer];
    const uint32_t hot = p.layer.hot_rows[layer];
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
        // Replicated hot rows are read locally by the gather, never pushed.
        const bool host = owner < p.world && p.inbox_base[owner] != 0 && uint32_t(x) >= hot;
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
    // Publish this CTA's peer stores system-wide before arriving: the barrier
    // orders every thread's stores before thread 0, whose system-scope fence
    // is cumulative over them.
    __syncthreads();
    if (threadIdx.x == 0) {
        fence_sc_sys();
        s_last = atom_add_acq_rel_gpu(p.layer_arrivals + layer, 1u) == gridDim.x - 1;
    }
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

// ------------------------------------------------------------------ serving
struct Claim {
    int32_t chunk;     // < 0: nothing to claim
    uint32_t epoch32;  // low 32 bits of the epoch the chunk belongs to
    uint32_t limit;    // that epoch's chunk count
};

__device__ __forceinline__ uint32_t chunk_count(uint32_t rows, uint32_t chunk_rows) {
    return (rows + chunk_rows - 1) / chunk_rows;
}

// Claims the next chunk of a request on `claim`.  Arms the word for `epoch`
// (with `chunks` as its limit) if it is still armed for an earlier epoch, then
// takes a chunk with one fetch-and-add.  A CAS claim would let only one of the
// CTAs racing for the word succeed per L2 round trip; additions do not retry
// and pipeline in the L2.  The returned chunk can belong to a later epoch: the
// epoch the caller meant finished and the next one, already published, was
// armed between the look and the addition.
__device__ __forceinline__ Claim claim_chunk(uint64_t *claim, uint64_t epoch, uint32_t chunks, ErrorSink error,
                                             uint32_t l, uint32_t r) {
    unsigned long long *word = reinterpret_cast<unsigned long long *>(claim);
    const uint32_t e32 = uint32_t(epoch);
    unsigned long long old = *reinterpret_cast<volatile unsigned long long *>(word);
    for (uint32_t tries = 0;; ++tries) {
        const int32_t ahead = int32_t(uint32_t(old >> 32) - e32);
        if (ahead > 0)
            return {-1, 0, 0};  // a later epoch is armed: this one is done
        if (ahead == 0) {
            // Every chunk already taken: leave without adding, so the 16-bit
            // count only grows past the limit by additions that raced.
            if ((uint32_t(old) & 0xFFFFu) >= (uint32_t(old >> 16) & 0xFFFFu))
                return {-1, 0, 0};
            break;
        }
        // Every failed CAS saw another worker arm the word or add to it.
        if (tries >= kMaxServeChunks) {
            report_error(error, kServeProtocol, l, r, old, epoch);
            return {-1, 0, 0};
        }
        const unsigned long long armed = (uint64_t(e32) << 32) | (uint64_t(chunks) << 16);
        const unsigned long long seen = atomicCAS(word, old, armed);
        if (seen == old)
            break;
        old = seen;
    }
    const unsigned long long v = atomicAdd(word, 1ull);
    const uint32_t at = uint32_t(v >> 32), limit = uint32_t(v >> 16) & 0xFFFFu, count = uint32_t(v) & 0xFFFFu;
    if (int32_t(at - e32) < 0) {
        report_error(error, kServeProtocol, l, r, v, epoch);  // the word went back
        return {-1, 0, 0};
    }
    if (count >= limit)
        return {-1, 0, 0};
    return {int32_t(count), at, limit};
}

// Stages the inbox entries of chunk `c` (row, output position) into shared
// memory; rows or positions out of bounds are reported and skipped.  Run by
// one warp.
__device__ __forceinline__ void stage_chunk(const ServeParams &s, const uint64_t *inbox, uint32_t c, uint32_t rows,
                                            uint32_t l, uint32_t r, uint32_t *s_row, uint32_t *s_pos) {
    const uint32_t lo = c * s.chunk_rows, n = min(lo + s.chunk_rows, rows) - lo;
#pragma unroll 4
    for (uint32_t i = threadIdx.x % 32; i < n; i += 32) {
        const uint64_t entry = __ldcg(reinterpret_cast<const unsigned long long *>(inbox) + lo + i);
        uint32_t row = uint32_t(entry);
        const uint32_t pos = uint32_t(entry >> 32);
        if (!(row < s.table_rows && pos < s.capacity)) {
            report_error(s.error, kPushBounds, l, r, entry, s.table_rows);
            row = kSkipRow;
        }
        s_row[i] = row;
        s_pos[i] = pos;
    }
}

// Counts one copied chunk of (r, l, epoch).  Its stores were issued before a
// CTA barrier that the calling thread passed, so one cumulative system-scope
// fence orders them before the count.  The worker whose count completes the
// epoch resets the finish word for epoch + 1 and releases done at the
// requester; the claim word is armed for epoch + 1 by the first worker that
// sees it published.
__device__ __forceinline__ void finish_chunk(const ServeParams &s, uint32_t r, uint32_t l, uint32_t slot,
                                             uint64_t epoch, uint32_t chunks) {
    fence_sc_sys();
    unsigned long long *fin = reinterpret_cast<unsigned long long *>(s.finish + slot);
    const unsigned long long prev = atomicAdd(fin, 1ull);
    if (uint32_t(prev >> 32) != uint32_t(epoch - 1))
        report_error(s.error, kServeProtocol, l, r, prev, epoch);
    if (uint32_t(prev) + 1 == chunks) {
        *reinterpret_cast<volatile unsigned long long *>(fin) = epoch << 32;
        fence_sc_sys();
        auto *done = reinterpret_cast<uint64_t *>(s.done_base[r]) + (uint64_t(l) * s.world + s.rank);
        st_release_sys_u64(done, epoch);
    }
}

// Whole-CTA worker: copies chunks of request (r, l, epoch) from this rank's
// table (HBM mirror or host shard) to the requester's output until none is
// left.  Returns true if it copied anything.  Every thread of the CTA must
// call it.
//
// Warp 0 is the control warp: while warps 1.. copy the current chunk, it
// counts the previously copied one (system-scope fence, finish count, done
// release), claims the next one and stages its entries in the other shared
// buffer.  A chunk boundary then costs one CTA barrier, so CTAs that reach
// their boundaries at the same time (claims by fetch-and-add let them start
// together) do not leave the link idle while each fences and claims.
__device__ bool serve_request(const ServeParams &s, uint32_t r, uint32_t l, uint64_t epoch, uint32_t rows) {
    __shared__ int32_t s_chunk[2];
    __shared__ uint32_t s_rows;
    __shared__ uint64_t s_epoch;
    __shared__ uint32_t s_row[2][kMaxServeChunkRows], s_pos[2][kMaxServeChunkRows];
    // Published requests are never empty (epochs advance only for non-empty
    // ones); a zero here must not arm the word with a limit of 0.
    if (s.out_base[r] == 0 || rows == 0)
        return false;
    // Callers run this back to back: no thread may still be reading the
    // previous call's shared words when thread 0 writes them below.
    __syncthreads();
    const uint32_t slot = r * s.layers + l;
    const uint64_t *inbox = s.inbox + uint64_t(slot) * s.capacity;
    uint8_t *out = reinterpret_cast<uint8_t *>(s.out_base[r]) + uint64_t(l) * s.capacity * s.row_bytes;
    const bool control = threadIdx.x < 32;
    // First claim: may arm the word, or land on a later (published) epoch.
    if (threadIdx.x == 0) {
        const Claim c = claim_chunk(s.claim + slot, epoch, chunk_count(rows, s.chunk_rows), s.error, l, r);
        int32_t chunk = c.chunk;
        if (chunk >= 0 && c.epoch32 != uint32_t(epoch)) {
            // A chunk of a later epoch; its header is published and cannot
            // move on before this chunk is finished.
            const uint64_t later = epoch + uint32_t(c.epoch32 - uint32_t(epoch));
            const MailboxHeader *h = s.headers + slot;
            const uint64_t ready = ld_acquire_sys_u64(&h->ready);
            const uint32_t later_rows = *reinterpret_cast<const volatile uint32_t *>(&h->rows);
            if (ready != later) {
                report_error(s.error, kServeProtocol, l, r, ready, later);
                chunk = -1;
            } else {
                epoch = later;
                rows = later_rows;
            }
        }
        if (chunk >= 0 && chunk_count(rows, s.chunk_rows) != c.limit) {
            report_error(s.error, kServeProtocol, l, r, rows, c.limit);
            chunk = -1;
        }
        s_chunk[0] = chunk;
        s_epoch = epoch;
        s_rows = rows;
    }
    __syncthreads();
    int32_t c = s_chunk[0];
    epoch = s_epoch;
    rows = s_rows;
    if (c < 0)
        return false;
    const uint32_t chunks = chunk_count(rows, s.chunk_rows);
    if (control)
        stage_chunk(s, inbox, uint32_t(c), rows, l, r, s_row[0], s_pos[0]);
    __syncthreads();

    constexpr uint32_t kCopyThreads = kPushThreads - 32;
    constexpr uint32_t kRowsPerStep = kCopyThreads / kPushLanesPerRow;
    constexpr int kUnroll = 8;  // 112 rows of a chunk in flight per CTA
    const uint32_t sub = (threadIdx.x - 32) / kPushLanesPerRow, vlane = threadIdx.x % kPushLanesPerRow;
    const uint32_t vectors = s.row_bytes / 16;
    uint32_t b = 0;
    bool copied_one = false;
    while (true) {
        if (control) {
            if (threadIdx.x == 0) {
                if (copied_one)
                    finish_chunk(s, r, l, slot, epoch, chunks);
                // The chunk in hand is unfinished, so the word is still armed
                // for this epoch: the addition cannot land on another one.
                const unsigned long long v = atomicAdd(reinterpret_cast<unsigned long long *>(s.claim + slot), 1ull);
                const uint32_t limit = uint32_t(v >> 16) & 0xFFFFu, count = uint32_t(v) & 0xFFFFu;
                int32_t next = count < limit ? int32_t(count) : -1;
                if (uint32_t(v >> 32) != uint32_t(epoch)) {
                    report_error(s.error, kServeProtocol, l, r, v, epoch);
                    next = -1;
                }
                s_chunk[b ^ 1] = next;
            }
            __syncwarp();
            const int32_t next = *reinterpret_cast<volatile int32_t *>(&s_chunk[b ^ 1]);
            if (next >= 0)
                stage_chunk(s, inbox, uint32_t(next), rows, l, r, s_row[b ^ 1], s_pos[b ^ 1]);
        } else {
            const uint32_t lo = uint32_t(c) * s.chunk_rows, n = min(lo + s.chunk_rows, rows) - lo;
            const uint32_t *rows_in = s_row[b], *pos_in = s_pos[b];
            for (uint32_t base = 0; base < n; base += kRowsPerStep * kUnroll) {
                const uint8_t *src[kUnroll];
                uint8_t *dst[kUnroll];
#pragma unroll
                for (int u = 0; u < kUnroll; ++u) {
                    const uint32_t i = base + u * kRowsPerStep + sub;
                    src[u] = nullptr;
                    dst[u] = nullptr;
                    if (i < n && rows_in[i] != kSkipRow) {
                        src[u] = s.table + uint64_t(rows_in[i]) * s.row_bytes;
                        dst[u] = out + uint64_t(pos_in[i]) * s.row_bytes;
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
        }
        // Chunk c's stores are issued and the next chunk is staged.
        __syncthreads();
        copied_one = true;
        const int32_t next = s_chunk[b ^ 1];
        if (next < 0)
            break;
        c = next;
        b ^= 1;
    }
    if (threadIdx.x == 0)
        finish_chunk(s, r, l, slot, epoch, chunks);
    return true;
}

// Launched by the owner service for the requests it found in the mailbox.
// Requests another worker already finished are skipped by the claim.
__global__ void __launch_bounds__(kPushThreads) push_kernel(const __grid_constant__ PushParams p) {
    // CTA b starts at task b (mod the count): the CTAs spread over the
    // requesters at once instead of all storing into one requester's links.
    for (uint32_t t = 0; t < p.num_tasks; ++t) {
        const PushTask &task = p.tasks[(t + blockIdx.x) % p.num_tasks];
        serve_request(p.s, task.requester, task.layer, task.epoch, task.rows);
    }
}

// Copies this rank's mailbox (host memory) into the device board; warp 0 of
// block 0 only, so the polling costs one PCIe read per slot per pass.
__device__ __forceinline__ void refresh_board(const ServeParams &s) {
    const uint32_t slots = s.world * s.layers;
    for (uint32_t i = threadIdx.x; i < slots; i += 32) {
        const uint32_t r = i / s.layers;
        if (!((s.serve_mask >> r) & 1ull))
            continue;
        const MailboxHeader *h = s.headers + i;
        const uint64_t epoch = ld_acquire_sys_u64(&h->ready);
        if (epoch == 0)
            continue;
        const uint32_t rows = *reinterpret_cast<const volatile uint32_t *>(&h->rows);
        *reinterpret_cast<volatile unsigned long long *>(s.board + i) = (epoch << 32) | rows;
    }
}

// Hook kernel: waits until every host-route owner of `layer` that received a
// request has released the expected epoch.  While it waits, all its CTAs serve
// requests addressed to this rank, so two ranks whose hooks wait on each other
// always make progress without depending on another kernel being scheduled.
__global__ void __launch_bounds__(kPushThreads) hook_kernel(const __grid_constant__ HookParams p) {
    __shared__ int32_t s_state;
    __shared__ uint64_t s_task;
    const ServeParams &s = p.s;
    const uint64_t start = global_timer_ns();
    const uint64_t max_polls = p.timeout_ns / 16 + 1024;  // holds even if the timer stalled
    uint64_t polls = 0;
    uint32_t backoff = 64;
    while (true) {
        if (threadIdx.x == 0) {
            int32_t state = 1;  // 1: all done, 0: waiting, 2: timed out
            ++polls;
            for (uint32_t o = 0; o < s.world; ++o) {
                const uint32_t slot = p.layer * s.world + o;
                if (p.totals[slot] == 0)
                    continue;
                const uint64_t expected = p.epochs[slot];
                const uint64_t seen = ld_acquire_sys_u64(p.done + slot);
                if (seen != expected) {
                    state = 0;
                    if (global_timer_ns() - start > p.timeout_ns || polls > max_polls) {
                        report_error(s.error, kWaitTimeout, p.layer, o, seen, expected);
                        state = 2;
                    }
                    break;
                }
            }
            s_state = state;
        }
        __syncthreads();
        if (s_state != 0)
            return;
        __syncthreads();
        bool worked = false;
        if (p.serve) {
            if (blockIdx.x == 0 && threadIdx.x < 32)
                refresh_board(s);
            __syncthreads();
            const uint32_t slots = s.world * s.layers;
            // CTA b starts at slot b (mod the slot count), so an owner's CTAs
            // serve every requester at once rather than one after another.
            for (uint32_t j = 0; j < slots; ++j) {
                const uint32_t i = (j + blockIdx.x) % slots;
                if (threadIdx.x == 0) {
                    uint64_t task = 0;
                    if ((s.serve_mask >> (i / s.layers)) & 1ull) {
                        const uint64_t b = *reinterpret_cast<const volatile unsigned long long *>(s.board + i);
                        const uint64_t epoch = b >> 32;
                        const uint32_t rows = uint32_t(b);
                        // Worth serving: the word is still armed for an earlier
                        // epoch (this one needs arming) or has chunks left.
                        const uint64_t armed = *reinterpret_cast<const volatile unsigned long long *>(s.claim + i);
                        const int32_t ahead = int32_t(uint32_t(armed >> 32) - uint32_t(epoch));
                        const uint32_t limit = uint32_t(armed >> 16) & 0xFFFFu, count = uint32_t(armed) & 0xFFFFu;
                        if (epoch != 0 && rows != 0 && (ahead < 0 || (ahead == 0 && count < limit)))
                            task = b;
                    }
                    s_task = task;
                }
                __syncthreads();
                const uint64_t task = s_task;
                __syncthreads();
                if (task != 0)
                    worked |= serve_request(s, i / s.layers, i % s.layers, task >> 32, uint32_t(task));
            }
        }
        if (!worked) {
            __nanosleep(backoff);
            backoff = backoff < 2048 ? backoff * 2 : 2048;
        } else {
            backoff = 64;
        }
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
    if (p.s.chunk_rows == 0 || p.s.chunk_rows > kMaxServeChunkRows)
        return cudaErrorInvalidValue;  // a chunk's entries are staged in shared memory
    push_kernel<<<blocks, kPushThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_hook_wait(const HookParams &p, int serve_ctas, cudaStream_t stream) {
    if (p.serve && (p.s.chunk_rows == 0 || p.s.chunk_rows > kMaxServeChunkRows))
        return cudaErrorInvalidValue;  // a chunk's entries are staged in shared memory
    // Serving needs enough CTAs to keep reads of the table in flight (16 keep
    // PCIe reads of a pinned shard at its envelope; reads of an HBM mirror
    // want one per SM); a rank that serves nobody only waits.
    hook_kernel<<<p.serve ? (serve_ctas > 0 ? serve_ctas : 16) : 1, kPushThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_wait_probe(const uint64_t *flag, uint64_t expected, uint64_t timeout_ns, ErrorSink error,
                              cudaStream_t stream) {
    wait_probe_kernel<<<1, 32, 0, stream>>>(flag, expected, timeout_ns, error);
    return cudaGetLastError();
}

} // namespace engram
