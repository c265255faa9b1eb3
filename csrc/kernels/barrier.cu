// Bounded device barrier over NVLink (sm_100a).
//
// Parity: the reference's NVLink barrier (deepep/deep_ep/include/deep_ep/comm/
// barrier.cuh:88-131, launched by deepep/csrc/kernels/comm/barrier.hpp:17-54),
// which adds to a phase slot in every peer and polls its own slots, trapping
// on timeout.  Here one warp per GPU runs it on the caller's stream:
//   * each rank keeps a monotonically increasing barrier count in its arena
//     (device memory, so CUDA Graph replays advance it too);
//   * lane p stores the new count into slot[rank] of peer p's arena with
//     st.release.sys (after a system-scope fence, so every write the stream
//     made before the barrier is visible to peers that pass it);
//   * lane p then polls this rank's slot[p] with ld.acquire.sys until it
//     reaches the count.  A rank that is one barrier ahead has already stored
//     a larger count, so ">=" keeps ranks that run back-to-back barriers
//     correct without resetting anything;
//   * the wait is bounded by the global timer and a poll count; on expiry the
//     warp records the owner and the counts in the error record and returns.
//     Nothing traps.  After a timeout the ranks' counts disagree, so the
//     error stays latched until the buffer is destroyed.
#include "params.h"
#include "ptx.cuh"

namespace engram {

namespace {

__global__ void __launch_bounds__(32) barrier_kernel(const __grid_constant__ BarrierParams p) {
    const uint32_t lane = threadIdx.x;
    uint64_t count = 0;
    if (lane == 0) {
        count = *p.count + 1;
        *p.count = count;
    }
    count = __shfl_sync(0xFFFFFFFFu, count, 0);
    fence_sc_sys();
    for (uint32_t peer = lane; peer < p.world; peer += 32)
        st_release_sys_u64(reinterpret_cast<void *>(p.peer_slot[peer]), count);
    const uint64_t start = global_timer_ns();
    const uint64_t max_polls = p.timeout_ns / 16 + 1024;  // holds even if the timer stalled
    for (uint32_t peer = lane; peer < p.world; peer += 32) {
        uint64_t polls = 0;
        uint32_t backoff = 16;
        uint64_t seen = ld_acquire_sys_u64(p.slots + peer);
        while (seen < count) {
            if (global_timer_ns() - start > p.timeout_ns || ++polls > max_polls) {
                report_error(p.error, kBarrierTimeout, 0, peer, seen, count);
                break;
            }
            __nanosleep(backoff);
            backoff = backoff < 256 ? backoff * 2 : 256;
            seen = ld_acquire_sys_u64(p.slots + peer);
        }
    }
    __syncwarp();
}

} // namespace

cudaError_t launch_barrier(const BarrierParams &p, cudaStream_t stream) {
    barrier_kernel<<<1, 32, 0, stream>>>(p);
    return cudaGetLastError();
}

} // namespace engram
