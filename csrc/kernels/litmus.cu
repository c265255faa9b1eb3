// Message-passing litmus test for the flag protocol of the host route (sm_100a).
//
// The owner push and the hook rely on one ordering pattern:
//   producer CTAs: weak 16-byte stores of the data (to a peer GPU's memory)
//                  -> __syncthreads -> thread 0: fence.sc.sys, atomic arrival
//                  -> the last CTA: st.release.sys of the flag (in the peer's memory)
//   consumer:      thread 0 polls the flag with ld.acquire.sys -> __syncthreads
//                  -> every thread reads the data (L2-only loads as the serving
//                  path does, or weak loads to test the memory model itself).
// This kernel runs that pattern for many epochs and counts every word a
// consumer reads that is not the producer's value for the epoch it acquired.
// The consumer acknowledges each epoch the same way, so the producer never
// overwrites data that is still being checked.  Every wait is bounded: on a
// timeout the side records where it gave up and returns (no trap).
//
// Roles: on two GPUs, one launch per GPU (producer writes the peer's data and
// flag through its mapping; consumer acknowledges into the producer's
// memory).  On one GPU, one cooperative launch runs both roles in disjoint
// CTAs over local memory, so no kernel waits on another launch.
// No reference counterpart: the reference relies on its protocol without a test.
#include "params.h"
#include "ptx.cuh"

namespace engram {

namespace {

constexpr int kLitmusThreads = 256;

__device__ __forceinline__ uint32_t pattern(uint32_t epoch, uint32_t i) {
    uint32_t h = epoch * 0x9E3779B9u ^ (i + 0x7F4A7C15u) * 0x85EBCA6Bu;
    h ^= h >> 15;
    h *= 0x2C1B3C6Du;
    h ^= h >> 12;
    return h;
}

__device__ void record(LitmusResult *r, uint32_t status, uint32_t epoch, uint64_t observed) {
    if (atomicCAS(&r->status, 0u, status) == 0u) {
        r->epoch = epoch;
        r->observed = observed;
    }
}

__device__ void produce(const LitmusParams &p, uint32_t cta, uint32_t ctas) {
    __shared__ int s_abort;
    for (uint32_t e = 1; e <= p.epochs; ++e) {
        if (threadIdx.x == 0) {
            s_abort = 0;
            bool timed_out = false;
            const uint64_t seen = wait_flag_eq(p.ack_local, e - 1, p.timeout_ns, &timed_out);
            if (timed_out) {
                record(p.result, kLitmusProducerTimeout, e, seen);
                s_abort = 1;
            }
        }
        __syncthreads();
        if (s_abort)
            return;
        for (uint32_t i = (cta * blockDim.x + threadIdx.x) * 4; i < p.words; i += ctas * blockDim.x * 4) {
            const Vec16 v{pattern(e, i), pattern(e, i + 1), pattern(e, i + 2), pattern(e, i + 3)};
            st_v4(p.data_remote + i, v);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            fence_sc_sys();
            if (atom_add_acq_rel_gpu(p.prod_count, 1u) == e * ctas - 1)
                st_release_sys_u64(p.flag_remote, e);
        }
    }
}

__device__ void consume(const LitmusParams &p, uint32_t cta, uint32_t ctas) {
    __shared__ int s_abort;
    __shared__ uint32_t s_bad;
    for (uint32_t e = 1; e <= p.epochs; ++e) {
        if (threadIdx.x == 0) {
            s_abort = 0;
            s_bad = 0;
            bool timed_out = false;
            const uint64_t seen = wait_flag_eq(p.flag_local, e, p.timeout_ns, &timed_out);
            if (timed_out) {
                record(p.result, kLitmusConsumerTimeout, e, seen);
                s_abort = 1;
            }
        }
        __syncthreads();
        if (s_abort)
            return;
        uint32_t bad = 0;
        for (uint32_t i = (cta * blockDim.x + threadIdx.x) * 4; i < p.words; i += ctas * blockDim.x * 4) {
            // L2-only loads are what the serving path uses; weak loads test
            // the memory model's acquire-then-barrier guarantee itself.
            const Vec16 v = p.weak_loads ? ld_v4(p.data_local + i) : ld_cg_v4(p.data_local + i);
            bad += (v.x != pattern(e, i)) + (v.y != pattern(e, i + 1)) + (v.z != pattern(e, i + 2)) +
                   (v.w != pattern(e, i + 3));
        }
        if (bad)
            atomicAdd(&s_bad, bad);
        __syncthreads();
        if (threadIdx.x == 0) {
            if (s_bad) {
                atomicAdd(&p.result->mismatches, s_bad);
                atomicMin(&p.result->first_bad_epoch, e);
            }
            fence_sc_sys();
            if (atom_add_acq_rel_gpu(p.cons_count, 1u) == e * ctas - 1) {
                st_release_sys_u64(p.ack_remote, e);
                p.result->epochs_done = e;
            }
        }
    }
}

__global__ void __launch_bounds__(kLitmusThreads) litmus_kernel(const __grid_constant__ LitmusParams p) {
    if (p.role == kLitmusProducer) {
        produce(p, blockIdx.x, gridDim.x);
    } else if (p.role == kLitmusConsumer) {
        consume(p, blockIdx.x, gridDim.x);
    } else {
        const uint32_t half = gridDim.x / 2;
        if (blockIdx.x < half)
            produce(p, blockIdx.x, half);
        else
            consume(p, blockIdx.x - half, gridDim.x - half);
    }
}

} // namespace

cudaError_t launch_litmus(const LitmusParams &p, uint32_t ctas, cudaStream_t stream) {
    // Cooperative: every CTA is resident at once, or the launch fails; the
    // CTAs of one role wait on the other role's progress.
    const uint32_t grid = p.role == kLitmusBoth ? 2 * ctas : ctas;
    void *args[] = {const_cast<LitmusParams *>(&p)};
    return cudaLaunchCooperativeKernel(reinterpret_cast<const void *>(litmus_kernel), dim3(grid),
                                       dim3(kLitmusThreads), args, 0, stream);
}

} // namespace engram
