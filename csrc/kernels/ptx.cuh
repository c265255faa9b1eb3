// Device primitives for the Engram data plane (sm_100a).
//
// Everything here is data movement and cross-GPU ordering; there is no math.
// Ordering protocol used by every producer/consumer pair in this project:
//   producer: data stores (local or peer) -> fence.sc.sys -> st.release.sys flag
//   consumer: ld.acquire.sys flag (bounded poll) -> data loads
// Waits are bounded by the global nanosecond timer and report through an error
// record instead of trapping, so a missing peer never hangs or faults the GPU.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "params.h"

namespace engram {

struct alignas(16) Vec16 {
    uint32_t x, y, z, w;
};

// 32-byte vector (sm_100 256-bit loads and stores).
struct alignas(32) Vec32 {
    uint32_t v[8];
};

// 16-byte read-only load that bypasses L1 allocation; the table rows are read
// once per fetch and must not evict the caller's working set from L1.
__device__ __forceinline__ Vec16 ld_nc_na_v4(const void *ptr) {
    Vec16 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(ptr));
    return v;
}

// 32-byte read-only load without L1 allocation: one request per 32-byte
// sector.  Over NVLink, 8 lanes x 32 B per 256-byte row moved random rows
// ~5% faster than 16 lanes x 16 B (benchmarks/peer_bandwidth.py, rows family).
__device__ __forceinline__ Vec32 ld_nc_na_v8(const void *ptr) {
    Vec32 r;
    asm volatile("ld.global.nc.L1::no_allocate.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r.v[0]), "=r"(r.v[1]), "=r"(r.v[2]), "=r"(r.v[3]), "=r"(r.v[4]), "=r"(r.v[5]), "=r"(r.v[6]),
                   "=r"(r.v[7])
                 : "l"(ptr));
    return r;
}

__device__ __forceinline__ void st_v8(void *ptr, const Vec32 &r) {
    asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(ptr), "r"(r.v[0]), "r"(r.v[1]),
                 "r"(r.v[2]), "r"(r.v[3]), "r"(r.v[4]), "r"(r.v[5]), "r"(r.v[6]), "r"(r.v[7])
                 : "memory");
}

// Width-generic row-vector helpers for the gather kernels.
template <int BYTES> struct RowVec;
template <> struct RowVec<16> {
    using T = Vec16;
    static __device__ __forceinline__ T zero() { return Vec16{0, 0, 0, 0}; }
    static __device__ __forceinline__ T load(const void *p) { return ld_nc_na_v4(p); }
    static __device__ __forceinline__ void store(void *p, const T &v) {
        asm volatile("st.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                     : "memory");
    }
};
template <> struct RowVec<32> {
    using T = Vec32;
    static __device__ __forceinline__ T zero() { return Vec32{{0, 0, 0, 0, 0, 0, 0, 0}}; }
    static __device__ __forceinline__ T load(const void *p) { return ld_nc_na_v8(p); }
    static __device__ __forceinline__ void store(void *p, const T &v) { st_v8(p, v); }
};

// 32-byte read-only load with the 256-byte L2 prefetch-size hint: the L2
// fetches the whole 256-byte block the sector belongs to.  For 256-byte rows
// the first lane's access brings the row in; over NVLink it moved random rows
// 2% faster in the probe (517.8 vs 507.5 GB/s per GPU at 8 GPUs).
__device__ __forceinline__ Vec32 ld_nc_na_l2_256_v8(const void *ptr) {
    Vec32 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r.v[0]), "=r"(r.v[1]), "=r"(r.v[2]), "=r"(r.v[3]), "=r"(r.v[4]), "=r"(r.v[5]), "=r"(r.v[6]),
                   "=r"(r.v[7])
                 : "l"(ptr));
    return r;
}

// RowVec<32> whose loads carry the 256-byte L2 prefetch-size hint.
struct RowVec32L2 : RowVec<32> {
    static __device__ __forceinline__ T load(const void *p) { return ld_nc_na_l2_256_v8(p); }
};

// Plain 16-byte load for memory another agent may be writing concurrently
// (host shards under a rewrite are quiesced by write(), so .nc is safe there
// too; this variant is kept for the inbox, which peers fill).
__device__ __forceinline__ Vec16 ld_v4(const void *ptr) {
    Vec16 v;
    asm volatile("ld.global.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(ptr));
    return v;
}

// 16-byte load cached in L2 only: never a stale L1 line of memory that a peer
// rewrites while this kernel runs.
__device__ __forceinline__ Vec16 ld_cg_v4(const void *ptr) {
    Vec16 v;
    asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(ptr));
    return v;
}

__device__ __forceinline__ void st_v4(void *ptr, const Vec16 &v) {
    asm volatile("st.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(ptr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

// Streaming store: the output is consumed by a later kernel, keep L1 clean.
__device__ __forceinline__ void st_na_v4(void *ptr, const Vec16 &v) {
    asm volatile("st.global.L1::no_allocate.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(ptr), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}

__device__ __forceinline__ uint64_t ld_acquire_sys_u64(const void *ptr) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(ptr) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys_u64(void *ptr, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(ptr), "l"(v) : "memory");
}

__device__ __forceinline__ void st_relaxed_sys_u32(void *ptr, uint32_t v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_sc_sys() { asm volatile("fence.sc.sys;" ::: "memory"); }

__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// Device-scope acq_rel fetch-add on a 32-bit counter (last-block-done pattern).
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t *ptr, uint32_t v) {
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(ptr), "r"(v) : "memory");
    return old;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void st_relaxed_sys_u64(void *ptr, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(ptr), "l"(v) : "memory");
}

__device__ __forceinline__ void st_release_sys_u32(void *ptr, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}

// First reporter wins (device-scope CAS); it mirrors the record to the host
// copy with the status written last.  Later reports only bump the count.
__device__ __forceinline__ void report_error(const ErrorSink &sink, uint32_t code, uint32_t layer, uint32_t owner,
                                             uint64_t observed, uint64_t expected) {
    ErrorRecord *dev = sink.dev;
    if (dev == nullptr)
        return;
    const uint32_t count = atomicAdd(&dev->count, 1u) + 1;
    if (atomicCAS(&dev->status, 0u, code) != 0u) {
        if (sink.host != nullptr)
            st_relaxed_sys_u32(&sink.host->count, count);
        return;
    }
    dev->layer = layer;
    dev->owner = owner;
    dev->observed = observed;
    dev->expected = expected;
    if (ErrorRecord *host = sink.host) {
        st_relaxed_sys_u32(&host->layer, layer);
        st_relaxed_sys_u32(&host->owner, owner);
        st_relaxed_sys_u32(&host->count, count);
        st_relaxed_sys_u64(&host->observed, observed);
        st_relaxed_sys_u64(&host->expected, expected);
        st_release_sys_u32(&host->status, code);
    }
}

// ---------------------------------------------------------------- mbarrier / bulk copy
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Make barrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
                 : "=r"(ok)
                 : "r"(smem_addr(bar)), "r"(parity)
                 : "memory");
    return ok != 0;
}

// Bounded wait for a barrier phase; false after `timeout_ns` (or as many
// polls, a cap that holds even if the timer stalled).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint64_t timeout_ns) {
    if (mbar_try_wait(bar, parity))
        return true;
    const uint64_t start = global_timer_ns();
    uint64_t polls = 0;
    while (!mbar_try_wait(bar, parity))
        if (global_timer_ns() - start > timeout_ns || ++polls > timeout_ns)
            return false;
    return true;
}

// Non-multicast bulk copy global -> this CTA's shared memory, completing
// `bytes` of transaction count on `bar`.  Source and size are 16-byte multiples.
__device__ __forceinline__ void bulk_load(void *dst_smem, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst_smem)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

// 4-byte asynchronous global -> shared copy (completes with cp.async.wait_group).
__device__ __forceinline__ void cp_async_4(void *dst_smem, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst_smem)), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ Vec16 ld_shared_v4(const void *p) {
    Vec16 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(smem_addr(p)));
    return v;
}

// Epoch of the fetch in flight for request deduplication (dedup.cu).
__device__ __forceinline__ uint32_t dedup_epoch(const uint32_t *state) {
    const uint32_t e = (state[0] + 1) & ((1u << 28) - 1);
    return e == 0 ? 1 : e;
}

// True if `item` repeats an earlier request of this fetch (its row arrives by
// a local copy from the first occurrence instead of the gather).
__device__ __forceinline__ bool dedup_duplicate(const GatherParams &p, uint32_t item, uint32_t epoch) {
    const uint32_t slot = __ldcg(p.dedup_slots + item);
    if (slot == kDedupNone)
        return false;
    const uint64_t v = __ldcg(reinterpret_cast<const unsigned long long *>(p.dedup_vals) + slot);
    return (v >> 32) == epoch && (0xFFFFFFFFu - uint32_t(v)) != item;
}

// Poll `flag` until it equals `expected` or `timeout_ns` passes.  Returns the
// last value read.  Never traps; the caller reports a timeout.  An iteration
// cap (each poll sleeps at least ~8 ns) bounds the loop even if the timer
// stalled.
__device__ __forceinline__ uint64_t wait_flag_eq(const void *flag, uint64_t expected, uint64_t timeout_ns,
                                                 bool *timed_out) {
    const uint64_t start = global_timer_ns();
    const uint64_t max_polls = timeout_ns / 8 + 1024;
    uint64_t polls = 0;
    uint32_t backoff = 32;
    uint64_t value = ld_acquire_sys_u64(flag);
    while (value != expected) {
        if (global_timer_ns() - start > timeout_ns || ++polls > max_polls) {
            *timed_out = true;
            return value;
        }
        __nanosleep(backoff);
        backoff = backoff < 1024 ? backoff * 2 : 1024;
        value = ld_acquire_sys_u64(flag);
    }
    *timed_out = false;
    return value;
}

} // namespace engram
