// Launch parameters of the Engram kernels.  Plain structs passed by value, so
// CUDA Graph capture records them in the kernel node and replays never need a
// device-side metadata table.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace engram {

constexpr int kMaxRanks = 64;
constexpr int kMaxLayers = 32;
constexpr int kHeaderBytes = 64;
constexpr int kMaxPushTasks = 64;
// Largest claimable chunk of an owner-push request; the serving code stages a
// chunk's inbox entries in shared memory.
constexpr uint32_t kMaxServeChunkRows = 512;
// Largest chunk count of one request: the claim word keeps the limit and the
// claimed count in 16 bits each, with headroom above the limit for additions
// that find every chunk taken.
constexpr uint32_t kMaxServeChunks = 1u << 15;

// Error record shared with the host through mapped pinned memory.  The first
// failing thread wins; later failures only bump the count.
struct ErrorRecord {
    uint32_t status;   // 0 = healthy, else one of ErrorCode
    uint32_t layer;
    uint32_t owner;
    uint32_t count;
    uint64_t observed;
    uint64_t expected;
};

// Where kernels report errors: atomics go to a device-resident record (atomics
// on mapped host memory are not guaranteed over PCIe); the winning thread then
// mirrors its report into host-mapped memory with plain system-scope stores,
// status last, so the host can poll it without synchronising the stream.
struct ErrorSink {
    ErrorRecord *dev;
    ErrorRecord *host;
};

enum ErrorCode : uint32_t {
    kOk = 0,
    kWaitTimeout = 1,      // hook gave up waiting for an owner's done flag
    kIndexOutOfRange = 2,  // a request named a row beyond the global vocabulary
    kInboxOverflow = 3,    // a request list exceeded the inbox slot
    kPushBounds = 4,       // an owner got a row id or position out of bounds
    kPipelineTimeout = 5,  // a shared-memory pipeline barrier never completed
    kBarrierTimeout = 6,   // a peer never reached the device barrier
    kServeProtocol = 7,    // a serving claim disagreed with the mailbox header
};

constexpr uint32_t kGatherBulk = 0;  // TMA bulk-copy ring (opt-in)
constexpr uint32_t kGatherSimt = 1;  // per-thread 16- or 32-byte vector loads (default)


// Mailbox header written by a requester's GPU into the owner's host shard and
// polled by the owner's service thread.  One slot per [requester][layer].
struct alignas(64) MailboxHeader {
    uint64_t ready;     // request epoch, published last with st.release.sys
    uint32_t rows;      // number of (row, position) entries in the inbox slot
    uint32_t layer;
    uint32_t requester;
    uint32_t channels;  // push CTAs the requester asks for (its num_qps)
    uint32_t reserved[10];
};
static_assert(sizeof(MailboxHeader) == kHeaderBytes, "mailbox header ABI");

// Per-layer geometry shared by all kernels.
struct LayerTable {
    uint32_t entries[kMaxLayers];      // rows per rank (n_l)
    uint32_t table_bases[kMaxLayers];  // first local row of layer l in a shard
    uint32_t sf_bases[kMaxLayers];     // first float of layer l in a scale table
    // Hot-prefix replication: global ids [0, hot_rows[l]) of layer l are read
    // from this rank's replica (row hot_bases[l] + x), never from their owner.
    uint32_t hot_rows[kMaxLayers];
    uint32_t hot_bases[kMaxLayers];
};

// Requester-side gather: every row with a direct source (the owner's HBM
// mirror through NVLink, this rank's own shard, or this rank's replica of the
// hot id prefix) is copied into the output; padding rows become zero; FP8
// scales are gathered for all rows.  `indices` may be a device pointer or the
// device mapping of pinned host memory.
struct GatherParams {
    const int32_t *indices;       // [layers][rows]
    uint8_t *output;              // [layers][capacity][row_bytes]
    float *sf_output;             // layer l at sf_output + l * sf_layer_stride
    ErrorSink error;
    LayerTable layer;
    uint64_t direct_base[kMaxRanks];  // per owner; 0 = rows arrive by owner push
    uint64_t sf_base[kMaxRanks];      // per scale shard
    uint64_t hot_base;                // local replica of the hot prefixes (LayerTable::hot_rows)
    uint32_t layers, rows, ept;
    uint32_t capacity, row_bytes, world, packs;
    uint32_t sf_shard_div;        // global row -> shard: x / (n * sf_shard_div)
    uint32_t sf_token_stride, sf_hidden_stride, sf_layer_stride;  // either scale layout
    uint32_t variant;             // kGatherBulk or kGatherSimt
    uint32_t ctas_per_sm;         // SIMT grid cap per SM (0 = default 2)
    uint32_t unroll;              // SIMT row-steps in flight for 256-byte rows (0 = default)
    uint32_t strided;             // SIMT: 1 = warps stride over 32-row groups, 0 = equal contiguous ranges
    uint32_t vector_bytes;        // SIMT: 32 = 256-bit loads and stores where the row size allows, else 16
    uint32_t l2_prefetch;         // SIMT, 32-byte loads of rows up to 512 B: add the 256-byte L2 prefetch-size hint
    // Request deduplication (see DedupParams): when `dedup` is set, an item whose
    // slot's elected first occurrence is another item is skipped here and
    // copied locally by the expand kernel afterwards.
    uint32_t dedup;
    const uint32_t *dedup_slots;  // [layers * rows] table slot per item, kDedupNone if not deduplicated
    const uint64_t *dedup_vals;   // [table] (epoch << 32) | ~first_item
    const uint32_t *dedup_state;  // [0] epoch of the previous fetch
};

constexpr uint32_t kDedupNone = 0xFFFFFFFFu;

// Per-fetch request deduplication for direct-route rows.  keys/vals form an
// open-addressing table of `table_mask + 1` slots that is never cleared:
// keys carry the fetch epoch in bits 36-63 (layer in 31-35, row id in 0-30),
// so entries of older fetches read as empty.  vals hold (epoch << 32) |
// (0xFFFFFFFF - item) and are combined with atomicMax, which elects the
// smallest item of the current epoch as the key's first occurrence.
struct DedupParams {
    const int32_t *indices;
    uint64_t *keys;
    uint64_t *vals;
    uint32_t *slots;              // [layers * rows]
    uint32_t *state;              // [0] last epoch, [1] uniques, [2] items, [3] arrivals
    uint32_t *host_stats;         // host-mapped: [0] uniques, [1] items, [2] epoch of the last finished fetch
    uint8_t *output;
    LayerTable layer;
    uint64_t direct_base[kMaxRanks];
    uint32_t layers, rows, world, table_mask, capacity, row_bytes;
};

// Requester-side dispatch for host-route owners: append (row, position) pairs
// into each owner's inbox slot through peer stores, then the last CTA of each
// layer publishes the per-owner mailbox headers.
struct DispatchParams {
    const int32_t *indices;
    uint32_t *cursors;            // [layers][world] scratch, zero between fetches
    uint32_t *layer_arrivals;     // [layers]
    uint32_t *totals;             // [layers][world] rows requested this fetch
    uint64_t *epochs;             // [layers][world] last published epoch
    ErrorSink error;
    LayerTable layer;
    uint64_t inbox_base[kMaxRanks];   // owner arena inbox (peer mapping), 0 if direct
    uint64_t header_base[kMaxRanks];  // owner host-shard header region (mapping)
    uint32_t layers, rows, capacity, world, rank, channels;
    uint32_t tile_rows;
};

struct PushTask {
    uint32_t requester, layer, rows, channels;
    uint64_t epoch;
};

// Owner-side serving state shared by the push kernel (launched by the owner
// service) and the hook kernel (which serves inbound requests while it waits).
// A request (requester r, layer l, epoch e) is split into chunks of
// `chunk_rows` rows.  claim[r][l] holds (armed epoch << 32) | (chunk limit <<
// 16) | chunks claimed: a worker that knows epoch e is published and finds the
// word armed for an earlier epoch arms it for e by CAS; every claim is then one
// fetch-and-add.  An addition that lands after the word was armed for a later
// (necessarily published) epoch claims a chunk of that epoch, which the worker
// serves with the rows from the mailbox header.  finish[r][l] holds
// ((e - 1) << 32) | chunks finished; the worker that finishes the last chunk
// resets it for e + 1 and only then releases done = e at the requester, so a
// request is executed exactly once whoever runs it.
struct ServeParams {
    const uint8_t *table;             // this rank's HBM mirror if it keeps one, else its host shard (mapped)
    const uint64_t *inbox;            // this rank's inbox [world][layers][capacity]
    uint64_t *claim;                  // [world][layers]
    uint64_t *finish;                 // [world][layers]
    uint64_t *board;                  // [world][layers] (epoch << 32) | rows seen in the mailbox
    const MailboxHeader *headers;     // this rank's mailbox headers (host memory, device-visible)
    ErrorSink error;
    uint64_t out_base[kMaxRanks];     // requester arena output region (mapping)
    uint64_t done_base[kMaxRanks];    // requester arena done region (mapping)
    uint64_t serve_mask;              // bit r: requester r reaches me through the host route
    uint32_t layers, world, rank, capacity, row_bytes, chunk_rows;
    uint64_t table_rows;
};

// Owner-side push for the requests the owner service found.
struct PushParams {
    ServeParams s;
    PushTask tasks[kMaxPushTasks];
    uint32_t num_tasks;
};

// Hook-side wait for one layer: every host-route owner that received a
// non-empty request must publish the matching epoch in done[layer][owner].
// While waiting, the kernel also serves requests addressed to this rank.
struct HookParams {
    ServeParams s;
    const uint32_t *totals;
    const uint64_t *epochs;
    const uint64_t *done;             // this rank's done region [layers][world]
    uint32_t layer, serve;
    uint64_t timeout_ns;
};

// Bounded device barrier over NVLink (barrier.cu): one warp per GPU.
struct BarrierParams {
    uint64_t *count;                  // this rank's barrier count (arena scratch)
    const uint64_t *slots;            // this rank's arrival slots [world]; peer p writes slot p
    uint64_t peer_slot[kMaxRanks];    // address of slot[rank] in each rank's arena (own included)
    ErrorSink error;
    uint32_t world, rank;
    uint64_t timeout_ns;
};

// Host launchers (defined in the .cu files).
cudaError_t launch_gather(const GatherParams &p, int num_sms, cudaStream_t stream);
cudaError_t launch_dispatch(const DispatchParams &p, cudaStream_t stream);
cudaError_t launch_push(const PushParams &p, int blocks, cudaStream_t stream);
cudaError_t launch_hook_wait(const HookParams &p, int serve_ctas, cudaStream_t stream);
cudaError_t launch_barrier(const BarrierParams &p, cudaStream_t stream);
// 16-byte streaming copy (peer-bandwidth diagnostics).
cudaError_t launch_stream_copy(const void *src, void *dst, uint64_t bytes, int blocks, cudaStream_t stream);
// Request deduplication around the gather (dedup.cu).
cudaError_t launch_dedup(const DedupParams &p, int num_sms, cudaStream_t stream);
cudaError_t launch_expand(const DedupParams &p, int num_sms, cudaStream_t stream);
// Bounded wait on a flag nothing sets; used by the timeout self-test.
cudaError_t launch_wait_probe(const uint64_t *flag, uint64_t expected, uint64_t timeout_ns, ErrorSink error,
                              cudaStream_t stream);

// Peer-memory probe (peer_probe.cu): random rows moved between this GPU and
// its peers with one access mechanism per CTA parity (diagnostics only).
enum ProbeMode : uint32_t {
    kProbePullV4 = 0,      // 16-byte loads from the peer, 4 row groups in flight
    kProbePullV4Deep = 1,  // the same with 8 row groups in flight
    kProbePullV8 = 2,      // 32-byte loads from the peer
    kProbePullLdgsts = 3,  // 16-byte cp.async from the peer into a shared ring
    kProbePushV4 = 4,      // 16-byte stores into the peer
    kProbePushV8 = 5,      // 32-byte stores into the peer
    kProbePushBulk = 6,    // bulk copies shared -> peer global (local bulk loads feed them)
    kProbePushSeqV8 = 7,   // 32-byte stores of random local rows into consecutive peer rows
    kProbePullSeqV8 = 8,   // 32-byte loads of consecutive peer rows into consecutive local rows
    kProbePullV8L2 = 9,    // 32-byte loads from the peer with the 256-byte L2 prefetch-size hint
};

struct PeerProbeParams {
    uint64_t peer_table[kMaxRanks];  // pull sources: each rank's table (this rank's own included)
    uint64_t peer_out[kMaxRanks];    // push destinations: each rank's output region
    const uint8_t *local_table;      // push source
    uint8_t *local_out;              // pull destination
    ErrorSink error;
    uint64_t table_rows, out_rows;
    uint32_t rows, world, rank, row_bytes;
    uint32_t mode_even, mode_odd;    // ProbeMode of even / odd CTAs
    uint32_t even_share_pct;         // rows taken by the even CTAs when the modes differ
    uint32_t seed;
};

cudaError_t launch_peer_probe(const PeerProbeParams &p, int blocks, cudaStream_t stream);

// Message-passing litmus test of the release/acquire flag protocol.
enum LitmusRole : uint32_t { kLitmusProducer = 0, kLitmusConsumer = 1, kLitmusBoth = 2 };
enum LitmusStatus : uint32_t { kLitmusProducerTimeout = 1, kLitmusConsumerTimeout = 2 };

struct LitmusResult {
    uint32_t status;           // 0, or the LitmusStatus of the side that gave up first
    uint32_t epoch;            // epoch of that wait
    uint32_t mismatches;       // words that differed from the acquired epoch's values
    uint32_t first_bad_epoch;  // 0xFFFFFFFF when none
    uint32_t epochs_done;      // last epoch the consumer acknowledged
    uint32_t pad;
    uint64_t observed;         // flag value seen when the wait gave up
};

struct LitmusParams {
    uint32_t *data_remote;       // producer: data in the consumer's memory
    const uint32_t *data_local;  // consumer: the same data, local
    uint64_t *flag_remote;       // producer releases epochs here (consumer's memory)
    const uint64_t *flag_local;  // consumer polls
    uint64_t *ack_remote;        // consumer acknowledges here (producer's memory)
    const uint64_t *ack_local;   // producer polls
    uint32_t *prod_count;        // arrivals of this GPU's producer CTAs
    uint32_t *cons_count;        // arrivals of this GPU's consumer CTAs
    LitmusResult *result;
    uint32_t words;  // per epoch, a multiple of 4
    uint32_t epochs;
    uint32_t role;   // LitmusRole
    uint32_t weak_loads;
    uint64_t timeout_ns;
};

// Cooperative launch of `ctas` CTAs per role (2 x ctas for kLitmusBoth).
cudaError_t launch_litmus(const LitmusParams &p, uint32_t ctas, cudaStream_t stream);

} // namespace engram
