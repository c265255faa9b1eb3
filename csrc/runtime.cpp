// Native runtime of the B200 Engram buffer, exposed to Python as `_C.Runtime`.
//
// Parity: `engram_sge::Runtime` (sge_write/csrc/runtime.cpp:23-662) and the
// native `deep_ep::engram::EngramBuffer` (deepep/csrc/buffers/engram.hpp).
// Responsibilities:
//   * allocate this rank's host shard and device arena (memory.h) and serve
//     their descriptors to peers (fdpass.h);
//   * map every same-node peer's shard and arena, probe the peer-HBM route per
//     owner, and commit the negotiated route table into kernel parameters;
//   * write(): fill the host shard, the optional HBM mirror and the FP8 scale
//     table;
//   * fetch(): enqueue dispatch (host-route owners) and gather (direct owners,
//     padding, scales) on the caller's stream and return per-layer views;
//   * wait_layer(): make the caller's stream depend on the fetch, enqueue the
//     bounded done-flag wait for host-route owners, record the layer event;
//   * run the owner service that launches push kernels for requesters;
//   * keep the optional replica of each layer's hot id prefix and export a
//     layer's stored rows and scales for checkpoints.
// Capture-aware event wiring follows the reference (runtime.cpp:412-568): an
// eager fetch waits for the previous round's per-layer completion events;
// under capture an internal event joins cross-stream hooks into the graph and
// EXTERNAL events carry completion to work outside the graph.
#include <ATen/core/CachingHostAllocator.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDACachingAllocator.h>
#include <c10/cuda/CUDAGuard.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include <unistd.h>

#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "driver.h"
#include "fdpass.h"
#include "kernels/params.h"
#include "memory.h"
#include "bindings.h"
#include "owner_service.h"
#include "trace.h"

namespace py = pybind11;

// Types holding Python objects get hidden visibility, like pybind11's own;
// the module init function below is exported explicitly by PYBIND11_MODULE.
#pragma GCC visibility push(hidden)

namespace engram {

enum Route : int { kHostRoute = 0, kPeerHbm = 1 };

// Default rows per claimable unit of an owner-push request: 512 rows per chunk
// halves the claims against 256 while a 2-GPU fetch of the headline shape
// still splits into 192 chunks.
constexpr uint32_t kServeChunkRows = 512;

namespace {

template <class T> T get(const py::dict &d, const char *key) {
    if (!d.contains(key))
        throw std::runtime_error(std::string("missing config key: ") + key);
    return py::cast<T>(d[key]);
}

bool capturing(cudaStream_t s) {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    check_cuda(cudaStreamIsCapturing(s, &st), "query capture status");
    return st == cudaStreamCaptureStatusActive;
}

} // namespace

class Runtime : public std::enable_shared_from_this<Runtime> {
  public:
    explicit Runtime(const py::dict &cfg) {
        rank_ = get<uint32_t>(cfg, "rank");
        world_ = get<uint32_t>(cfg, "world");
        local_rank_ = get<uint32_t>(cfg, "local_rank");
        local_size_ = get<uint32_t>(cfg, "local_size");
        device_ = get<int>(cfg, "device");
        entries_ = get<std::vector<uint32_t>>(cfg, "entries");
        hidden_ = get<uint32_t>(cfg, "hidden");
        elem_ = get<uint32_t>(cfg, "element_bytes");
        max_tokens_ = get<uint32_t>(cfg, "max_tokens");
        ept_ = get<uint32_t>(cfg, "ept");
        packs_ = get<uint32_t>(cfg, "packs");
        channels_ = get<uint32_t>(cfg, "channels");
        egm_ = get<bool>(cfg, "egm");
        local_sf_ = get<bool>(cfg, "local_sf");
        timeout_ns_ = uint64_t(get<double>(cfg, "timeout_s") * 1e9);
        token_ = get<std::string>(cfg, "token");
        allow_host_vmm_ = get<bool>(cfg, "allow_host_vmm");
        gather_choice_ = get<std::string>(cfg, "gather_kernel");
        gather_variant_ = gather_choice_ == "bulk" ? kGatherBulk : kGatherSimt;  // "auto" and "simt": SIMT
        tuning_ctas_per_sm_ = get<uint32_t>(cfg, "gather_ctas_per_sm");
        dedup_mode_ = get<int>(cfg, "dedup");
        tuning_unroll_ = get<uint32_t>(cfg, "gather_unroll");
        if (cfg.contains("gather_strided"))
            tuning_strided_ = get<uint32_t>(cfg, "gather_strided");
        if (cfg.contains("gather_vector"))
            tuning_vector_ = get<uint32_t>(cfg, "gather_vector");
        if (cfg.contains("gather_l2_prefetch"))
            tuning_l2_prefetch_ = get<bool>(cfg, "gather_l2_prefetch");
        if (cfg.contains("peer_transport"))
            push_peers_ = get<std::string>(cfg, "peer_transport") == "push";
        if (cfg.contains("serve_chunk_rows"))
            serve_chunk_rows_ = get<uint32_t>(cfg, "serve_chunk_rows");
        check(serve_chunk_rows_ >= 16 && serve_chunk_rows_ <= kMaxServeChunkRows && serve_chunk_rows_ % 16 == 0,
              "serve chunk rows must be a multiple of 16 in [16, 512]");
        check(tuning_vector_ == 0 || tuning_vector_ == 16 || tuning_vector_ == 32,
              "gather vector bytes must be 0 (auto), 16 or 32");
        layers_ = uint32_t(entries_.size());
        row_bytes_ = hidden_ * elem_;
        capacity_ = max_tokens_ * ept_;
        check((uint64_t(capacity_) + serve_chunk_rows_ - 1) / serve_chunk_rows_ <= kMaxServeChunks,
              "a request can exceed 32768 serving chunks: raise ENGRAM_SERVE_CHUNK_ROWS");
        check(world_ >= 1 && world_ <= kMaxRanks, "world size out of range");
        check(layers_ >= 1 && layers_ <= kMaxLayers, "layer count out of range");
        check(rank_ < world_ && local_size_ >= 1 && world_ % local_size_ == 0 && local_rank_ == rank_ % local_size_,
              "rank layout");
        check(row_bytes_ % 16 == 0 && row_bytes_ > 0, "row bytes must be a positive multiple of 16");
        check(channels_ >= 1 && channels_ <= 16, "channels out of range");
        uint64_t at = 0, sf_at = 0;
        for (uint32_t n : entries_) {
            check(n > 0 && uint64_t(n) * world_ <= 0x7FFFFFFFull, "vocabulary index limit");
            table_bases_.push_back(uint32_t(at));
            sf_bases_.push_back(uint32_t(sf_at));
            at += n;
            sf_at += uint64_t(n) * (local_sf_ ? world_ : 1) * packs_;
        }
        check(at < (1ull << 32) && sf_at < (1ull << 32), "local vocabulary too large");
        table_rows_ = at;

        if (cfg.contains("index_staging"))
            stage_indices_ = get<bool>(cfg, "index_staging");
        if (cfg.contains("nvtx") && get<bool>(cfg, "nvtx"))
            nvtx_enabled().store(true);
        py::dict plan = get<py::dict>(cfg, "plan");
        auto off = [&](const char *k) { return get<size_t>(plan, k); };
        dev_mirror_ = off("dev_mirror");
        dev_mirror_bytes_ = off("dev_mirror_bytes");
        dev_sf_table_ = off("dev_sf_table");
        dev_output_ = off("dev_output");
        dev_sf_output_ = off("dev_sf_output");
        dev_done_ = off("dev_done");
        dev_inbox_ = off("dev_inbox");
        dev_dedup_ = off("dev_dedup");
        dev_dedup_bytes_ = off("dev_dedup_bytes");
        dev_replica_ = off("dev_replica");
        dev_replica_bytes_ = off("dev_replica_bytes");
        hot_rows_.assign(layers_, 0);
        hot_bases_.assign(layers_, 0);
        if (cfg.contains("hot_rows")) {
            const auto hot = get<std::vector<uint32_t>>(cfg, "hot_rows");
            check(hot.size() == layers_, "hot_rows needs one count per layer");
            uint64_t at = 0;
            for (uint32_t l = 0; l < layers_; ++l) {
                check(uint64_t(hot[l]) <= uint64_t(entries_[l]) * world_, "hot_rows exceeds the layer's global rows");
                hot_rows_[l] = hot[l];
                hot_bases_[l] = uint32_t(at);
                at += hot[l];
            }
            check(at * row_bytes_ == dev_replica_bytes_, "replica region does not match hot_rows");
        }
        dev_scratch_ = off("dev_scratch");
        dev_scratch_bytes_ = off("dev_scratch_bytes");
        device_bytes_ = off("device_bytes");
        table_bytes_ = off("table_bytes");
        mailbox_bytes_ = off("mailbox_bytes");
        check(!egm_ || dev_mirror_bytes_ == table_rows_ * row_bytes_, "mirror size does not match the vocabulary");

        c10::cuda::CUDAGuard guard(device_);
        check_cuda(cudaFree(nullptr), "initialise CUDA context");
        check_cuda(cudaDeviceGetAttribute(&num_sms_, cudaDevAttrMultiProcessorCount, device_), "SM count");
        try {
            arena_ = SharedAllocation::device(device_bytes_, device_);
            host_ = SharedAllocation::host(table_bytes_, device_, allow_host_vmm_);
            mailbox_ = SharedAllocation::host(mailbox_bytes_, device_, allow_host_vmm_);
            carve_scratch();
            check_cuda(cudaHostAlloc(reinterpret_cast<void **>(&host_error_), sizeof(ErrorRecord), cudaHostAllocMapped),
                       "error record");
            std::memset(host_error_, 0, sizeof(ErrorRecord));
            check_cuda(cudaHostGetDevicePointer(reinterpret_cast<void **>(&host_error_dev_), host_error_, 0),
                       "error record device pointer");
            check_cuda(cudaHostAlloc(reinterpret_cast<void **>(&dedup_stats_), 16, cudaHostAllocMapped), "dedup stats");
            std::memset(dedup_stats_, 0, 16);
            check_cuda(cudaHostGetDevicePointer(reinterpret_cast<void **>(&dedup_stats_dev_), dedup_stats_, 0),
                       "dedup stats device pointer");
            check_cuda(cudaEventCreateWithFlags(&issued_, cudaEventDisableTiming), "issue event");
            check_cuda(cudaEventCreateWithFlags(&capture_issued_, cudaEventDisableTiming), "capture event");
            for (uint32_t l = 0; l < layers_; ++l) {
                cudaEvent_t e;
                check_cuda(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "layer event");
                finished_.push_back(e);
                finished_stream_.push_back(nullptr);
            }
            int lo = 0, hi = 0;
            check_cuda(cudaDeviceGetStreamPriorityRange(&lo, &hi), "stream priorities");
            check_cuda(cudaStreamCreateWithPriority(&owner_stream_, cudaStreamNonBlocking, hi), "owner stream");
            if (stage_indices_) {
                check_cuda(cudaStreamCreateWithFlags(&stage_stream_, cudaStreamNonBlocking), "staging stream");
                for (int i = 0; i < 2; ++i) {
                    check_cuda(cudaEventCreateWithFlags(&stage_copied_[i], cudaEventDisableTiming), "staging event");
                    check_cuda(cudaEventCreateWithFlags(&stage_free_[i], cudaEventDisableTiming), "staging event");
                    check_cuda(cudaMalloc(reinterpret_cast<void **>(&stage_buf_[i]),
                                          std::max<size_t>(size_t(layers_) * capacity_ * 4, 16)),
                               "staging buffer");
                }
            }
        } catch (...) {
            release();
            throw;
        }
        peer_host_.resize(world_);
        peer_dev_.resize(world_);
        routes_.assign(world_, kHostRoute);
        mapping_errors_.assign(world_, "");
    }

    ~Runtime() { release(); }

    // ------------------------------------------------------------- bootstrap
    py::dict bootstrap() {
        check(!closed_, "runtime closed");
        if (!fd_server_)
            fd_server_ = std::make_unique<FdServer>(socket_name(rank_), std::vector<int>{mailbox_->fd(), arena_->fd()});
        py::dict d;
        d["pid"] = int(getpid());
        d["socket"] = socket_name(rank_);
        d["host_kind"] = int(mailbox_->kind());
        d["host_kind_name"] = memory_kind_name(mailbox_->kind());
        d["host_bytes"] = mailbox_->bytes();
        d["host_numa"] = mailbox_->numa();
        d["dev_bytes"] = arena_->bytes();
        d["mirror"] = egm_;
        d["mirror_offset"] = dev_mirror_;
        d["mirror_bytes"] = egm_ ? dev_mirror_bytes_ : size_t(0);
        d["config"] = py::make_tuple(world_, local_size_, entries_, hidden_, elem_, max_tokens_, ept_, packs_, egm_,
                                     local_sf_, device_bytes_, table_bytes_, mailbox_bytes_);
        return d;
    }

    py::dict probe_routes(const py::list &peers, const std::vector<int> &candidates) {
        check(!probed_ && !closed_ && peers.size() == world_ && candidates.size() == world_, "route probe state");
        routes_.assign(candidates.begin(), candidates.end());
        mapping_errors_.assign(world_, "");
        c10::cuda::CUDAGuard guard(device_);
        for (uint32_t p = 0; p < world_; ++p) {
            check(candidates[p] == kHostRoute || (candidates[p] == kPeerHbm && egm_), "invalid route candidate");
            if (p == rank_)
                continue;
            py::dict d = peers[p].cast<py::dict>();
            check(p / local_size_ == rank_ / local_size_,
                  "owner " + std::to_string(p) + " is on another node; this transport spans one NVLink node");
            // Mandatory mappings: every same-node peer's host shard (mailbox
            // headers) and device arena (inbox, outputs, done flags).
            const std::string sock = get<std::string>(d, "socket");
            peer_host_[p] = std::make_unique<PeerMapping>(MemoryKind(get<int>(d, "host_kind")), fetch_fd(sock, 0),
                                                          get<size_t>(d, "host_bytes"), device_,
                                                          get<int>(d, "host_numa"));
            peer_dev_[p] = std::make_unique<PeerMapping>(MemoryKind::DeviceVmm, fetch_fd(sock, 1),
                                                         get<size_t>(d, "dev_bytes"), device_, -1);
            check(peer_dev_[p]->bytes() >= device_bytes_ && peer_host_[p]->bytes() >= mailbox_bytes_,
                  "peer allocation smaller than the agreed plan");
            if (candidates[p] != kPeerHbm)
                continue;
            try {
                check(get<bool>(d, "mirror"), "owner keeps no HBM mirror");
                check(get<size_t>(d, "mirror_bytes") == table_rows_ * row_bytes_ &&
                          get<size_t>(d, "mirror_offset") == dev_mirror_,
                      "owner HBM mirror size or offset mismatch");
                check(peer_dev_[p]->readable(dev_mirror_, device_), "owner HBM mirror is not readable from this GPU");
            } catch (const std::runtime_error &e) {
                routes_[p] = kHostRoute;
                mapping_errors_[p] = e.what();
            }
        }
        routes_[rank_] = egm_ ? kPeerHbm : kHostRoute;
        probed_ = true;
        py::dict r;
        r["routes"] = routes_;
        r["errors"] = mapping_errors_;
        return r;
    }

    void prepare_routes(const std::vector<int> &selected) {
        check(probed_ && !ready_ && !closed_ && selected.size() == world_, "route commit state");
        for (uint32_t p = 0; p < world_; ++p)
            check(selected[p] <= routes_[p], "route exceeds probed capability");
        routes_ = selected;
        // Transport per pair: peer-HBM pairs are pulled by the requester, or
        // (ENGRAM_PEER_TRANSPORT=push) dispatched to the owner, which pushes
        // the rows from its HBM mirror with the host route's serving code.
        // Both sides agreed on the same switch, so the pairs stay symmetric.
        pushed_.assign(world_, 0);
        has_host_routes_ = false;
        serves_any_ = false;
        serve_.assign(world_, 0);
        for (uint32_t p = 0; p < world_; ++p)
            if (p != rank_ && (routes_[p] == kHostRoute || push_peers_)) {
                pushed_[p] = 1;
                has_host_routes_ = true;
                serves_any_ = true;
                serve_[p] = 1;
            }
        // "auto" is the SIMT kernel on every route: its vector loads from a
        // peer's mirror are plain per-thread loads.  The TMA ring, which
        // issues bulk copies whose source is a peer's memory, runs only when
        // asked for by name.
        if (gather_choice_ == "auto")
            gather_variant_ = kGatherSimt;
        // Vector width "auto": 32-byte accesses when rows come over NVLink
        // (random 256-byte rows moved 5% faster than with 16-byte ones), 16-byte
        // ones when every row is local (4% faster from local HBM).
        bool remote_direct = false;
        for (uint32_t p = 0; p < world_; ++p)
            remote_direct |= (p != rank_ && !pushed_[p]);
        vector_bytes_ = tuning_vector_ ? tuning_vector_ : (remote_direct ? 32u : 16u);
        build_params();
        // Every peer imported our descriptors during its probe, which finished
        // before the probe reports were exchanged.
        if (fd_server_) {
            fds_served_ = fd_server_->served();
            fd_server_.reset();
        }
        ready_ = true;
    }

    void connect() {
        check(ready_ && !connected_ && !closed_, "connect state");
        if (serves_any_) {
            OwnerServiceConfig c;
            c.world = world_;
            c.layers = layers_;
            c.capacity = capacity_;
            c.rank = rank_;
            c.headers = reinterpret_cast<const MailboxHeader *>(mailbox_->host_ptr());
            c.serve = serve_;
            const int dev = device_;
            service_.start(
                std::move(c), [this](const std::vector<PushTask> &batch) { launch_push_batch(batch); },
                [dev] { check_cuda(cudaSetDevice(dev), "owner service device"); });
        }
        connected_ = true;
    }

    // ------------------------------------------------------------------ write
    void write(uint32_t layer, const torch::Tensor &storage, const c10::optional<torch::Tensor> &scales) {
        TraceRange trace("engram/write");
        check_health();
        check(ready_ && !closed_, "runtime not ready");
        check(layer < layers_, "write layer out of range");
        c10::cuda::CUDAGuard guard(device_);
        const size_t bytes = size_t(entries_[layer]) * row_bytes_;
        check(size_t(storage.nbytes()) == bytes && storage.is_contiguous(), "storage shape");
        uint8_t *dst = static_cast<uint8_t *>(host_->host_ptr()) + size_t(table_bases_[layer]) * row_bytes_;
        if (storage.is_cuda())
            check_cuda(cudaMemcpy(dst, storage.data_ptr(), bytes, cudaMemcpyDefault), "write vocabulary to host shard");
        else
            std::memcpy(dst, storage.data_ptr(), bytes);
        if (egm_) {
            void *mirror = reinterpret_cast<uint8_t *>(arena_->ptr()) + dev_mirror_ +
                           size_t(table_bases_[layer]) * row_bytes_;
            check_cuda(cudaMemcpy(mirror, dst, bytes, cudaMemcpyDefault), "write HBM mirror");
        }
        if (packs_) {
            check(scales.has_value(), "missing scales");
            const size_t rows = size_t(entries_[layer]) * (local_sf_ ? world_ : 1);
            const size_t count = rows * packs_;
            const auto &sf = *scales;
            check(sf.scalar_type() == torch::kFloat32 && sf.is_contiguous() &&
                      size_t(sf.numel()) == size_t(entries_[layer]) * world_ * packs_,
                  "scale shape");
            const float *src = sf.data_ptr<float>() + (local_sf_ ? 0 : size_t(rank_) * entries_[layer] * packs_);
            void *target = reinterpret_cast<uint8_t *>(arena_->ptr()) + dev_sf_table_ + size_t(sf_bases_[layer]) * 4;
            check_cuda(cudaMemcpy(target, src, count * 4, cudaMemcpyDefault), "write scale table");
        }
        check_cuda(cudaDeviceSynchronize(), "write synchronise");
    }

    // Copy of layer `layer` as stored on this rank (checkpoints): the host
    // shard's rows and the scale rows this rank holds (all `world * n` with a
    // full local scale table, else its own `n`).  Quiesced like write().
    py::tuple read_layer(uint32_t layer) {
        check_health();
        check(ready_ && !closed_, "runtime not ready");
        check(layer < layers_, "layer out of range");
        c10::cuda::CUDAGuard guard(device_);
        check_cuda(cudaDeviceSynchronize(), "read_layer synchronise");
        const int64_t n = entries_[layer];
        auto rows = torch::empty({n, int64_t(row_bytes_)}, torch::TensorOptions().dtype(torch::kUInt8));
        std::memcpy(rows.data_ptr(), static_cast<const uint8_t *>(host_->host_ptr()) + size_t(table_bases_[layer]) * row_bytes_,
                    size_t(n) * row_bytes_);
        if (!packs_)
            return py::make_tuple(rows, py::none());
        const int64_t sf_rows = n * (local_sf_ ? world_ : 1);
        auto scales = torch::empty({sf_rows, int64_t(packs_)}, torch::TensorOptions().dtype(torch::kFloat32));
        const void *src = reinterpret_cast<const uint8_t *>(arena_->ptr()) + dev_sf_table_ + size_t(sf_bases_[layer]) * 4;
        check_cuda(cudaMemcpy(scales.data_ptr(), src, size_t(sf_rows) * packs_ * 4, cudaMemcpyDeviceToHost),
                   "read scale table");
        return py::make_tuple(rows, scales);
    }

    // ------------------------------------------------------------------ fetch
    // The kernels read `indices` on the current stream.  A device tensor is
    // recorded on that stream for the caching allocator.  A pinned host
    // tensor is read in place over PCIe through its device mapping (the
    // step's H2D happens inside the kernels that consume it, with no copy
    // engine round trip); its pinned block is recorded on the stream so the
    // host allocator does not hand it out again before they finish.
    const int32_t *index_pointer(const torch::Tensor &indices) {
        auto stream = at::cuda::getCurrentCUDAStream(device_);
        if (indices.is_cuda()) {
            try {
                c10::cuda::CUDACachingAllocator::recordStream(indices.storage().data_ptr(), stream);
            } catch (const c10::Error &) {
                // Not from the caching allocator: the caller owns its lifetime.
            }
            return indices.data_ptr<int32_t>();
        }
        if (indices.numel() == 0)
            return nullptr;
        const int32_t *host = indices.data_ptr<int32_t>();
        cudaPointerAttributes attr{};
        const bool mapped = cudaPointerGetAttributes(&attr, host) == cudaSuccess &&
                            attr.type == cudaMemoryTypeHost && attr.devicePointer != nullptr;
        if (!mapped) {
            cudaGetLastError();
            check(false, "host indices must be in pinned (page-locked, mapped) memory");
        }
        const auto &storage = indices.storage();
        at::getHostAllocator(at::kCUDA)->record_event(storage.mutable_data(), storage.data_ptr().get_context(),
                                                      stream.unwrap());
        return static_cast<const int32_t *>(attr.devicePointer);
    }

    // Index staging (ENGRAM_INDEX_STAGING=1, eager fetches of pinned host
    // indices): the copy engine moves them into one of two device slots on a
    // side stream and the compute stream waits for that copy only.  When the
    // host enqueues a step ahead, the next step's copy runs while this step's
    // gather does, instead of the gather waiting on PCIe reads itself.  A
    // slot is refilled only after the kernels of the fetch that read it two
    // steps earlier (stage_free_).
    const int32_t *stage_host_indices(const torch::Tensor &indices, cudaStream_t s, uint32_t *slot_out) {
        // Checks that the memory is pinned and ties its block to the compute
        // stream, which outlives this runtime and waits for the copy below
        // (torch's host allocator records an event there when the block is
        // freed; a private stream could be gone by then).
        index_pointer(indices);
        const uint32_t slot = stage_next_;
        stage_next_ ^= 1u;
        if (stage_used_[slot])
            check_cuda(cudaStreamWaitEvent(stage_stream_, stage_free_[slot], 0), "staging slot reuse");
        check_cuda(cudaMemcpyAsync(stage_buf_[slot], indices.data_ptr<int32_t>(), size_t(indices.numel()) * 4,
                                   cudaMemcpyHostToDevice, stage_stream_),
                   "stage indices");
        check_cuda(cudaEventRecord(stage_copied_[slot], stage_stream_), "record staged indices");
        check_cuda(cudaStreamWaitEvent(s, stage_copied_[slot], 0), "wait for staged indices");
        stage_used_[slot] = true;
        *slot_out = slot;
        return stage_buf_[slot];
    }

    py::list fetch(const torch::Tensor &indices, uint32_t channels, bool col_major) {
        TraceRange trace("engram/fetch");
        check_health();
        check(connected_ && !closed_, "runtime is not connected");
        check(indices.dim() == 3 && indices.scalar_type() == torch::kInt && indices.is_contiguous() &&
                  indices.size(0) == layers_ && indices.size(2) == ept_ && indices.size(1) <= max_tokens_ &&
                  (indices.is_cpu() || (indices.is_cuda() && indices.get_device() == device_)),
              "indices must be contiguous int32 [layers, tokens, ept] on this GPU or in pinned host memory");
        check(channels >= 1 && channels <= channels_, "channels exceed the allocation");
        c10::cuda::CUDAGuard guard(device_);
        cudaStream_t s = at::cuda::getCurrentCUDAStream(device_).stream();
        issue_captured_ = capturing(s);
        issue_stream_ = s;
        // An eager fetch reuses the output region: wait for the previous
        // round's layer completions, unless they were recorded on this very
        // stream outside a capture (stream order already covers them).
        if (!issue_captured_)
            for (uint32_t l = 0; l < layers_; ++l)
                if (finished_stream_[l] != s)
                    check_cuda(cudaStreamWaitEvent(s, finished_[l], 0), "workspace reuse dependency");
        uint32_t staged_slot = 2;  // 2 = not staged
        const int32_t *idx = (stage_indices_ && indices.is_cpu() && !issue_captured_ && indices.numel() > 0)
                                 ? stage_host_indices(indices, s, &staged_slot)
                                 : index_pointer(indices);
        tokens_ = uint32_t(indices.size(1));
        const uint32_t rows = tokens_ * ept_;
        uint32_t ts, hs, ls;
        sf_strides(tokens_, col_major, &ts, &hs, &ls);
        if (rows > 0) {
            if (has_host_routes_) {
                DispatchParams d = dispatch_;
                d.indices = idx;
                d.rows = rows;
                d.channels = channels;
                check_cuda(launch_dispatch(d, s), "launch dispatch");
                ++launches_;
            }
            const bool dedup = use_dedup();
            DedupParams dp{};
            if (dedup) {
                dp = dedup_;
                dp.indices = idx;
                dp.rows = rows;
                check_cuda(launch_dedup(dp, num_sms_, s), "launch dedup");
                ++launches_;
                ++dedup_fetches_;
            }
            GatherParams g = gather_;
            g.dedup = dedup ? 1 : 0;
            g.indices = idx;
            g.rows = rows;
            g.sf_token_stride = ts;
            g.sf_hidden_stride = hs;
            g.sf_layer_stride = ls;
            check_cuda(launch_gather(g, num_sms_, s), "launch gather");
            ++launches_;
            if (dedup) {
                check_cuda(launch_expand(dp, num_sms_, s), "launch expand");
                ++launches_;
            }
        }
        if (staged_slot < 2)
            check_cuda(cudaEventRecord(stage_free_[staged_slot], s), "staging slot read");
        if (issue_captured_) {
            check_cuda(cudaEventRecord(capture_issued_, s), "record capture issue");
            check_cuda(cudaEventRecordWithFlags(issued_, s, cudaEventRecordExternal), "record external issue");
        } else {
            check_cuda(cudaEventRecord(issued_, s), "record issue");
        }
        ++fetches_;
        if (tokens_ != cached_tokens_ || col_major != cached_col_major_ || cached_outputs_.size() == 0) {
            cached_outputs_ = make_outputs(ts, hs, ls);
            cached_tokens_ = tokens_;
            cached_col_major_ = col_major;
        }
        return py::list(cached_outputs_);
    }

    // fetch() followed by wait_layer() of every layer on the same stream, in
    // one call: for callers that consume every layer at once, the host cost
    // of the per-layer hooks (one Python call and two stream queries each)
    // drops out.  Returns the same output views as fetch().
    py::list fetch_all(const torch::Tensor &indices, uint32_t channels, bool col_major) {
        py::list outputs = fetch(indices, channels, col_major);
        for (uint32_t l = 0; l < layers_; ++l)
            wait_layer(l);
        return outputs;
    }

    void wait_layer(uint32_t layer) {
        TraceRange trace("engram/hook");
        check_health();
        check(connected_ && !closed_, "runtime is not connected");
        check(layer < layers_, "hook layer out of range");
        c10::cuda::CUDAGuard guard(device_);
        cudaStream_t s = at::cuda::getCurrentCUDAStream(device_).stream();
        bool source_active = issue_captured_ && capturing(issue_stream_);
        if (source_active) {
            check_cuda(cudaStreamWaitEvent(s, capture_issued_, 0), "capture issue to hook dependency");
        } else {
            check_cuda(cudaStreamWaitEvent(s, issued_, capturing(s) ? cudaEventWaitExternal : 0),
                       "issue to hook dependency");
        }
        if (has_host_routes_ && tokens_ > 0) {
            HookParams h{};
            h.s = serve_params_;
            h.totals = totals_;
            h.epochs = epochs_;
            h.done = reinterpret_cast<const uint64_t *>(arena_->ptr() + dev_done_);
            h.layer = layer;
            h.serve = serves_any_ ? 1 : 0;
            h.timeout_ns = timeout_ns_;
            check_cuda(launch_hook_wait(h, serve_ctas(), s), "launch hook wait");
            ++launches_;
        }
        const bool hook_captured = capturing(s);
        check_cuda(cudaEventRecordWithFlags(finished_[layer], s, hook_captured ? cudaEventRecordExternal : 0),
                   "record layer completion");
        finished_stream_[layer] = hook_captured ? nullptr : s;
    }

    // Device barrier over every rank of the buffer, enqueued on the current
    // stream (capturable: the count lives in device memory).  Work the stream
    // enqueued before it is visible to every peer's work enqueued after
    // theirs.  Bounded by the buffer's GPU timeout; a timeout is reported
    // like any device error.
    void barrier() {
        check_health();
        check(connected_ && !closed_, "runtime is not connected");
        BarrierParams b{};
        const uint64_t own = arena_->ptr();
        for (uint32_t o = 0; o < world_; ++o) {
            const uint64_t base = o == rank_ ? own : peer_dev_[o]->ptr();
            b.peer_slot[o] = base + barrier_slots_offset_ + uint64_t(rank_) * 8;
        }
        b.count = barrier_count_;
        b.slots = reinterpret_cast<const uint64_t *>(own + barrier_slots_offset_);
        b.error = sink();
        b.world = world_;
        b.rank = rank_;
        b.timeout_ns = timeout_ns_;
        c10::cuda::CUDAGuard guard(device_);
        check_cuda(launch_barrier(b, at::cuda::getCurrentCUDAStream(device_).stream()), "launch barrier");
        ++launches_;
    }

    // Synchronous snapshot of the barrier count and slots (tests only).
    py::dict barrier_state() {
        c10::cuda::CUDAGuard guard(device_);
        check_cuda(cudaDeviceSynchronize(), "barrier state sync");
        uint64_t count = 0;
        std::vector<uint64_t> slots(world_);
        check_cuda(cudaMemcpy(&count, barrier_count_, 8, cudaMemcpyDeviceToHost), "read barrier count");
        check_cuda(cudaMemcpy(slots.data(), reinterpret_cast<void *>(arena_->ptr() + barrier_slots_offset_),
                              size_t(world_) * 8, cudaMemcpyDeviceToHost),
                   "read barrier slots");
        py::dict d;
        d["count"] = count;
        d["slots"] = slots;
        return d;
    }

    // ------------------------------------------------------------- inspection
    void check_health() {
        service_.check();
        if (host_error_ != nullptr) {
            volatile ErrorRecord *e = host_error_;
            if (e->status != 0)
                throw std::runtime_error(describe_error());
        }
    }

    py::dict error_state() {
        py::dict d;
        volatile ErrorRecord *e = host_error_;
        d["status"] = e ? e->status : 0u;
        d["layer"] = e ? e->layer : 0u;
        d["owner"] = e ? e->owner : 0u;
        d["count"] = e ? e->count : 0u;
        d["observed"] = e ? e->observed : 0ull;
        d["expected"] = e ? e->expected : 0ull;
        d["owner_service_error"] = service_.error();
        return d;
    }

    py::dict memory_usage() {
        py::dict d;
        d["rank"] = rank_;
        d["device_allocation_bytes"] = arena_ ? arena_->bytes() : 0;
        d["host_allocation_bytes"] = (host_ ? host_->bytes() : 0) + (mailbox_ ? mailbox_->bytes() : 0);
        d["output_bytes"] = size_t(layers_) * capacity_ * row_bytes_;
        d["cpu_vocabulary_bytes"] = size_t(table_rows_) * row_bytes_;
        d["hbm_mirror_bytes"] = egm_ ? dev_mirror_bytes_ : size_t(0);
        d["mailbox_bytes"] = size_t(world_) * layers_ * kHeaderBytes;
        d["inbox_bytes"] = size_t(world_) * layers_ * capacity_ * 8;
        d["owner_threads"] = service_.running() ? 1 : 0;
        d["served_requests"] = service_.requests();
        d["served_rows"] = service_.rows();
        d["push_batches"] = service_.batches();
        d["epochs_served_by_hooks_unseen"] = service_.skipped();
        d["max_push_launch_us"] = service_.max_launch_us();
        d["egm_enabled"] = egm_;
        bool direct_remote = false;
        for (uint32_t p = 0; p < world_; ++p)
            direct_remote |= (p != rank_ && routes_[p] == kPeerHbm);
        d["has_egm_routes"] = direct_remote;
        d["has_host_routes"] = has_host_routes_;
        d["routes"] = routes_;
        d["egm_mapping_errors"] = mapping_errors_;
        d["local_sf"] = local_sf_;
        d["table_numa"] = host_ ? host_->numa() : -1;
        d["host_memory_kind"] = host_ ? memory_kind_name(host_->kind()) : "none";
        d["host_memory_note"] = host_ ? host_->note() : "";
        d["cpu_vocabulary_allocations"] = 1;
        d["cpu_vocabulary_allocated_bytes"] = host_ ? host_->bytes() : 0;
        d["fd_transport"] = "unix_socket_scm_rights";
        d["fds_served"] = fds_served_;
        d["fetches"] = fetches_;
        d["kernel_launches"] = launches_;
        d["num_sms"] = num_sms_;
        d["gather_kernel"] = gather_variant_ == kGatherSimt ? "simt" : "tma_bulk";
        d["gather_vector_bytes"] = vector_bytes_;
        d["peer_transport"] = push_peers_ ? "push" : "pull";
        d["gather_l2_prefetch"] = tuning_l2_prefetch_;
        d["serve_chunk_rows"] = serve_chunk_rows_;
        d["dedup_mode"] = dedup_mode_ == 0 ? "off" : (dedup_mode_ == 1 ? "on" : "auto");
        d["dedup_fetches"] = dedup_fetches_;
        d["dedup_last_unique_ratio"] = dedup_ratio_;
        d["hot_rows"] = hot_rows_;
        d["hot_replica_bytes"] = dev_replica_bytes_;
        d["hot_replica_active"] = hot_active_;
        d["index_staging"] = stage_indices_;
        return d;
    }

    // Hot-prefix replica.  replica_view() is this rank's replica region as a
    // [sum(hot_rows), row_bytes] uint8 tensor (valid until close()); the
    // buffer fills it after write() through ordinary fetches, with the replica
    // switched off so those fetches read the owners.
    torch::Tensor replica_view() {
        check(connected_ && !closed_, "runtime is not connected");
        const int64_t rows = int64_t(dev_replica_bytes_ / (row_bytes_ ? row_bytes_ : 1));
        auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device_);
        return torch::from_blob(reinterpret_cast<void *>(arena_->ptr() + dev_replica_), {rows, int64_t(row_bytes_)},
                                opts);
    }

    void set_hot_active(bool on) {
        check(connected_ && !closed_, "runtime is not connected");
        hot_active_ = on && dev_replica_bytes_ > 0;
        for (uint32_t l = 0; l < layers_; ++l) {
            const uint32_t v = hot_active_ ? hot_rows_[l] : 0;
            gather_.layer.hot_rows[l] = v;
            dispatch_.layer.hot_rows[l] = v;
            dedup_.layer.hot_rows[l] = v;
        }
    }

    // Synchronous snapshot of the per-(layer, owner) counters (tests only).
    py::dict debug_state() {
        c10::cuda::CUDAGuard guard(device_);
        check_cuda(cudaDeviceSynchronize(), "debug sync");
        const size_t n = size_t(layers_) * world_;
        std::vector<uint64_t> epochs(n), done(n);
        std::vector<uint32_t> totals(n);
        check_cuda(cudaMemcpy(epochs.data(), epochs_, n * 8, cudaMemcpyDeviceToHost), "read epochs");
        check_cuda(cudaMemcpy(totals.data(), totals_, n * 4, cudaMemcpyDeviceToHost), "read totals");
        check_cuda(cudaMemcpy(done.data(), reinterpret_cast<void *>(arena_->ptr() + dev_done_), n * 8,
                              cudaMemcpyDeviceToHost),
                   "read done flags");
        std::vector<uint64_t> served;
        for (uint32_t r = 0; r < world_; ++r)
            for (uint32_t l = 0; l < layers_; ++l)
                served.push_back(service_.completed(r, l));
        py::dict d;
        d["epochs"] = epochs;
        d["totals"] = totals;
        d["done"] = done;
        d["served_epochs"] = served;
        return d;
    }

    // Bounded wait on a flag nothing sets: the GPU must give up after
    // `timeout_ms` and report a timeout without faulting (tests only).
    py::dict run_wait_probe(double timeout_ms) {
        c10::cuda::CUDAGuard guard(device_);
        uint64_t *flag = nullptr;
        ErrorRecord *dev = nullptr, *host = nullptr, *host_dev = nullptr;
        check_cuda(cudaMalloc(&flag, 8), "probe flag");
        check_cuda(cudaMalloc(&dev, sizeof(ErrorRecord)), "probe record");
        check_cuda(cudaMemset(flag, 0, 8), "clear probe flag");
        check_cuda(cudaMemset(dev, 0, sizeof(ErrorRecord)), "clear probe record");
        check_cuda(cudaHostAlloc(reinterpret_cast<void **>(&host), sizeof(ErrorRecord), cudaHostAllocMapped),
                   "probe host record");
        std::memset(host, 0, sizeof(ErrorRecord));
        check_cuda(cudaHostGetDevicePointer(reinterpret_cast<void **>(&host_dev), host, 0), "probe host pointer");
        cudaStream_t s = at::cuda::getCurrentCUDAStream(device_).stream();
        cudaEvent_t a, b;
        cudaEventCreate(&a);
        cudaEventCreate(&b);
        cudaEventRecord(a, s);
        check_cuda(launch_wait_probe(flag, 1, uint64_t(timeout_ms * 1e6), ErrorSink{dev, host_dev}, s), "probe");
        cudaEventRecord(b, s);
        check_cuda(cudaStreamSynchronize(s), "probe synchronise");
        float ms = 0;
        cudaEventElapsedTime(&ms, a, b);
        py::dict d;
        volatile ErrorRecord *h = host;
        d["status"] = h->status;
        d["observed"] = h->observed;
        d["expected"] = h->expected;
        d["elapsed_ms"] = ms;
        cudaEventDestroy(a);
        cudaEventDestroy(b);
        cudaFree(flag);
        cudaFree(dev);
        cudaFreeHost(host);
        return d;
    }

    // Peer bandwidth diagnostic: copy `bytes` between this GPU's output region
    // and peer `peer`'s (push = store into the peer, else load from it).
    // Returns the device time in microseconds.  Not for use during fetches.
    double debug_peer_copy(uint32_t peer, size_t bytes, bool push, int blocks) {
        check(connected_ && peer < world_ && (peer == rank_ || peer_dev_[peer]), "peer not mapped");
        const size_t region = size_t(layers_) * capacity_ * row_bytes_;
        bytes = std::min(bytes, region) / 16 * 16;
        c10::cuda::CUDAGuard guard(device_);
        cudaStream_t s = at::cuda::getCurrentCUDAStream(device_).stream();
        void *mine = reinterpret_cast<void *>(arena_->ptr() + dev_output_);
        void *theirs = reinterpret_cast<void *>((peer == rank_ ? arena_->ptr() : peer_dev_[peer]->ptr()) +
                                                dev_output_);
        cudaEvent_t a, b;
        cudaEventCreate(&a);
        cudaEventCreate(&b);
        cudaEventRecord(a, s);
        check_cuda(push ? launch_stream_copy(mine, theirs, bytes, blocks, s)
                        : launch_stream_copy(theirs, mine, bytes, blocks, s),
                   "peer copy");
        cudaEventRecord(b, s);
        check_cuda(cudaEventSynchronize(b), "peer copy sync");
        float ms = 0;
        cudaEventElapsedTime(&ms, a, b);
        cudaEventDestroy(a);
        cudaEventDestroy(b);
        return double(ms) * 1e3;
    }

    // Random-row peer probe (peer_probe.cu): `rows` rows of the agreed row size
    // move between this GPU and pseudo-random remote peers, even CTAs with
    // `mode_even`, odd CTAs with `mode_odd` (ProbeMode).  Pull reads the peers'
    // HBM mirrors into this rank's output region; push reads this rank's mirror
    // and writes the peers' output regions.  Returns the device time in
    // microseconds.  Diagnostics only: needs the mirror (ENGRAM_EGM_ENABLE=1)
    // and every peer on the peer-HBM route, and runs between fetches.
    double debug_peer_probe(uint32_t mode_even, uint32_t mode_odd, uint32_t rows, int blocks, uint32_t even_share_pct,
                            uint32_t seed) {
        check(connected_ && !closed_ && egm_, "the probe needs a connected buffer with the HBM mirror");
        check(mode_even <= kProbePullV8L2 && mode_odd <= kProbePullV8L2 && even_share_pct <= 100, "probe mode");
        check(row_bytes_ % 256 == 0 && row_bytes_ <= 1024, "the probe moves rows of 256, 512 or 1024 bytes");
        PeerProbeParams pp{};
        const uint64_t arena = arena_->ptr();
        for (uint32_t o = 0; o < world_; ++o) {
            check(o == rank_ || (peer_dev_[o] && routes_[o] == kPeerHbm), "probe needs every peer on the peer-HBM route");
            const uint64_t base = o == rank_ ? arena : peer_dev_[o]->ptr();
            pp.peer_table[o] = base + dev_mirror_;
            pp.peer_out[o] = base + dev_output_;
        }
        pp.local_table = reinterpret_cast<const uint8_t *>(arena + dev_mirror_);
        pp.local_out = reinterpret_cast<uint8_t *>(arena + dev_output_);
        pp.error = sink();
        pp.table_rows = table_rows_;
        pp.out_rows = uint64_t(layers_) * capacity_;
        pp.rows = rows;
        pp.world = world_;
        pp.rank = rank_;
        pp.row_bytes = row_bytes_;
        pp.mode_even = mode_even;
        pp.mode_odd = mode_odd;
        pp.even_share_pct = even_share_pct;
        pp.seed = seed * 0x9E3779B9u + rank_;
        c10::cuda::CUDAGuard guard(device_);
        cudaStream_t s = at::cuda::getCurrentCUDAStream(device_).stream();
        cudaEvent_t a, b;
        cudaEventCreate(&a);
        cudaEventCreate(&b);
        cudaEventRecord(a, s);
        const cudaError_t rc = launch_peer_probe(pp, blocks, s);
        cudaEventRecord(b, s);
        check_cuda(rc, "peer probe");
        check_cuda(cudaEventSynchronize(b), "peer probe sync");
        float ms = 0;
        cudaEventElapsedTime(&ms, a, b);
        cudaEventDestroy(a);
        cudaEventDestroy(b);
        check_health();
        return double(ms) * 1e3;
    }

    // Host-route serving on one GPU (diagnostics and single-GPU profiling):
    // this rank files a request to itself for `rows` pseudo-random rows of
    // layer 0 and one worker serves it through the host route's own code: the
    // push kernel ("push", `blocks` CTAs, the owner service's launch) or a hook
    // kernel that serves while it waits for its own done flag ("hook").  Rows
    // are read zero-copy from the pinned host shard and stored at their output
    // positions.  Returns the device time, the bytes moved and the rows whose
    // bytes differ from the shard.  Uses the [layer 0][this rank] slots of the
    // serving words, which the fetch path never uses for the rank itself.
    py::dict debug_serve_local(uint32_t rows, const std::string &worker, int blocks) {
        check(connected_ && !closed_, "runtime is not connected");
        check(worker == "push" || worker == "hook", "worker must be 'push' or 'hook'");
        check(rows >= 1 && rows <= capacity_ && entries_[0] >= 1, "rows must be in [1, capacity]");
        c10::cuda::CUDAGuard guard(device_);
        check_cuda(cudaDeviceSynchronize(), "serve_local sync");
        const uint32_t slot = rank_ * layers_;          // [requester = rank][layer 0]
        const uint32_t done_slot = 0 * world_ + rank_;  // done[layer 0][owner = rank]
        uint64_t epoch = 0;
        check_cuda(cudaMemcpy(&epoch, finish_ + slot, 8, cudaMemcpyDeviceToHost), "read finish word");
        epoch = (epoch >> 32) + 1;  // the finish word holds (next epoch - 1) << 32 once reset
        // Claim word armed for the previous epoch with every chunk taken: the
        // first worker arms it for `epoch`.  Finish word ready for `epoch`.
        const uint64_t armed = (epoch - 1) << 32;
        std::vector<uint64_t> entries(rows);
        std::vector<uint32_t> local_rows(rows);
        uint64_t h = 0x9E3779B97F4A7C15ull ^ (uint64_t(rows) << 17) ^ epoch;
        for (uint32_t i = 0; i < rows; ++i) {
            h ^= h >> 31;
            h *= 0xBF58476D1CE4E5B9ull;
            h ^= h >> 29;
            local_rows[i] = uint32_t(h % entries_[0]);  // layer 0 rows start at table base 0
            entries[i] = (uint64_t(i) << 32) | local_rows[i];
        }
        uint64_t *inbox = reinterpret_cast<uint64_t *>(arena_->ptr() + dev_inbox_) + uint64_t(slot) * capacity_;
        uint64_t *done = reinterpret_cast<uint64_t *>(arena_->ptr() + dev_done_) + done_slot;
        const uint32_t total = rows;
        check_cuda(cudaMemcpy(inbox, entries.data(), size_t(rows) * 8, cudaMemcpyHostToDevice), "fill inbox");
        check_cuda(cudaMemcpy(claim_ + slot, &armed, 8, cudaMemcpyHostToDevice), "arm claim");
        check_cuda(cudaMemcpy(finish_ + slot, &armed, 8, cudaMemcpyHostToDevice), "arm finish");
        check_cuda(cudaMemcpy(totals_ + done_slot, &total, 4, cudaMemcpyHostToDevice), "request total");
        check_cuda(cudaMemcpy(epochs_ + done_slot, &epoch, 8, cudaMemcpyHostToDevice), "request epoch");
        check_cuda(cudaMemset(reinterpret_cast<uint8_t *>(arena_->ptr() + dev_output_), 0,
                              size_t(rows) * row_bytes_), "clear output rows");
        auto *header = reinterpret_cast<MailboxHeader *>(mailbox_->host_ptr()) + slot;
        header->rows = rows;
        header->layer = 0;
        header->requester = rank_;
        header->channels = channels_;
        __atomic_store_n(&header->ready, epoch, __ATOMIC_RELEASE);
        ServeParams v = serve_params_;
        v.out_base[rank_] = arena_->ptr() + dev_output_;
        v.done_base[rank_] = arena_->ptr() + dev_done_;
        v.serve_mask = 1ull << rank_;
        cudaStream_t s = at::cuda::getCurrentCUDAStream(device_).stream();
        cudaEvent_t a, b;
        cudaEventCreate(&a);
        cudaEventCreate(&b);
        cudaEventRecord(a, s);
        cudaError_t rc;
        if (worker == "push") {
            PushParams pp{};
            pp.s = v;
            pp.tasks[0] = PushTask{rank_, 0, rows, channels_, epoch};
            pp.num_tasks = 1;
            rc = launch_push(pp, blocks, s);
        } else {
            HookParams hp{};
            hp.s = v;
            hp.totals = totals_;
            hp.epochs = epochs_;
            hp.done = reinterpret_cast<const uint64_t *>(arena_->ptr() + dev_done_);
            hp.layer = 0;
            hp.serve = 1;
            hp.timeout_ns = timeout_ns_;
            rc = launch_hook_wait(hp, serve_ctas(), s);
        }
        cudaEventRecord(b, s);
        check_cuda(rc, "serve_local launch");
        check_cuda(cudaEventSynchronize(b), "serve_local wait");
        float ms = 0;
        cudaEventElapsedTime(&ms, a, b);
        cudaEventDestroy(a);
        cudaEventDestroy(b);
        uint64_t seen = 0;
        check_cuda(cudaMemcpy(&seen, done, 8, cudaMemcpyDeviceToHost), "read done");
        std::vector<uint8_t> out(size_t(rows) * row_bytes_);
        check_cuda(cudaMemcpy(out.data(), reinterpret_cast<void *>(arena_->ptr() + dev_output_), out.size(),
                              cudaMemcpyDeviceToHost),
                   "read output rows");
        const uint8_t *table = static_cast<const uint8_t *>(host_->host_ptr());
        uint64_t bad = 0;
        for (uint32_t i = 0; i < rows; ++i)
            bad += std::memcmp(out.data() + size_t(i) * row_bytes_, table + size_t(local_rows[i]) * row_bytes_,
                               row_bytes_) != 0;
        check_health();
        py::dict d;
        d["us"] = double(ms) * 1e3;
        d["bytes"] = uint64_t(rows) * row_bytes_;
        d["mismatched_rows"] = bad;
        d["done_epoch"] = seen;
        d["expected_epoch"] = epoch;
        return d;
    }

    // Litmus test of the release/acquire flag protocol (between fetches only;
    // it overwrites the output region).  Header words sit at the start of
    // each rank's output region, the data after 4 KiB.  reset() zeroes this
    // rank's header; call it on both ranks and barrier before run().
    static constexpr size_t kLitmusData = 4096;
    void debug_litmus_reset() {
        c10::cuda::CUDAGuard guard(device_);
        check_cuda(cudaMemset(reinterpret_cast<void *>(arena_->ptr() + dev_output_), 0, kLitmusData), "litmus reset");
        check_cuda(cudaDeviceSynchronize(), "litmus reset sync");
    }

    py::dict debug_litmus(uint32_t peer, const std::string &role, uint32_t epochs, uint32_t words, uint32_t ctas,
                          bool weak_loads, double timeout_ms) {
        check(connected_ && peer < world_ && (peer == rank_ || peer_dev_[peer]), "peer not mapped");
        const size_t region = size_t(layers_) * capacity_ * row_bytes_;
        words = words / 4 * 4;
        check(words > 0 && kLitmusData + size_t(words) * 4 <= region, "litmus data exceeds the output region");
        check(ctas >= 1 && ctas <= 256, "litmus ctas out of range");
        LitmusParams lp{};
        if (role == "producer")
            lp.role = kLitmusProducer;
        else if (role == "consumer")
            lp.role = kLitmusConsumer;
        else if (role == "both")
            lp.role = kLitmusBoth;
        else
            check(false, "litmus role must be producer, consumer or both");
        check((lp.role == kLitmusBoth) == (peer == rank_), "role 'both' runs on this GPU alone");
        c10::cuda::CUDAGuard guard(device_);
        uint8_t *mine = reinterpret_cast<uint8_t *>(arena_->ptr() + dev_output_);
        uint8_t *theirs =
            reinterpret_cast<uint8_t *>((peer == rank_ ? arena_->ptr() : peer_dev_[peer]->ptr()) + dev_output_);
        // Producer writes data and flag into the consumer's region; the
        // consumer acknowledges into the producer's region.
        uint8_t *consumer_base = lp.role == kLitmusConsumer ? mine : theirs;
        uint8_t *producer_base = lp.role == kLitmusConsumer ? theirs : mine;
        lp.data_remote = reinterpret_cast<uint32_t *>(consumer_base + kLitmusData);
        lp.data_local = reinterpret_cast<const uint32_t *>(mine + kLitmusData);
        lp.flag_remote = reinterpret_cast<uint64_t *>(consumer_base);
        lp.flag_local = reinterpret_cast<const uint64_t *>(mine);
        lp.ack_remote = reinterpret_cast<uint64_t *>(producer_base + 64);
        lp.ack_local = reinterpret_cast<const uint64_t *>(mine + 64);
        lp.prod_count = reinterpret_cast<uint32_t *>(mine + 128);
        lp.cons_count = reinterpret_cast<uint32_t *>(mine + 192);
        lp.words = words;
        lp.epochs = epochs;
        lp.weak_loads = weak_loads ? 1 : 0;
        lp.timeout_ns = uint64_t(timeout_ms * 1e6);
        LitmusResult init{};
        init.first_bad_epoch = 0xFFFFFFFFu;
        LitmusResult *result = nullptr;
        check_cuda(cudaMalloc(&result, sizeof(LitmusResult)), "litmus result");
        lp.result = result;
        cudaStream_t s = at::cuda::getCurrentCUDAStream(device_).stream();
        cudaEvent_t a, b;
        cudaEventCreate(&a);
        cudaEventCreate(&b);
        LitmusResult out{};
        cudaError_t rc = cudaMemcpyAsync(result, &init, sizeof(init), cudaMemcpyHostToDevice, s);
        if (rc == cudaSuccess) {
            cudaEventRecord(a, s);
            rc = launch_litmus(lp, ctas, s);
            cudaEventRecord(b, s);
        }
        if (rc == cudaSuccess)
            rc = cudaMemcpyAsync(&out, result, sizeof(out), cudaMemcpyDeviceToHost, s);
        if (rc == cudaSuccess)
            rc = cudaStreamSynchronize(s);
        float ms = 0;
        if (rc == cudaSuccess)
            cudaEventElapsedTime(&ms, a, b);
        cudaEventDestroy(a);
        cudaEventDestroy(b);
        cudaFree(result);
        check_cuda(rc, "litmus run");
        py::dict d;
        d["status"] = out.status;
        d["epoch"] = out.epoch;
        d["observed"] = out.observed;
        d["mismatches"] = out.mismatches;
        d["first_bad_epoch"] = out.first_bad_epoch == 0xFFFFFFFFu ? -1 : int64_t(out.first_bad_epoch);
        d["epochs_done"] = out.epochs_done;
        d["ms"] = double(ms);
        return d;
    }

    // Fault injection for tests: stop serving requesters, as a dead owner
    // process would.  Requesters then see their bounded hook wait run out.
    void debug_stop_service() {
        py::gil_scoped_release release;
        service_.stop_and_join();
    }

    void close() {
        if (closed_)
            return;
        // The cached views keep this runtime alive; drop them so the memory
        // is released once the caller's own references are gone.
        cached_outputs_ = py::list();
        {
            c10::cuda::CUDAGuard guard(device_);
            cudaError_t rc = cudaDeviceSynchronize();
            py::gil_scoped_release release;
            service_.stop_and_join();
            if (owner_stream_)
                cudaStreamSynchronize(owner_stream_);
            check_cuda(rc, "synchronise before close");
        }
        fd_server_.reset();
        peer_dev_.clear();
        peer_host_.clear();
        closed_ = true;
        connected_ = false;
    }

    bool closed() const { return closed_; }

  private:
    std::string socket_name(uint32_t r) const { return "engram-b200." + token_ + "." + std::to_string(r); }

    ErrorSink sink() const { return ErrorSink{dev_error_, host_error_dev_}; }

    void carve_scratch() {
        uint8_t *base = reinterpret_cast<uint8_t *>(arena_->ptr()) + dev_scratch_;
        size_t at = 0;
        auto take = [&](size_t bytes) {
            at = align_up(at, 16);
            uint8_t *p = base + at;
            at += bytes;
            return p;
        };
        const size_t lw = size_t(layers_) * world_;
        epochs_ = reinterpret_cast<uint64_t *>(take(lw * 8));
        totals_ = reinterpret_cast<uint32_t *>(take(lw * 4));
        cursors_ = reinterpret_cast<uint32_t *>(take(lw * 4));
        layer_arrivals_ = reinterpret_cast<uint32_t *>(take(layers_ * 4));
        claim_ = reinterpret_cast<uint64_t *>(take(lw * 8));
        finish_ = reinterpret_cast<uint64_t *>(take(lw * 8));
        board_ = reinterpret_cast<uint64_t *>(take(lw * 8));
        dev_error_ = reinterpret_cast<ErrorRecord *>(take(sizeof(ErrorRecord)));
        dedup_state_ = reinterpret_cast<uint32_t *>(take(16));
        barrier_count_ = reinterpret_cast<uint64_t *>(take(8));
        barrier_slots_offset_ = size_t(reinterpret_cast<uint8_t *>(take(size_t(world_) * 8)) -
                                       reinterpret_cast<uint8_t *>(arena_->ptr()));
        check(at <= dev_scratch_bytes_, "scratch region too small");
    }

    void sf_strides(uint32_t tokens, bool col_major, uint32_t *ts, uint32_t *hs, uint32_t *ls) const {
        if (col_major) {
            *ts = 1;
            *hs = (tokens + 3) / 4 * 4;
            *ls = *hs * ept_ * packs_;
        } else {
            *ts = ept_ * packs_;
            *hs = 1;
            *ls = tokens * ept_ * packs_;
        }
    }

    void build_params() {
        LayerTable lt{};
        for (uint32_t l = 0; l < layers_; ++l) {
            lt.entries[l] = entries_[l];
            lt.table_bases[l] = table_bases_[l];
            lt.sf_bases[l] = sf_bases_[l];
            lt.hot_rows[l] = hot_active_ ? hot_rows_[l] : 0;
            lt.hot_bases[l] = hot_bases_[l];
        }
        const uint64_t arena = arena_->ptr();
        GatherParams &g = gather_;
        g = GatherParams{};
        g.output = reinterpret_cast<uint8_t *>(arena + dev_output_);
        g.sf_output = reinterpret_cast<float *>(arena + dev_sf_output_);
        g.error = sink();
        g.layer = lt;
        g.hot_base = arena + dev_replica_;
        for (uint32_t o = 0; o < world_; ++o) {
            if (o == rank_)
                g.direct_base[o] = egm_ ? arena + dev_mirror_ : host_->ptr();
            else if (!pushed_[o])
                g.direct_base[o] = peer_dev_[o]->ptr() + dev_mirror_;
            else
                g.direct_base[o] = 0;
        }
        if (local_sf_) {
            g.sf_base[0] = arena + dev_sf_table_;
            g.sf_shard_div = world_;
        } else {
            for (uint32_t o = 0; o < world_; ++o)
                g.sf_base[o] = o == rank_ ? arena + dev_sf_table_ : peer_dev_[o]->ptr() + dev_sf_table_;
            g.sf_shard_div = 1;
        }
        g.layers = layers_;
        g.ept = ept_;
        g.capacity = capacity_;
        g.row_bytes = row_bytes_;
        g.world = world_;
        g.packs = packs_;
        g.variant = gather_variant_;
        const uint32_t slots = dev_dedup_bytes_ ? uint32_t((dev_dedup_bytes_ - size_t(layers_) * capacity_ * 4) / 16) : 0;
        g.dedup_slots = reinterpret_cast<const uint32_t *>(arena + dev_dedup_ + size_t(slots) * 16);
        g.dedup_vals = reinterpret_cast<const uint64_t *>(arena + dev_dedup_ + size_t(slots) * 8);
        g.dedup_state = dedup_state_;
        DedupParams &dd = dedup_;
        dd = DedupParams{};
        dd.keys = reinterpret_cast<uint64_t *>(arena + dev_dedup_);
        dd.vals = reinterpret_cast<uint64_t *>(arena + dev_dedup_ + size_t(slots) * 8);
        dd.slots = reinterpret_cast<uint32_t *>(arena + dev_dedup_ + size_t(slots) * 16);
        dd.state = dedup_state_;
        dd.host_stats = dedup_stats_dev_;
        dd.output = reinterpret_cast<uint8_t *>(arena + dev_output_);
        dd.layer = lt;
        for (uint32_t o = 0; o < world_; ++o)
            dd.direct_base[o] = g.direct_base[o];
        dd.layers = layers_;
        dd.world = world_;
        dd.table_mask = slots ? slots - 1 : 0;
        dd.capacity = capacity_;
        dd.row_bytes = row_bytes_;
        dedup_slots_ = slots;
        g.ctas_per_sm = tuning_ctas_per_sm_;
        g.unroll = tuning_unroll_;
        g.strided = tuning_strided_;
        g.vector_bytes = vector_bytes_;
        g.l2_prefetch = tuning_l2_prefetch_ ? 1u : 0u;

        DispatchParams &d = dispatch_;
        d = DispatchParams{};
        d.cursors = cursors_;
        d.layer_arrivals = layer_arrivals_;
        d.totals = totals_;
        d.epochs = epochs_;
        d.error = sink();
        d.layer = lt;
        for (uint32_t o = 0; o < world_; ++o) {
            const bool host = o != rank_ && pushed_[o];
            d.inbox_base[o] = host ? peer_dev_[o]->ptr() + dev_inbox_ : 0;
            d.header_base[o] = host ? peer_host_[o]->ptr() : 0;
        }
        d.layers = layers_;
        d.capacity = capacity_;
        d.world = world_;
        d.rank = rank_;
        d.tile_rows = 512;

        ServeParams &v = serve_params_;
        v = ServeParams{};
        // Serving reads the HBM mirror when this owner keeps one (a pair that
        // fell back to the host route while the mirror is on); the rows are
        // the same bytes as the pinned host shard, which is read otherwise.
        v.table = reinterpret_cast<const uint8_t *>(egm_ ? arena + dev_mirror_ : host_->ptr());
        v.inbox = reinterpret_cast<const uint64_t *>(arena + dev_inbox_);
        v.claim = claim_;
        v.finish = finish_;
        v.board = board_;
        v.headers = reinterpret_cast<const MailboxHeader *>(mailbox_->ptr());
        v.error = sink();
        for (uint32_t r = 0; r < world_; ++r) {
            const bool serve = r != rank_ && pushed_[r];
            v.out_base[r] = serve ? peer_dev_[r]->ptr() + dev_output_ : 0;
            v.done_base[r] = serve ? peer_dev_[r]->ptr() + dev_done_ : 0;
            if (serve)
                v.serve_mask |= 1ull << r;
        }
        v.layers = layers_;
        v.world = world_;
        v.rank = rank_;
        v.capacity = capacity_;
        v.row_bytes = row_bytes_;
        v.chunk_rows = serve_chunk_rows_;
        v.table_rows = table_rows_;
    }

    // Runs on the owner-service thread: one push kernel per batch of up to
    // kMaxPushTasks requests; its CTAs claim chunks of every request in turn.
    void launch_push_batch(const std::vector<PushTask> &batch) {
        size_t at = 0;
        while (at < batch.size()) {
            PushParams p{};
            p.s = serve_params_;
            const size_t n = std::min(batch.size() - at, size_t(kMaxPushTasks));
            uint32_t chunks = 0, channels = 1;
            for (size_t i = 0; i < n; ++i) {
                p.tasks[i] = batch[at + i];
                chunks += (p.tasks[i].rows + serve_chunk_rows_ - 1) / serve_chunk_rows_;
                channels = std::max(channels, std::min(p.tasks[i].channels, 16u));
            }
            p.num_tasks = uint32_t(n);
            const uint32_t blocks = std::max(1u, std::min(chunks, std::max(uint32_t(serve_ctas()), channels * 2)));
            check_cuda(launch_push(p, int(blocks), owner_stream_), "launch push");
            at += n;
        }
    }

    // CTAs that serve requests (push kernels and serving hooks): one per SM
    // when the rows come from the HBM mirror (NVLink-bound), 16 when they come
    // from the pinned host shard, where 16 CTAs of 256 threads already keep
    // PCIe reads at the envelope (50.2 of 51.2 GB/s measured; 8 CTAs: 38).
    int serve_ctas() const { return egm_ ? num_sms_ : 16; }

    py::list make_outputs(uint32_t ts, uint32_t hs, uint32_t sf_layer_stride) {
        py::list out;
        auto keep = shared_from_this();
        const auto dtype = packs_ ? torch::kFloat8_e4m3fn : torch::kBFloat16;
        auto opts = torch::TensorOptions().dtype(dtype).device(torch::Device(torch::kCUDA, device_));
        auto fopts = torch::TensorOptions().dtype(torch::kFloat32).device(torch::Device(torch::kCUDA, device_));
        const uint64_t arena = arena_->ptr();
        for (uint32_t l = 0; l < layers_; ++l) {
            void *ptr = reinterpret_cast<void *>(arena + dev_output_ + uint64_t(l) * capacity_ * row_bytes_);
            auto data = torch::from_blob(ptr, {int64_t(tokens_), int64_t(hidden_) * ept_}, [keep](void *) {}, opts);
            if (packs_) {
                void *sptr = reinterpret_cast<void *>(arena + dev_sf_output_ + uint64_t(l) * sf_layer_stride * 4);
                auto scales = torch::from_blob(sptr, {int64_t(tokens_), int64_t(ept_) * packs_},
                                               {int64_t(ts), int64_t(hs)}, [keep](void *) {}, fopts);
                out.append(py::make_tuple(data, scales));
            } else {
                out.append(data);
            }
        }
        return out;
    }

    void release() noexcept {
        service_.stop_and_join();
        fd_server_.reset();
        peer_dev_.clear();
        peer_host_.clear();
        if (issued_)
            cudaEventDestroy(issued_);
        if (capture_issued_)
            cudaEventDestroy(capture_issued_);
        for (auto e : finished_)
            cudaEventDestroy(e);
        finished_.clear();
        issued_ = capture_issued_ = nullptr;
        if (owner_stream_) {
            cudaStreamSynchronize(owner_stream_);
            cudaStreamDestroy(owner_stream_);
            owner_stream_ = nullptr;
        }
        if (stage_stream_) {
            cudaStreamSynchronize(stage_stream_);
            cudaStreamDestroy(stage_stream_);
            stage_stream_ = nullptr;
        }
        for (int i = 0; i < 2; ++i) {
            if (stage_copied_[i])
                cudaEventDestroy(stage_copied_[i]);
            if (stage_free_[i])
                cudaEventDestroy(stage_free_[i]);
            if (stage_buf_[i])
                cudaFree(stage_buf_[i]);
            stage_copied_[i] = stage_free_[i] = nullptr;
            stage_buf_[i] = nullptr;
        }
        if (host_error_) {
            cudaFreeHost(host_error_);
            host_error_ = nullptr;
        }
        if (dedup_stats_) {
            cudaFreeHost(dedup_stats_);
            dedup_stats_ = nullptr;
        }
        mailbox_.reset();
        host_.reset();
        arena_.reset();
    }

    // configuration
    uint32_t rank_ = 0, world_ = 1, local_rank_ = 0, local_size_ = 1, layers_ = 0;
    int device_ = 0, num_sms_ = 0;
    std::vector<uint32_t> entries_, table_bases_, sf_bases_;
    uint32_t hidden_ = 0, elem_ = 0, max_tokens_ = 0, ept_ = 0, packs_ = 0, channels_ = 1;
    uint32_t row_bytes_ = 0, capacity_ = 0;
    uint64_t table_rows_ = 0, timeout_ns_ = 0;
    bool egm_ = false, local_sf_ = false, allow_host_vmm_ = true;
    uint32_t gather_variant_ = kGatherBulk, tuning_ctas_per_sm_ = 0, tuning_unroll_ = 0, tuning_strided_ = 0;
    uint32_t tuning_vector_ = 0, vector_bytes_ = 16;  // requested (0 = auto) and chosen SIMT vector bytes
    bool tuning_l2_prefetch_ = false;  // ENGRAM_GATHER_L2_PREFETCH
    uint32_t serve_chunk_rows_ = kServeChunkRows;  // ENGRAM_SERVE_CHUNK_ROWS
    std::string gather_choice_ = "auto";
    // request deduplication: mode 0 off, 1 on, 2 auto (on while the last
    // measured unique ratio is below kDedupOnRatio; re-measured every
    // kDedupProbeEvery fetches while off)
    int dedup_mode_ = 2;
    size_t dev_dedup_ = 0, dev_dedup_bytes_ = 0;
    // hot-prefix replication: global ids [0, hot_rows_[l]) of layer l are read
    // from the local replica once it is filled (hot_active_)
    size_t dev_replica_ = 0, dev_replica_bytes_ = 0;
    std::vector<uint32_t> hot_rows_, hot_bases_;
    bool hot_active_ = false;
    // index staging (see stage_host_indices)
    bool stage_indices_ = false;
    cudaStream_t stage_stream_ = nullptr;
    cudaEvent_t stage_copied_[2] = {nullptr, nullptr}, stage_free_[2] = {nullptr, nullptr};
    int32_t *stage_buf_[2] = {nullptr, nullptr};
    uint32_t stage_next_ = 0;
    bool stage_used_[2] = {false, false};
    uint32_t *dedup_state_ = nullptr, *dedup_stats_ = nullptr, *dedup_stats_dev_ = nullptr;
    uint32_t dedup_slots_ = 0, dedup_seen_epoch_ = 0, dedup_since_probe_ = 0;
    double dedup_ratio_ = -1.0;
    uint64_t dedup_fetches_ = 0;
    DedupParams dedup_{};
    static constexpr double kDedupOnRatio = 0.75;
    static constexpr uint32_t kDedupProbeEvery = 256;

    bool use_dedup() {
        if (dedup_mode_ == 0 || dedup_slots_ == 0)
            return false;
        // Fold in the counts of the last finished deduplicated fetch (host-mapped,
        // written by the GPU; read without synchronising).
        volatile uint32_t *st = dedup_stats_;
        const uint32_t epoch = st[2];
        if (epoch != dedup_seen_epoch_) {
            const uint32_t uniques = st[0], items = st[1];
            dedup_seen_epoch_ = epoch;
            if (items > 0)
                dedup_ratio_ = double(uniques) / double(items);
        }
        if (dedup_mode_ == 1)
            return true;
        if (dedup_ratio_ < 0.0 || dedup_ratio_ < kDedupOnRatio) {
            dedup_since_probe_ = 0;
            return true;
        }
        if (++dedup_since_probe_ >= kDedupProbeEvery) {
            dedup_since_probe_ = 0;
            return true;
        }
        return false;
    }
    std::string token_;
    size_t dev_mirror_ = 0, dev_mirror_bytes_ = 0, dev_sf_table_ = 0, dev_output_ = 0, dev_sf_output_ = 0, dev_done_ = 0,
           dev_inbox_ = 0, dev_scratch_ = 0, dev_scratch_bytes_ = 0, device_bytes_ = 0;
    size_t table_bytes_ = 0, mailbox_bytes_ = 0;
    // memory
    std::unique_ptr<SharedAllocation> arena_, host_, mailbox_;
    std::vector<std::unique_ptr<PeerMapping>> peer_host_, peer_dev_;
    std::unique_ptr<FdServer> fd_server_;
    long fds_served_ = 0;
    uint64_t *epochs_ = nullptr;
    uint32_t *totals_ = nullptr, *cursors_ = nullptr, *layer_arrivals_ = nullptr;
    uint64_t *claim_ = nullptr, *finish_ = nullptr, *board_ = nullptr;
    // device barrier: this rank's count and the arena offset of the slots
    // every peer writes (the same offset on every rank: the plan is agreed)
    uint64_t *barrier_count_ = nullptr;
    size_t barrier_slots_offset_ = 0;
    ErrorRecord *dev_error_ = nullptr, *host_error_ = nullptr, *host_error_dev_ = nullptr;
    // routes
    std::vector<int> routes_;
    std::vector<std::string> mapping_errors_;
    std::vector<uint8_t> serve_;
    std::vector<uint8_t> pushed_;  // per owner: rows arrive by owner push (host route, or push transport)
    bool push_peers_ = false;      // ENGRAM_PEER_TRANSPORT=push
    bool probed_ = false, ready_ = false, connected_ = false, closed_ = false;
    bool has_host_routes_ = false, serves_any_ = false;
    GatherParams gather_{};
    DispatchParams dispatch_{};
    ServeParams serve_params_{};
    // streams and events
    cudaEvent_t issued_ = nullptr, capture_issued_ = nullptr;
    std::vector<cudaEvent_t> finished_;
    std::vector<cudaStream_t> finished_stream_;  // stream of the last eager hook per layer
    // Output views of the last (tokens, scale layout); rebuilt when either changes.
    py::list cached_outputs_;
    uint32_t cached_tokens_ = 0xFFFFFFFFu;
    bool cached_col_major_ = true;
    cudaStream_t issue_stream_ = nullptr, owner_stream_ = nullptr;
    bool issue_captured_ = false;
    uint32_t tokens_ = 0;
    uint64_t fetches_ = 0, launches_ = 0;
    OwnerService service_;

    std::string describe_error() const {
        volatile ErrorRecord *e = host_error_;
        static const char *names[] = {"ok", "hook wait timed out", "index outside the vocabulary",
                                      "inbox overflow", "push bounds", "gather pipeline stalled",
                                      "device barrier timed out", "serving claim disagreed with the mailbox"};
        const uint32_t s = e->status;
        std::string what = s < 8 ? names[s] : "unknown error";
        return "Engram device error: " + what + " (layer " + std::to_string(e->layer) + ", owner " +
               std::to_string(e->owner) + ", observed " + std::to_string(e->observed) + ", expected " +
               std::to_string(e->expected) + ", reports " + std::to_string(e->count) + ")";
    }
};

} // namespace engram

#pragma GCC visibility pop

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    using namespace engram;
    m.doc() = "B200 Engram runtime: VMM shards, peer mappings, sm_100a gather/dispatch/push kernels";
    m.attr("MAX_RANKS") = kMaxRanks;
    m.attr("MAX_LAYERS") = kMaxLayers;
    m.attr("HEADER_BYTES") = kHeaderBytes;
    m.attr("MAX_PUSH_TASKS") = kMaxPushTasks;
    m.attr("KERNELS") = py::make_tuple("gather_simt_kernel", "gather_bulk_kernel", "dispatch_kernel", "push_kernel",
                                       "hook_kernel", "dedup_kernel", "expand_kernel", "litmus_kernel",
                                       "wait_probe_kernel", "stream_copy_kernel", "peer_probe_kernel",
                                       "barrier_kernel");
    py::class_<Runtime, std::shared_ptr<Runtime>>(m, "Runtime")
        .def(py::init<const py::dict &>())
        .def("bootstrap", &Runtime::bootstrap)
        .def("probe_routes", &Runtime::probe_routes)
        .def("prepare_routes", &Runtime::prepare_routes)
        .def("connect", &Runtime::connect)
        .def("write", &Runtime::write, py::arg("layer"), py::arg("storage"), py::arg("scales") = py::none())
        .def("fetch", &Runtime::fetch)
        .def("wait_layer", &Runtime::wait_layer)
        .def("fetch_all", &Runtime::fetch_all)
        .def("check_health", &Runtime::check_health)
        .def("barrier", &Runtime::barrier)
        .def("barrier_state", &Runtime::barrier_state)
        .def("error_state", &Runtime::error_state)
        .def("memory_usage", &Runtime::memory_usage)
        .def("debug_state", &Runtime::debug_state)
        .def("run_wait_probe", &Runtime::run_wait_probe)
        .def("debug_stop_service", &Runtime::debug_stop_service)
        .def("debug_peer_copy", &Runtime::debug_peer_copy)
        .def("debug_serve_local", &Runtime::debug_serve_local, py::arg("rows"), py::arg("worker") = "push",
             py::arg("blocks") = 8)
        .def("debug_peer_probe", &Runtime::debug_peer_probe, py::arg("mode_even"), py::arg("mode_odd"),
             py::arg("rows"), py::arg("blocks"), py::arg("even_share_pct") = 50, py::arg("seed") = 1)
        .def("debug_litmus_reset", &Runtime::debug_litmus_reset)
        .def("replica_view", &Runtime::replica_view)
        .def("read_layer", &Runtime::read_layer)
        .def("set_hot_active", &Runtime::set_hot_active)
        .def("debug_litmus", &Runtime::debug_litmus, py::arg("peer"), py::arg("role"), py::arg("epochs"),
             py::arg("words"), py::arg("ctas") = 32, py::arg("weak_loads") = false, py::arg("timeout_ms") = 2000.0)
        .def("close", &Runtime::close)
        .def_property_readonly("closed", &Runtime::closed);
    bind_ops(m);
    bind_harness(m);
}
