// Standalone operators of the extension: the per-owner request pack (the
// dispatch kernel aimed at caller-owned buffers), zero-copy host reads and
// writes by SM loads and stores through pinned memory's device mapping (the
// PCIe envelope of kernels that read pinned host memory; small results to the
// host without a copy engine) and the NVTX switch.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include <vector>

#include "bindings.h"
#include "driver.h"
#include "kernels/params.h"
#include "trace.h"

namespace py = pybind11;

namespace engram {

namespace {

// Standalone per-owner pack (the dispatch kernel aimed at local buffers).
// packed: int64 [world, layers, capacity]; counts: int32 [layers, world];
// scratch: int32 with at least layers * world * 4 + layers elements, owned by
// the caller (cursors, arrival counters, epochs).  Owners with owners[o] == 0
// are skipped.  Within one owner the order of entries is not specified.
void route_pack(const torch::Tensor &indices, const std::vector<uint32_t> &entries, uint32_t world,
                const std::vector<uint8_t> &owners, torch::Tensor &packed, torch::Tensor &counts,
                torch::Tensor &scratch) {
    check(indices.is_cuda() && indices.dim() == 3 && indices.scalar_type() == torch::kInt && indices.is_contiguous(),
          "indices must be contiguous CUDA int32 [layers, tokens, ept]");
    const uint32_t layers = uint32_t(indices.size(0)), rows = uint32_t(indices.size(1) * indices.size(2));
    check(layers >= 1 && layers <= kMaxLayers && entries.size() == layers, "layers");
    check(world >= 1 && world <= kMaxRanks && owners.size() == world, "world");
    check(packed.is_cuda() && packed.scalar_type() == torch::kLong && packed.is_contiguous() && packed.dim() == 3 &&
              packed.size(0) == world && packed.size(1) == layers && packed.size(2) >= rows,
          "packed must be contiguous CUDA int64 [world, layers, capacity >= tokens*ept]");
    check(counts.is_cuda() && counts.scalar_type() == torch::kInt && counts.is_contiguous() &&
              counts.numel() == int64_t(layers) * world,
          "counts must be contiguous CUDA int32 [layers, world]");
    const size_t lw = size_t(layers) * world;
    check(scratch.is_cuda() && scratch.scalar_type() == torch::kInt && scratch.is_contiguous() &&
              size_t(scratch.numel()) >= lw * 4 + layers,
          "scratch must be contiguous CUDA int32 with layers*world*4 + layers elements");
    const int dev = indices.get_device();
    check(packed.get_device() == dev && counts.get_device() == dev && scratch.get_device() == dev, "devices");
    c10::cuda::CUDAGuard guard(dev);
    cudaStream_t s = at::cuda::getCurrentCUDAStream(dev).stream();
    DispatchParams d{};
    uint32_t at = 0;
    for (uint32_t l = 0; l < layers; ++l) {
        check(entries[l] > 0 && uint64_t(entries[l]) * world <= 0x7FFFFFFFull, "entries");
        d.layer.entries[l] = entries[l];
        d.layer.table_bases[l] = at;
        at += entries[l];
    }
    uint32_t *base = reinterpret_cast<uint32_t *>(scratch.data_ptr<int32_t>());
    d.epochs = reinterpret_cast<uint64_t *>(base);  // 2 * lw words
    d.cursors = base + 2 * lw;                      // lw words
    d.layer_arrivals = base + 3 * lw;               // layers words
    d.totals = reinterpret_cast<uint32_t *>(counts.data_ptr<int32_t>());
    d.error = ErrorSink{nullptr, nullptr};
    const uint64_t cap = uint64_t(packed.size(2));
    for (uint32_t o = 0; o < world; ++o)
        d.inbox_base[o] =
            owners[o] ? reinterpret_cast<uint64_t>(packed.data_ptr<int64_t>()) + uint64_t(o) * layers * cap * 8 : 0;
    d.indices = indices.data_ptr<int32_t>();
    d.layers = layers;
    d.rows = rows;
    d.capacity = uint32_t(cap);
    d.world = world;
    d.rank = 0;
    d.channels = 1;
    d.tile_rows = 512;
    check_cuda(cudaMemsetAsync(d.cursors, 0, (lw + layers) * 4, s), "clear pack scratch");
    if (rows == 0) {
        check_cuda(cudaMemsetAsync(d.totals, 0, lw * 4, s), "clear counts");
        return;
    }
    check_cuda(launch_dispatch(d, s), "launch route pack");
}


// Streams `src` (pinned host memory, read in place through its device
// mapping with 16-byte SM loads) into `dst` (this GPU) on the current stream.
// Both are contiguous with the same byte size, a multiple of 16.
void host_read(const torch::Tensor &src, torch::Tensor &dst, int blocks) {
    check(src.is_cpu() && src.is_contiguous() && dst.is_cuda() && dst.is_contiguous() && src.nbytes() == dst.nbytes() &&
              src.nbytes() % 16 == 0 && blocks >= 1 && blocks <= 65535,
          "host_read: pinned contiguous source and a CUDA destination of the same size (16-byte multiple)");
    cudaPointerAttributes attr{};
    const bool mapped = cudaPointerGetAttributes(&attr, src.data_ptr()) == cudaSuccess &&
                        attr.type == cudaMemoryTypeHost && attr.devicePointer != nullptr;
    if (!mapped) {
        cudaGetLastError();
        check(false, "host_read: the source must be pinned (page-locked, mapped) host memory");
    }
    c10::cuda::CUDAGuard guard(dst.get_device());
    cudaStream_t s = at::cuda::getCurrentCUDAStream(dst.get_device()).stream();
    check_cuda(launch_stream_copy(attr.devicePointer, dst.data_ptr(), uint64_t(src.nbytes()), blocks, s),
               "launch host read");
}

// Streams `src` (this GPU) into `dst` (pinned host memory, written in place
// through its device mapping with 16-byte SM stores) on the current stream.
// A device-to-host transfer that needs no copy engine: a small result can
// leave the GPU every step without queueing behind copies of the next step's
// inputs.  Both are contiguous with the same byte size, a multiple of 16.
void host_write(const torch::Tensor &src, torch::Tensor &dst, int blocks) {
    check(dst.is_cpu() && dst.is_contiguous() && src.is_cuda() && src.is_contiguous() && src.nbytes() == dst.nbytes() &&
              src.nbytes() % 16 == 0 && blocks >= 1 && blocks <= 65535,
          "host_write: a CUDA source and a pinned contiguous destination of the same size (16-byte multiple)");
    cudaPointerAttributes attr{};
    const bool mapped = cudaPointerGetAttributes(&attr, dst.data_ptr()) == cudaSuccess &&
                        attr.type == cudaMemoryTypeHost && attr.devicePointer != nullptr;
    if (!mapped) {
        cudaGetLastError();
        check(false, "host_write: the destination must be pinned (page-locked, mapped) host memory");
    }
    c10::cuda::CUDAGuard guard(src.get_device());
    cudaStream_t s = at::cuda::getCurrentCUDAStream(src.get_device()).stream();
    check_cuda(launch_stream_copy(src.data_ptr(), attr.devicePointer, uint64_t(src.nbytes()), blocks, s),
               "launch host write");
}

// Pinned, device-mapped host memory as a CPU uint8 tensor that frees itself
// (cudaFreeHost) when its storage goes.  With `write_combined` the pages are
// write-combined: the CPU writes them without filling its caches and the
// device reads them without snooping the CPU's caches, which is what an input
// buffer that the host writes and the GPU reads every step wants (CPU reads of
// it are slow).
torch::Tensor alloc_pinned(int64_t nbytes, bool write_combined) {
    check(nbytes > 0, "alloc_pinned: size must be positive");
    void *ptr = nullptr;
    const unsigned flags =
        cudaHostAllocMapped | cudaHostAllocPortable | (write_combined ? cudaHostAllocWriteCombined : 0u);
    check_cuda(cudaHostAlloc(&ptr, size_t(nbytes), flags), "alloc_pinned");
    return torch::from_blob(ptr, {nbytes}, [](void *p) { cudaFreeHost(p); },
                            torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCPU));
}

} // namespace

void bind_ops(py::module_ &m) {
    m.def("alloc_pinned", &alloc_pinned, py::arg("nbytes"), py::arg("write_combined") = true);
    m.def("host_write", &host_write, py::arg("src"), py::arg("dst"), py::arg("blocks") = 1);
    m.def("host_read", &host_read, py::arg("src"), py::arg("dst"), py::arg("blocks") = 592);
    m.def("route_pack", &route_pack, py::arg("indices"), py::arg("entries"), py::arg("world"), py::arg("owners"),
          py::arg("packed"), py::arg("counts"), py::arg("scratch"));
    m.def("set_nvtx", [](bool on) { nvtx_enabled().store(on); }, py::arg("enabled"),
          "Enable NVTX ranges around fetch, hook, write and owner-service launches.");
    m.def("nvtx_enabled", []() { return nvtx_enabled().load(); });
}

} // namespace engram
