// Exportable allocations and their peer mappings.
//
// Parity: the reference's `HostMemory` / `HostAlias` / `FabricAlias`
// (sge_write/csrc/storage.hpp:26-209) and `EngramHostMemory`
// (deepep/csrc/buffers/engram_storage.hpp).  Differences by design:
//   * besides the host-pinned vocabulary shard, every rank exports a device
//     arena (HBM mirror, inbox, outputs, done flags) that peers map through
//     NVLink; on one NVSwitch node this replaces the NIC windows;
//   * when the driver lacks HOST_NUMA virtual-memory support the host shard
//     falls back to a memfd that every process maps and registers with CUDA,
//     so the same shared pages are still visible to every GPU;
//   * file descriptors travel over Unix-domain sockets (fdpass.h) instead of
//     pidfd_getfd, which needs ptrace rights that containers usually drop.
#pragma once

#include <cuda.h>

#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>

namespace engram {

enum class MemoryKind : int { DeviceVmm = 0, HostVmm = 1, HostMemfd = 2 };

const char *memory_kind_name(MemoryKind kind);

// An allocation owned by this process and exportable to peers on the node.
class SharedAllocation {
  public:
    static std::unique_ptr<SharedAllocation> device(size_t bytes, int device);
    // Host-pinned memory near `device`.  `allow_vmm=false` forces the memfd path.
    static std::unique_ptr<SharedAllocation> host(size_t bytes, int device, bool allow_vmm = true);
    ~SharedAllocation();
    SharedAllocation(const SharedAllocation &) = delete;
    SharedAllocation &operator=(const SharedAllocation &) = delete;

    MemoryKind kind() const { return kind_; }
    CUdeviceptr ptr() const { return ptr_; }         // device-visible address
    void *host_ptr() const { return host_ptr_; }     // CPU address (host kinds only)
    size_t bytes() const { return bytes_; }
    int fd() const { return fd_; }
    int numa() const { return numa_; }
    const std::string &note() const { return note_; }

  private:
    SharedAllocation() = default;
    MemoryKind kind_ = MemoryKind::DeviceVmm;
    CUdeviceptr ptr_ = 0;
    void *host_ptr_ = nullptr;
    size_t bytes_ = 0;
    CUmemGenericAllocationHandle handle_ = 0;
    int fd_ = -1, numa_ = -1, device_ = -1;
    bool registered_ = false;
    std::string note_;
};

// A peer's allocation mapped into this process for this process's GPU.
class PeerMapping {
  public:
    // Takes ownership of `fd` (closed before returning or on failure).
    PeerMapping(MemoryKind kind, int fd, size_t bytes, int device, int numa);
    ~PeerMapping();
    PeerMapping(const PeerMapping &) = delete;
    PeerMapping &operator=(const PeerMapping &) = delete;

    CUdeviceptr ptr() const { return ptr_; }
    size_t bytes() const { return bytes_; }
    MemoryKind kind() const { return kind_; }
    // True if this GPU's mapping at [ptr()+offset] grants read access.
    bool readable(size_t offset, int device) const;

  private:
    MemoryKind kind_;
    CUdeviceptr ptr_ = 0;
    void *host_ptr_ = nullptr;
    size_t bytes_ = 0;
    CUmemGenericAllocationHandle handle_ = 0;
    bool registered_ = false;
};

} // namespace engram
