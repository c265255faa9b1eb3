#include "memory.h"

#include "driver.h"

#include <cuda_runtime.h>
#include <sys/mman.h>
#include <unistd.h>

#include <cstring>
#include <mutex>

namespace engram {

const DriverApi &driver() {
    static DriverApi api;
    static std::once_flag once;
    static std::string failure;
    std::call_once(once, [] {
        auto load = [](const char *name, auto &slot) {
            void *fn = nullptr;
            cudaDriverEntryPointQueryResult status{};
            cudaError_t rc = cudaGetDriverEntryPointByVersion(name, &fn, 12000, cudaEnableDefault, &status);
            if (rc != cudaSuccess || status != cudaDriverEntryPointSuccess || fn == nullptr) {
                cudaGetLastError();
                if (failure.empty())
                    failure = std::string("driver entry point ") + name + " unavailable";
                return;
            }
            slot = reinterpret_cast<std::remove_reference_t<decltype(slot)>>(fn);
        };
        load("cuMemCreate", api.MemCreate);
        load("cuMemRelease", api.MemRelease);
        load("cuMemAddressReserve", api.MemAddressReserve);
        load("cuMemAddressFree", api.MemAddressFree);
        load("cuMemMap", api.MemMap);
        load("cuMemUnmap", api.MemUnmap);
        load("cuMemSetAccess", api.MemSetAccess);
        load("cuMemGetAccess", api.MemGetAccess);
        load("cuMemExportToShareableHandle", api.MemExportToShareableHandle);
        load("cuMemImportFromShareableHandle", api.MemImportFromShareableHandle);
        load("cuMemGetAllocationGranularity", api.MemGetAllocationGranularity);
        load("cuDeviceGetAttribute", api.DeviceGetAttribute);
        load("cuGetErrorString", api.GetErrorString);
    });
    if (!failure.empty())
        throw std::runtime_error(failure);
    return api;
}

const char *memory_kind_name(MemoryKind kind) {
    switch (kind) {
    case MemoryKind::DeviceVmm: return "device_vmm";
    case MemoryKind::HostVmm: return "host_numa_vmm";
    case MemoryKind::HostMemfd: return "host_memfd_registered";
    }
    return "unknown";
}

namespace {

void unmap_release(CUdeviceptr ptr, size_t bytes, CUmemGenericAllocationHandle handle) noexcept {
    try {
        const auto &d = driver();
        if (ptr) {
            d.MemUnmap(ptr, bytes);
            d.MemAddressFree(ptr, bytes);
        }
        if (handle)
            d.MemRelease(handle);
    } catch (...) {
    }
}

int attr(CUdevice_attribute a, int device) {
    int v = 0;
    check_cu(driver().DeviceGetAttribute(&v, a, device), "cuDeviceGetAttribute");
    return v;
}

} // namespace

std::unique_ptr<SharedAllocation> SharedAllocation::device(size_t bytes, int device) {
    const auto &d = driver();
    std::unique_ptr<SharedAllocation> a(new SharedAllocation());
    a->kind_ = MemoryKind::DeviceVmm;
    a->device_ = device;
    check(attr(CU_DEVICE_ATTRIBUTE_VIRTUAL_MEMORY_MANAGEMENT_SUPPORTED, device) != 0,
          "device lacks virtual memory management");
    check(attr(CU_DEVICE_ATTRIBUTE_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR_SUPPORTED, device) != 0,
          "device cannot export POSIX file descriptors");
    CUmemAllocationProp prop{};
    prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    prop.location.id = device;
    prop.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    size_t gran = 0;
    check_cu(d.MemGetAllocationGranularity(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED), "granularity");
    a->bytes_ = align_up(bytes ? bytes : 1, gran);
    check_cu(d.MemCreate(&a->handle_, a->bytes_, &prop, 0), "cuMemCreate(device arena)");
    try {
        check_cu(d.MemAddressReserve(&a->ptr_, a->bytes_, gran, 0, 0), "reserve device arena");
        check_cu(d.MemMap(a->ptr_, a->bytes_, 0, a->handle_, 0), "map device arena");
        CUmemAccessDesc acc{};
        acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
        acc.location.id = device;
        acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
        check_cu(d.MemSetAccess(a->ptr_, a->bytes_, &acc, 1), "device arena access");
        check_cu(d.MemExportToShareableHandle(&a->fd_, a->handle_, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0),
                 "export device arena");
        check_cuda(cudaMemset(reinterpret_cast<void *>(a->ptr_), 0, a->bytes_), "clear device arena");
    } catch (...) {
        if (a->fd_ >= 0)
            ::close(a->fd_);
        unmap_release(a->ptr_, a->bytes_, a->handle_);
        a->ptr_ = 0;
        a->handle_ = 0;
        a->fd_ = -1;
        throw;
    }
    return a;
}

std::unique_ptr<SharedAllocation> SharedAllocation::host(size_t bytes, int device, bool allow_vmm) {
    std::unique_ptr<SharedAllocation> a(new SharedAllocation());
    a->device_ = device;
    bytes = bytes ? bytes : 1;
    const auto &d = driver();
    int numa = -1, numa_vmm = 0;
    try {
        numa = attr(CU_DEVICE_ATTRIBUTE_HOST_NUMA_ID, device);
        numa_vmm = attr(CU_DEVICE_ATTRIBUTE_HOST_NUMA_VIRTUAL_MEMORY_MANAGEMENT_SUPPORTED, device);
    } catch (const std::exception &) {
        numa_vmm = 0;
    }
    a->numa_ = numa;
    if (allow_vmm && numa_vmm && numa >= 0) {
        CUmemAllocationProp prop{};
        prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
        prop.location.type = CU_MEM_LOCATION_TYPE_HOST_NUMA;
        prop.location.id = numa;
        prop.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
        size_t gran = 0;
        CUresult rc = d.MemGetAllocationGranularity(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED);
        if (rc == CUDA_SUCCESS) {
            a->bytes_ = align_up(bytes, gran);
            rc = d.MemCreate(&a->handle_, a->bytes_, &prop, 0);
        }
        if (rc == CUDA_SUCCESS) {
            try {
                check_cu(d.MemAddressReserve(&a->ptr_, a->bytes_, gran, 0, 0), "reserve host shard");
                check_cu(d.MemMap(a->ptr_, a->bytes_, 0, a->handle_, 0), "map host shard");
                CUmemAccessDesc acc[2]{};
                acc[0].location.type = CU_MEM_LOCATION_TYPE_DEVICE;
                acc[0].location.id = device;
                acc[1].location.type = CU_MEM_LOCATION_TYPE_HOST_NUMA;
                acc[1].location.id = numa;
                acc[0].flags = acc[1].flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
                check_cu(d.MemSetAccess(a->ptr_, a->bytes_, acc, 2), "host shard access");
                check_cu(d.MemExportToShareableHandle(&a->fd_, a->handle_, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR,
                                                      0),
                         "export host shard");
                a->host_ptr_ = reinterpret_cast<void *>(a->ptr_);
                std::memset(a->host_ptr_, 0, a->bytes_);
                a->kind_ = MemoryKind::HostVmm;
                return a;
            } catch (const std::exception &e) {
                if (a->fd_ >= 0)
                    ::close(a->fd_);
                unmap_release(a->ptr_, a->bytes_, a->handle_);
                a->ptr_ = 0;
                a->handle_ = 0;
                a->fd_ = -1;
                a->note_ = std::string("HOST_NUMA VMM failed (") + e.what() + "); using memfd";
            }
        } else {
            a->note_ = "HOST_NUMA cuMemCreate rejected (" + std::to_string(int(rc)) + "); using memfd";
        }
    } else if (a->note_.empty()) {
        a->note_ = allow_vmm ? "HOST_NUMA VMM unsupported; using memfd" : "memfd requested";
    }
    // Fallback: shared memfd, mapped and registered (mapped, portable) by every process.
    a->kind_ = MemoryKind::HostMemfd;
    a->bytes_ = align_up(bytes, 2u << 20);
    a->fd_ = memfd_create("engram-host-shard", MFD_CLOEXEC);
    check(a->fd_ >= 0, "memfd_create failed");
    try {
        check(ftruncate(a->fd_, off_t(a->bytes_)) == 0, "ftruncate host shard");
        void *p = mmap(nullptr, a->bytes_, PROT_READ | PROT_WRITE, MAP_SHARED, a->fd_, 0);
        check(p != MAP_FAILED, "mmap host shard");
        a->host_ptr_ = p;
        check_cuda(cudaHostRegister(p, a->bytes_, cudaHostRegisterMapped | cudaHostRegisterPortable),
                   "register host shard");
        a->registered_ = true;
        void *dptr = nullptr;
        check_cuda(cudaHostGetDevicePointer(&dptr, p, 0), "host shard device pointer");
        a->ptr_ = reinterpret_cast<CUdeviceptr>(dptr);
    } catch (...) {
        if (a->registered_)
            cudaHostUnregister(a->host_ptr_);
        if (a->host_ptr_)
            munmap(a->host_ptr_, a->bytes_);
        ::close(a->fd_);
        a->fd_ = -1;
        a->host_ptr_ = nullptr;
        throw;
    }
    return a;
}

SharedAllocation::~SharedAllocation() {
    if (fd_ >= 0)
        ::close(fd_);
    if (kind_ == MemoryKind::HostMemfd) {
        if (registered_)
            cudaHostUnregister(host_ptr_);
        if (host_ptr_)
            munmap(host_ptr_, bytes_);
    } else {
        unmap_release(ptr_, bytes_, handle_);
    }
}

PeerMapping::PeerMapping(MemoryKind kind, int fd, size_t bytes, int device, int numa) : kind_(kind), bytes_(bytes) {
    struct Closer {
        int fd;
        ~Closer() {
            if (fd >= 0)
                ::close(fd);
        }
    } closer{fd};
    check(fd >= 0, "invalid peer file descriptor");
    check(bytes > 0, "invalid peer allocation size");
    if (kind == MemoryKind::HostMemfd) {
        void *p = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
        check(p != MAP_FAILED, "mmap peer host shard");
        host_ptr_ = p;
        cudaError_t rc = cudaHostRegister(p, bytes, cudaHostRegisterMapped | cudaHostRegisterPortable);
        if (rc != cudaSuccess) {
            munmap(p, bytes);
            host_ptr_ = nullptr;
            check_cuda(rc, "register peer host shard");
        }
        registered_ = true;
        void *dptr = nullptr;
        check_cuda(cudaHostGetDevicePointer(&dptr, p, 0), "peer host shard device pointer");
        ptr_ = reinterpret_cast<CUdeviceptr>(dptr);
        return;
    }
    const auto &d = driver();
    check_cu(d.MemImportFromShareableHandle(&handle_, reinterpret_cast<void *>(intptr_t(fd)),
                                            CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR),
             "import peer allocation");
    try {
        check_cu(d.MemAddressReserve(&ptr_, bytes_, 0, 0, 0), "reserve peer mapping");
        check_cu(d.MemMap(ptr_, bytes_, 0, handle_, 0), "map peer allocation");
        CUmemAccessDesc acc[2]{};
        acc[0].location.type = CU_MEM_LOCATION_TYPE_DEVICE;
        acc[0].location.id = device;
        acc[0].flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
        int count = 1;
        if (kind == MemoryKind::HostVmm) {
            acc[1].location.type = CU_MEM_LOCATION_TYPE_HOST_NUMA;
            acc[1].location.id = numa;
            acc[1].flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
            count = 2;
        }
        check_cu(d.MemSetAccess(ptr_, bytes_, acc, count), "peer mapping access");
    } catch (...) {
        unmap_release(ptr_, bytes_, handle_);
        ptr_ = 0;
        handle_ = 0;
        throw;
    }
}

bool PeerMapping::readable(size_t offset, int device) const {
    if (kind_ == MemoryKind::HostMemfd)
        return ptr_ != 0;
    CUmemLocation loc{};
    loc.type = CU_MEM_LOCATION_TYPE_DEVICE;
    loc.id = device;
    unsigned long long flags = 0;
    if (driver().MemGetAccess(&flags, &loc, ptr_ + offset) != CUDA_SUCCESS)
        return false;
    return (flags & CU_MEM_ACCESS_FLAGS_PROT_READ) != 0;
}

PeerMapping::~PeerMapping() {
    if (kind_ == MemoryKind::HostMemfd) {
        if (registered_)
            cudaHostUnregister(host_ptr_);
        if (host_ptr_)
            munmap(host_ptr_, bytes_);
    } else {
        unmap_release(ptr_, bytes_, handle_);
    }
}

} // namespace engram
