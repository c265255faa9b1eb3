// CUDA driver entry points resolved at run time through the runtime API.
//
// The extension never links libcuda, so it imports on machines without a GPU
// driver (the CPU unit tests) and always uses the driver that the CUDA runtime
// already loaded.  Only the virtual-memory-management calls are needed: the
// host shard and device arena are cuMemCreate allocations exported as POSIX
// file descriptors and mapped by every peer on the node.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

namespace engram {

struct DriverApi {
    decltype(&::cuMemCreate) MemCreate = nullptr;
    decltype(&::cuMemRelease) MemRelease = nullptr;
    decltype(&::cuMemAddressReserve) MemAddressReserve = nullptr;
    decltype(&::cuMemAddressFree) MemAddressFree = nullptr;
    decltype(&::cuMemMap) MemMap = nullptr;
    decltype(&::cuMemUnmap) MemUnmap = nullptr;
    decltype(&::cuMemSetAccess) MemSetAccess = nullptr;
    decltype(&::cuMemGetAccess) MemGetAccess = nullptr;
    decltype(&::cuMemExportToShareableHandle) MemExportToShareableHandle = nullptr;
    decltype(&::cuMemImportFromShareableHandle) MemImportFromShareableHandle = nullptr;
    decltype(&::cuMemGetAllocationGranularity) MemGetAllocationGranularity = nullptr;
    decltype(&::cuDeviceGetAttribute) DeviceGetAttribute = nullptr;
    decltype(&::cuGetErrorString) GetErrorString = nullptr;
};

// Loads the table once; throws if the runtime cannot provide a symbol.
const DriverApi &driver();

inline void check_cu(CUresult rc, const char *what) {
    if (rc != CUDA_SUCCESS) {
        const char *s = nullptr;
        if (driver().GetErrorString)
            driver().GetErrorString(rc, &s);
        throw std::runtime_error(std::string(what) + ": " + (s ? s : "CUDA driver error") + " (" +
                                 std::to_string(int(rc)) + ")");
    }
}

inline void check_cuda(cudaError_t rc, const char *what) {
    if (rc != cudaSuccess)
        throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(rc));
}

inline void check(bool ok, const std::string &what) {
    if (!ok)
        throw std::runtime_error(what);
}

inline size_t align_up(size_t n, size_t a) { return (n + a - 1) / a * a; }

} // namespace engram
