#include "host_memory.h"

#include <cstdlib>
#include <cstring>

#include <cuda_runtime_api.h>

namespace tutti {

bool cuda_device_present() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return n > 0;
}

Result<HostMappedBuffer> host_mapped_alloc(std::size_t bytes, bool write_combined) {
    HostMappedBuffer b;
    b.bytes = (bytes + 4095) & ~std::size_t(4095);
    if (b.bytes == 0) b.bytes = 4096;
    if (cuda_device_present()) {
        void* p = nullptr;
        cudaError_t e = cudaHostAlloc(&p, b.bytes,
                                      cudaHostAllocMapped | cudaHostAllocPortable |
                                          (write_combined ? cudaHostAllocWriteCombined : 0u));
        if (e != cudaSuccess) {
            cudaGetLastError();
            return Result<HostMappedBuffer>::Failure(
                {StatusCode::RESOURCE_EXHAUSTED,
                 std::string("cudaHostAlloc failed: ") + cudaGetErrorString(e)});
        }
        void* d = nullptr;
        e = cudaHostGetDevicePointer(&d, p, 0);
        if (e != cudaSuccess) {
            cudaFreeHost(p);
            cudaGetLastError();
            return Result<HostMappedBuffer>::Failure(
                {StatusCode::INTERNAL,
                 std::string("cudaHostGetDevicePointer failed: ") + cudaGetErrorString(e)});
        }
        std::memset(p, 0, b.bytes);
        b.host = p;
        b.device = d;
        b.cuda_pinned = true;
        return b;
    }
    void* p = nullptr;
    if (posix_memalign(&p, 4096, b.bytes) != 0 || p == nullptr)
        return Result<HostMappedBuffer>::Failure({StatusCode::RESOURCE_EXHAUSTED, "posix_memalign failed"});
    std::memset(p, 0, b.bytes);
    b.host = p;
    b.device = nullptr;
    b.cuda_pinned = false;
    return b;
}

void host_mapped_free(HostMappedBuffer& b) {
    if (b.host) {
        if (b.cuda_pinned)
            cudaFreeHost(b.host);
        else
            std::free(b.host);
    }
    b = HostMappedBuffer{};
}

}  // namespace tutti
