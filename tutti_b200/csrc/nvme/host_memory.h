#pragma once
// Host memory the GPU can reach: page-locked, mapped into the device address
// space (zero-copy). Used for NVMe queue rings, doorbells, PRP lists and the
// staging arena. Falls back to plain aligned host memory when no CUDA device is
// present so the host-side protocol (emulated controller, host submitter) is
// testable on CPU-only machines.

#include <cstddef>
#include <cstdint>

#include <tutti/status.h>

namespace tutti {

struct HostMappedBuffer {
    void* host = nullptr;    // CPU address
    void* device = nullptr;  // device address of the same bytes (nullptr without CUDA)
    std::size_t bytes = 0;
    bool cuda_pinned = false;

    template <typename T>
    T* host_as() const { return static_cast<T*>(host); }
    template <typename T>
    T* device_as() const { return static_cast<T*>(device); }
};

// True when the CUDA runtime reports at least one device.
bool cuda_device_present();

// Allocates `bytes` (rounded up to 4 KiB) zero-filled. With a CUDA device the
// memory is cudaHostAllocMapped|Portable; otherwise 4 KiB-aligned heap memory.
// write_combined: CPU stores stream without reading the lines first and the
// GPU reads them without snooping the CPU caches; CPU reads of it are slow.
Result<HostMappedBuffer> host_mapped_alloc(std::size_t bytes, bool write_combined = false);
void host_mapped_free(HostMappedBuffer& buf);

}  // namespace tutti
