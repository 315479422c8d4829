// Cross-GPU ready flags: ordering between ranks without a host round trip.
//
// Each rank owns a board of 64-bit flag words in its own HBM; every peer maps
// it through CUDA IPC. A producer rank, after its work on a stream (e.g. the
// io kernel that stored a layer into the peers' pools over NVLink), launches
// ready_signal_kernel on the same stream: a system-scope fence (the earlier
// kernel's peer stores are performed first) and a release store of `value`
// into its word of the slot on every board. A consumer launches
// ready_wait_kernel on the stream that will read the data: one thread spins
// with acquire loads until every producer's word of the slot holds at least
// `value`, bounded by a %globaltimer deadline; on expiry it records the
// producers it was still waiting for in a host-visible status word and
// returns, so the stream never hangs and the host decides what to do.
//
// Signal and wait run on different GPUs (one process per GPU); on one GPU a
// wait is only ever paired with a flag that is already set or never set.
//
// Parity: the reference orders replica consumers with interprocess CUDA
// events and a TCPStore handshake (tutti/storage/tutti_nvme/replica_direct.py:
// 82-190, 700-742); this replaces both with device-side flags.

#include <cstdint>

#include <cuda_runtime.h>

#include "ops_kernels.h"

namespace tutti {
namespace ops {

namespace {

__device__ __forceinline__ unsigned long long now_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ std::uint64_t load_acquire_sys(const std::uint64_t* p) {
    std::uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void store_release_sys(std::uint64_t* p, std::uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__global__ void ready_signal_kernel(std::uint64_t* const* targets, std::uint32_t n, std::uint64_t value) {
    if (threadIdx.x != 0) return;
    asm volatile("fence.sc.sys;" ::: "memory");  // earlier work's stores before the flags
    for (std::uint32_t i = 0; i < n; ++i) store_release_sys(targets[i], value);
}

// status: 0 = every producer reached `value`; otherwise bit r set for each
// producer r (r < 32) still below it at the deadline, or 1u << 31 for r >= 32.
__global__ void ready_wait_kernel(const std::uint64_t* words, std::uint32_t n, std::uint64_t value,
                                  std::uint64_t timeout_ns, std::uint32_t* status) {
    if (threadIdx.x != 0) return;
    const unsigned long long deadline = now_ns() + timeout_ns;
    std::uint32_t sleep = 32;
    for (;;) {
        std::uint32_t missing = 0;
        for (std::uint32_t r = 0; r < n; ++r)
            if (load_acquire_sys(words + r) < value) missing |= r < 31 ? (1u << r) : (1u << 31);
        if (missing == 0) {
            *reinterpret_cast<volatile std::uint32_t*>(status) = 0;
            return;
        }
        if (now_ns() > deadline) {
            *reinterpret_cast<volatile std::uint32_t*>(status) = missing;
            __threadfence_system();
            return;
        }
        __nanosleep(sleep);
        if (sleep < 2048) sleep <<= 1;
    }
}

}  // namespace

cudaError_t launch_ready_signal(std::uint64_t* const* targets, std::uint32_t n, std::uint64_t value,
                                cudaStream_t stream) {
    ready_signal_kernel<<<1, 32, 0, stream>>>(targets, n, value);
    return cudaGetLastError();
}

cudaError_t launch_ready_wait(const std::uint64_t* words, std::uint32_t n, std::uint64_t value,
                              std::uint64_t timeout_ns, std::uint32_t* status, cudaStream_t stream) {
    ready_wait_kernel<<<1, 32, 0, stream>>>(words, n, value, timeout_ns, status);
    return cudaGetLastError();
}

}  // namespace ops
}  // namespace tutti
