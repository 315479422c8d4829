// Batched page copy for sm_100a: the staged paged gather/scatter and the
// peer page pull, as one kernel over (src, dst, bytes) items.
//
// Local HBM (tma path): a persistent grid, one warp per CTA; lane 0 streams
// 16 KiB chunks through a 4-stage shared-memory ring with bulk-async copies
// (cp.async.bulk global->shared completing on an mbarrier, then
// cp.async.bulk shared->global in bulk groups), so each CTA keeps 64 KiB in
// flight with one issuing thread and no register traffic. Each copy targets
// the issuing CTA's own shared memory only.
// Peer memory (simt path): 16-byte vector loads/stores by all threads; used
// when a source or destination is another GPU's memory reached over NVLink.
//
// Parity: reference csrc/kv_transfer/src/mem_kernels.cu:66-130
// (single_layer_kv_transfer_kernel, one block per token, 64-bit words) and
// :373-387 (replica_page_scatter_kernel, peer pages over IPC mappings).

#include "ops_kernels.h"
#include "primitives.cuh"

namespace tutti {
namespace ops {

namespace {

constexpr int kStages = 4;
constexpr std::uint32_t kChunk = 16384;
constexpr std::uint32_t kWaitLimit = 1u << 26;

struct ChunkIter {
    const CopyItem* items;
    std::uint32_t n, step, item;
    std::uint32_t off;
    __device__ bool next(std::uint64_t& src, std::uint64_t& dst, std::uint32_t& bytes) {
        while (item < n) {
            const CopyItem it = items[item];
            if (off < it.bytes) {
                bytes = min(kChunk, it.bytes - off);
                src = it.src + off;
                dst = it.dst + off;
                off += bytes;
                return true;
            }
            item += step;
            off = 0;
        }
        return false;
    }
};

__global__ void __launch_bounds__(32) bulk_copy_kernel(const CopyItem* items, std::uint32_t n,
                                                       std::uint32_t* error) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) std::uint64_t bars[kStages];
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) dev::mbar_init(&bars[s], 1);
        dev::fence_barrier_init();
    }
    __syncwarp();
    if (threadIdx.x != 0) return;
    ChunkIter load{items, n, gridDim.x, blockIdx.x, 0};
    std::uint64_t dst_of[kStages];
    std::uint32_t bytes_of[kStages];
    std::uint32_t phase_bits = 0;
    int in_flight = 0, head = 0, tail = 0;  // stages are filled and drained in ring order
    // prologue
    while (in_flight < kStages) {
        std::uint64_t s, d;
        std::uint32_t b;
        if (!load.next(s, d, b)) break;
        dev::mbar_arrive_expect_tx(&bars[tail], b);
        dev::bulk_g2s(smem + tail * kChunk, reinterpret_cast<const void*>(s), b, &bars[tail]);
        dst_of[tail] = d;
        bytes_of[tail] = b;
        tail = (tail + 1) % kStages;
        ++in_flight;
    }
    while (in_flight > 0) {
        const std::uint32_t ph = (phase_bits >> head) & 1u;
        if (!dev::mbar_wait_bounded(&bars[head], ph, kWaitLimit)) {
            atomicOr(error, 1u);
            dev::bulk_wait<0>();
            return;
        }
        phase_bits ^= 1u << head;
        dev::bulk_s2g(reinterpret_cast<void*>(dst_of[head]), smem + head * kChunk, bytes_of[head]);
        dev::bulk_commit();
        --in_flight;
        // stage `head` is reused once this store has read it
        std::uint64_t s, d;
        std::uint32_t b;
        if (load.next(s, d, b)) {
            dev::bulk_wait_read<0>();
            dev::mbar_arrive_expect_tx(&bars[head], b);
            dev::bulk_g2s(smem + head * kChunk, reinterpret_cast<const void*>(s), b, &bars[head]);
            dst_of[head] = d;
            bytes_of[head] = b;
            ++in_flight;
        }
        head = (head + 1) % kStages;
    }
    dev::bulk_wait<0>();
}

__global__ void __launch_bounds__(512) simt_copy_kernel(const CopyItem* items, std::uint32_t n) {
    for (std::uint32_t i = blockIdx.x; i < n; i += gridDim.x) {
        const CopyItem it = items[i];
        const char* s = reinterpret_cast<const char*>(it.src);
        char* d = reinterpret_cast<char*>(it.dst);
        const std::uint32_t units = it.bytes >> 4;
        std::uint32_t u = threadIdx.x;
        for (; u + 3 * blockDim.x < units; u += 4 * blockDim.x) {
            uint4 v0 = *reinterpret_cast<const uint4*>(s + (std::uint64_t(u) << 4));
            uint4 v1 = *reinterpret_cast<const uint4*>(s + (std::uint64_t(u + blockDim.x) << 4));
            uint4 v2 = *reinterpret_cast<const uint4*>(s + (std::uint64_t(u + 2 * blockDim.x) << 4));
            uint4 v3 = *reinterpret_cast<const uint4*>(s + (std::uint64_t(u + 3 * blockDim.x) << 4));
            *reinterpret_cast<uint4*>(d + (std::uint64_t(u) << 4)) = v0;
            *reinterpret_cast<uint4*>(d + (std::uint64_t(u + blockDim.x) << 4)) = v1;
            *reinterpret_cast<uint4*>(d + (std::uint64_t(u + 2 * blockDim.x) << 4)) = v2;
            *reinterpret_cast<uint4*>(d + (std::uint64_t(u + 3 * blockDim.x) << 4)) = v3;
        }
        for (; u < units; u += blockDim.x)
            *reinterpret_cast<uint4*>(d + (std::uint64_t(u) << 4)) =
                *reinterpret_cast<const uint4*>(s + (std::uint64_t(u) << 4));
    }
}

}  // namespace

cudaError_t launch_copy_items(const CopyItem* items, std::uint32_t n, bool tma, std::uint32_t* error,
                              int sm_count, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    if (tma) {
        const int smem = kStages * kChunk;
        cudaError_t e = cudaFuncSetAttribute(bulk_copy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        const std::uint32_t grid = std::min<std::uint32_t>(n, static_cast<std::uint32_t>(sm_count) * 3);
        bulk_copy_kernel<<<grid, 32, smem, stream>>>(items, n, error);
    } else {
        const std::uint32_t grid = std::min<std::uint32_t>(n, static_cast<std::uint32_t>(sm_count) * 4);
        simt_copy_kernel<<<grid, 512, 0, stream>>>(items, n);
    }
    return cudaGetLastError();
}

}  // namespace ops
}  // namespace tutti
