#pragma once
// Launch entry points of the torch-facing sm_100a kernels (tutti_b200._ops).

#include <cstdint>

#include <cuda_runtime_api.h>

namespace tutti {
namespace ops {

struct CopyItem {  // 24 B
    std::uint64_t src;
    std::uint64_t dst;
    std::uint32_t bytes;  // multiple of 16; src/dst 16-byte aligned
    std::uint32_t pad;
};

// Batched copy; tma=true for local HBM (bulk-async), false for peer memory.
cudaError_t launch_copy_items(const CopyItem* items, std::uint32_t n, bool tma, std::uint32_t* error,
                              int sm_count, cudaStream_t stream);

// fp8 E4M3 with one fp32 scale per `group` consecutive elements of a row.
// in_dtype/out_dtype: 0 = bf16, 1 = fp32, 2 = fp16.
cudaError_t launch_fp8_quant(const void* x, int in_dtype, std::uint8_t* q, float* scale, std::uint64_t rows,
                             std::uint32_t cols, std::uint32_t group, int sm_count, cudaStream_t stream);
cudaError_t launch_fp8_dequant(const std::uint8_t* q, const float* scale, void* x, int out_dtype,
                               std::uint64_t rows, std::uint32_t cols, std::uint32_t group, int sm_count,
                               cudaStream_t stream);

// Paged fp8 transforms: rows of `cols` bf16 values at pool + row_offsets[i]
// (byte offsets) <-> dense fp8 rows + scales.
cudaError_t launch_fp8_gather_quant(const std::uint8_t* pool, const std::int64_t* row_offsets, std::uint64_t rows,
                                    std::uint32_t cols, std::uint8_t* q, float* scale, cudaStream_t stream);
cudaError_t launch_fp8_dequant_scatter(const std::uint8_t* q, const float* scale, std::uint8_t* pool,
                                       const std::int64_t* row_offsets, std::uint64_t rows, std::uint32_t cols,
                                       cudaStream_t stream);

// Chained BLAKE2b-128 chunk keys (RFC 7693), one request per thread.
// tokens: concatenated int64 token ids; starts[r] / lengths[r] per request;
// parents: 16-byte parent per request (used when parent_len[r] == 16, else the
// chain starts from the empty namespace); keys out: [sum chunks, 16] bytes at
// key_offsets[r] (in keys).
cudaError_t launch_prefix_hash(const std::int64_t* tokens, const std::int64_t* starts, const std::int64_t* lengths,
                               const std::uint8_t* parents, const std::int32_t* parent_len,
                               const std::int64_t* key_offsets, std::uint8_t* keys, std::uint32_t requests,
                               std::uint32_t chunk_tokens, cudaStream_t stream);

// 64-bit order-sensitive checksum of each item (bytes multiple of 8).
cudaError_t launch_checksum(const CopyItem* items, std::uint32_t n, std::uint64_t* out, cudaStream_t stream);
// Same digests when every item has `bytes` bytes (a multiple of 16, 16-byte aligned sources).
cudaError_t launch_checksum_uniform(const CopyItem* items, std::uint32_t n, std::uint64_t bytes, std::uint64_t* out,
                                    cudaStream_t stream);

// SM-filling compute stand-in for the interference benchmark: `blocks` CTAs of
// 256 threads, each thread running `iters` x 32 FMAs. `out` (blocks x 256
// floats) is written only if the chains hit an impossible value.
cudaError_t launch_persistent_fma(float* out, std::uint64_t iters, std::uint32_t blocks, cudaStream_t stream);

// Cross-GPU ready flags (ready_flags.cu): store `value` (system-scope release,
// after a system fence) into each of `targets` (device array of n pointers,
// peers' board words mapped through IPC); wait until all n words of `words`
// reach `value` or `timeout_ns` passes (status: 0, or a mask of the words
// still below; `status` may be host-mapped memory).
cudaError_t launch_ready_signal(std::uint64_t* const* targets, std::uint32_t n, std::uint64_t value,
                                cudaStream_t stream);
cudaError_t launch_ready_wait(const std::uint64_t* words, std::uint32_t n, std::uint64_t value,
                              std::uint64_t timeout_ns, std::uint32_t* status, cudaStream_t stream);

}  // namespace ops
}  // namespace tutti
