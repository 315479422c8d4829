// SM-filling persistent compute kernel for the io interference benchmark: it
// stands in for a persistent GEMM that keeps every SM busy while restores run.
// Each thread runs four independent FMA chains for a fixed number of
// iterations, so its duration depends only on how much of each SM it gets.
//
// Parity: reference examples/nvme_bw_probe/async_completion_bench_kernels.cu:43
// (persistent_compute, grid = number of SMs).

#include "ops_kernels.h"

namespace tutti {
namespace ops {

namespace {

__global__ void __launch_bounds__(256) persistent_fma_kernel(float* out, std::uint64_t iters) {
    float a = 1.0f + threadIdx.x * 1e-3f, b = 0.5f + blockIdx.x * 1e-4f;
    float c0 = 0.f, c1 = 1.f, c2 = 2.f, c3 = 3.f;
    for (std::uint64_t i = 0; i < iters; ++i) {
#pragma unroll 8
        for (int k = 0; k < 8; ++k) {
            c0 = fmaf(a, c0, b);
            c1 = fmaf(b, c1, a);
            c2 = fmaf(a, c2, -b);
            c3 = fmaf(-b, c3, a);
        }
        a = fmaf(c0, 1e-12f, a);  // loop-carried, so nothing can be hoisted
    }
    const float r = c0 + c1 + c2 + c3;
    if (r == 1234.5f) out[blockIdx.x * blockDim.x + threadIdx.x] = r;  // keeps the chains live
}

}  // namespace

cudaError_t launch_persistent_fma(float* out, std::uint64_t iters, std::uint32_t blocks, cudaStream_t stream) {
    if (blocks == 0) return cudaSuccess;
    persistent_fma_kernel<<<blocks, 256, 0, stream>>>(out, iters);
    return cudaGetLastError();
}

}  // namespace ops
}  // namespace tutti
