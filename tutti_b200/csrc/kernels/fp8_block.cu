// Block-scaled fp8 (E4M3, one fp32 scale per 1x128 group) for sm_100a.
//
// One warp owns one 128-element group: each lane holds 4 consecutive values,
// the group's absolute maximum is a warp xor-shuffle reduction, the scale is
// amax / 448 (the E4M3 finite maximum), and values are converted with CUDA's
// saturating fp8 conversion intrinsics. The paged variants read or write the
// bf16 rows in place in the paged pool (row byte offsets), so quantisation
// runs fused with the gather of a store and dequantisation with the scatter
// of a restore: no dense bf16 copy is materialised.
// The reference only copies the fp8 index-cache bytes it is given
// (csrc/kv_transfer/include/engine_kv_format.h:125-126); quantisation is new.

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "ops_kernels.h"

namespace tutti {
namespace ops {

namespace {

constexpr float kE4M3Max = 448.0f;

__device__ __forceinline__ void load4(const void* base, int dtype, std::uint64_t idx, float v[4]) {
    if (dtype == 0) {
        const uint2 raw = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(base) + idx);
        const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
        const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
        const float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
        v[0] = fa.x, v[1] = fa.y, v[2] = fb.x, v[3] = fb.y;
    } else if (dtype == 2) {
        const uint2 raw = *reinterpret_cast<const uint2*>(static_cast<const __half*>(base) + idx);
        const float2 fa = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
        const float2 fb = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
        v[0] = fa.x, v[1] = fa.y, v[2] = fb.x, v[3] = fb.y;
    } else {
        const float4 f = *reinterpret_cast<const float4*>(static_cast<const float*>(base) + idx);
        v[0] = f.x, v[1] = f.y, v[2] = f.z, v[3] = f.w;
    }
}

__device__ __forceinline__ void store4(void* base, int dtype, std::uint64_t idx, const float v[4]) {
    if (dtype == 0) {
        __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
        uint2 raw;
        raw.x = *reinterpret_cast<std::uint32_t*>(&a);
        raw.y = *reinterpret_cast<std::uint32_t*>(&b);
        *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(base) + idx) = raw;
    } else if (dtype == 2) {
        __half2 a = __floats2half2_rn(v[0], v[1]), b = __floats2half2_rn(v[2], v[3]);
        uint2 raw;
        raw.x = *reinterpret_cast<std::uint32_t*>(&a);
        raw.y = *reinterpret_cast<std::uint32_t*>(&b);
        *reinterpret_cast<uint2*>(static_cast<__half*>(base) + idx) = raw;
    } else {
        *reinterpret_cast<float4*>(static_cast<float*>(base) + idx) = make_float4(v[0], v[1], v[2], v[3]);
    }
}

__device__ __forceinline__ std::uint32_t quant4(const float v[4], float inv) {
    std::uint32_t out = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const __nv_fp8_storage_t q = __nv_cvt_float_to_fp8(v[k] * inv, __NV_SATFINITE, __NV_E4M3);
        out |= static_cast<std::uint32_t>(q) << (8 * k);
    }
    return out;
}

__device__ __forceinline__ void dequant4(std::uint32_t packed, float scale, float v[4]) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>((packed >> (8 * k)) & 0xFFu),
                                                     __NV_E4M3);
        v[k] = __half2float(__half(h)) * scale;
    }
}

__device__ __forceinline__ float warp_amax(float a) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    return a;
}

__global__ void __launch_bounds__(256) quant_kernel(const void* x, int dtype, std::uint8_t* q, float* scale,
                                                    std::uint64_t groups) {
    const int lane = threadIdx.x & 31;
    const std::uint64_t warps = std::uint64_t(gridDim.x) * (blockDim.x >> 5);
    for (std::uint64_t g = std::uint64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); g < groups;
         g += warps) {
        float v[4];
        const std::uint64_t idx = g * 128 + lane * 4;
        load4(x, dtype, idx, v);
        const float amax = warp_amax(fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3]))));
        const float s = amax > 0.f ? amax / kE4M3Max : 1.f;
        reinterpret_cast<std::uint32_t*>(q)[g * 32 + lane] = quant4(v, 1.f / s);
        if (lane == 0) scale[g] = s;
    }
}

__global__ void __launch_bounds__(256) dequant_kernel(const std::uint8_t* q, const float* scale, void* x, int dtype,
                                                      std::uint64_t groups) {
    const int lane = threadIdx.x & 31;
    const std::uint64_t warps = std::uint64_t(gridDim.x) * (blockDim.x >> 5);
    for (std::uint64_t g = std::uint64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); g < groups;
         g += warps) {
        float v[4];
        dequant4(reinterpret_cast<const std::uint32_t*>(q)[g * 32 + lane], scale[g], v);
        store4(x, dtype, g * 128 + lane * 4, v);
    }
}

// rows of `cols` bf16 at pool + row_offsets[r]; groups of 128 along the row
__global__ void __launch_bounds__(256) gather_quant_kernel(const std::uint8_t* pool, const std::int64_t* offs,
                                                           std::uint64_t rows, std::uint32_t cols, std::uint8_t* q,
                                                           float* scale) {
    const int lane = threadIdx.x & 31;
    const std::uint32_t gpr = cols / 128;
    const std::uint64_t groups = rows * gpr;
    const std::uint64_t warps = std::uint64_t(gridDim.x) * (blockDim.x >> 5);
    for (std::uint64_t g = std::uint64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); g < groups;
         g += warps) {
        const std::uint64_t r = g / gpr, c = (g % gpr) * 128 + lane * 4;
        float v[4];
        load4(pool + offs[r], 0, c, v);
        const float amax = warp_amax(fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3]))));
        const float s = amax > 0.f ? amax / kE4M3Max : 1.f;
        reinterpret_cast<std::uint32_t*>(q)[g * 32 + lane] = quant4(v, 1.f / s);
        if (lane == 0) scale[g] = s;
    }
}

__global__ void __launch_bounds__(256) dequant_scatter_kernel(const std::uint8_t* q, const float* scale,
                                                              std::uint8_t* pool, const std::int64_t* offs,
                                                              std::uint64_t rows, std::uint32_t cols) {
    const int lane = threadIdx.x & 31;
    const std::uint32_t gpr = cols / 128;
    const std::uint64_t groups = rows * gpr;
    const std::uint64_t warps = std::uint64_t(gridDim.x) * (blockDim.x >> 5);
    for (std::uint64_t g = std::uint64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); g < groups;
         g += warps) {
        const std::uint64_t r = g / gpr, c = (g % gpr) * 128 + lane * 4;
        float v[4];
        dequant4(reinterpret_cast<const std::uint32_t*>(q)[g * 32 + lane], scale[g], v);
        store4(pool + offs[r], 0, c, v);
    }
}

// bf16 fast path: a lane owns 16 consecutive values (two 16-byte loads), so 8
// lanes share a 128-value group, a warp covers 4 groups per iteration, the
// group maximum needs 3 shuffles, and the E4M3 conversions are done in pairs.
// The arithmetic (scale = amax/448, values * (1/scale), saturating E4M3) is the
// same as the per-value kernels above, so both produce identical bytes.
__global__ void __launch_bounds__(256) quant16_bf16_kernel(const __nv_bfloat16* x, std::uint8_t* q, float* scale,
                                                           std::uint64_t groups) {
    const int lane = threadIdx.x & 31;
    const std::uint64_t warps = std::uint64_t(gridDim.x) * (blockDim.x >> 5);
    for (std::uint64_t w = std::uint64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); w * 4 < groups;
         w += warps) {
        const std::uint64_t g = w * 4 + (lane >> 3);
        const bool live = g < groups;
        const std::uint64_t e = g * 128 + (lane & 7) * 16;
        uint4 a = make_uint4(0, 0, 0, 0), b = a;
        if (live) {
            a = *reinterpret_cast<const uint4*>(x + e);
            b = *reinterpret_cast<const uint4*>(x + e + 8);
        }
        const std::uint32_t raw[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        float2 v[8];
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            v[i] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw[i]));
            amax = fmaxf(amax, fmaxf(fabsf(v[i].x), fabsf(v[i].y)));
        }
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
        const float s = amax > 0.f ? amax / kE4M3Max : 1.f;
        const float inv = 1.f / s;
        std::uint32_t out[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __nv_fp8x2_storage_t lo =
                __nv_cvt_float2_to_fp8x2(make_float2(v[2 * i].x * inv, v[2 * i].y * inv), __NV_SATFINITE, __NV_E4M3);
            const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(
                make_float2(v[2 * i + 1].x * inv, v[2 * i + 1].y * inv), __NV_SATFINITE, __NV_E4M3);
            out[i] = static_cast<std::uint32_t>(lo) | (static_cast<std::uint32_t>(hi) << 16);
        }
        if (live) {
            *reinterpret_cast<uint4*>(q + e) = make_uint4(out[0], out[1], out[2], out[3]);
            if ((lane & 7) == 0) scale[g] = s;
        }
    }
}

__global__ void __launch_bounds__(256) dequant16_bf16_kernel(const std::uint8_t* q, const float* scale,
                                                             __nv_bfloat16* x, std::uint64_t groups) {
    const int lane = threadIdx.x & 31;
    const std::uint64_t warps = std::uint64_t(gridDim.x) * (blockDim.x >> 5);
    for (std::uint64_t w = std::uint64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); w * 4 < groups;
         w += warps) {
        const std::uint64_t g = w * 4 + (lane >> 3);
        if (g >= groups) continue;
        const std::uint64_t e = g * 128 + (lane & 7) * 16;
        const uint4 p = *reinterpret_cast<const uint4*>(q + e);
        const float s = scale[g];
        const std::uint32_t raw[4] = {p.x, p.y, p.z, p.w};
        std::uint32_t out[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const __half2_raw hr =
                    __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(raw[i] >> (16 * h)), __NV_E4M3);
                const float2 f = __half22float2(__half2(hr));
                __nv_bfloat162 b2 = __floats2bfloat162_rn(f.x * s, f.y * s);
                out[2 * i + h] = *reinterpret_cast<std::uint32_t*>(&b2);
            }
        }
        *reinterpret_cast<uint4*>(x + e) = make_uint4(out[0], out[1], out[2], out[3]);
        *reinterpret_cast<uint4*>(x + e + 8) = make_uint4(out[4], out[5], out[6], out[7]);
    }
}

unsigned grid_for(std::uint64_t groups, int sm_count) {
    const std::uint64_t want = (groups + 7) / 8;
    const std::uint64_t cap = static_cast<std::uint64_t>(sm_count > 0 ? sm_count : 148) * 8;
    return static_cast<unsigned>(std::max<std::uint64_t>(1, std::min(want, cap)));
}

}  // namespace

cudaError_t launch_fp8_quant(const void* x, int in_dtype, std::uint8_t* q, float* scale, std::uint64_t rows,
                             std::uint32_t cols, std::uint32_t group, int sm_count, cudaStream_t stream) {
    if (group != 128 || cols % 128) return cudaErrorInvalidValue;
    const std::uint64_t groups = rows * (cols / 128);
    if (!groups) return cudaSuccess;
    if (in_dtype == 0) {
        quant16_bf16_kernel<<<grid_for((groups + 3) / 4, sm_count), 256, 0, stream>>>(
            static_cast<const __nv_bfloat16*>(x), q, scale, groups);
        return cudaGetLastError();
    }
    quant_kernel<<<grid_for(groups, sm_count), 256, 0, stream>>>(x, in_dtype, q, scale, groups);
    return cudaGetLastError();
}

cudaError_t launch_fp8_dequant(const std::uint8_t* q, const float* scale, void* x, int out_dtype, std::uint64_t rows,
                               std::uint32_t cols, std::uint32_t group, int sm_count, cudaStream_t stream) {
    if (group != 128 || cols % 128) return cudaErrorInvalidValue;
    const std::uint64_t groups = rows * (cols / 128);
    if (!groups) return cudaSuccess;
    if (out_dtype == 0) {
        dequant16_bf16_kernel<<<grid_for((groups + 3) / 4, sm_count), 256, 0, stream>>>(
            q, scale, static_cast<__nv_bfloat16*>(x), groups);
        return cudaGetLastError();
    }
    dequant_kernel<<<grid_for(groups, sm_count), 256, 0, stream>>>(q, scale, x, out_dtype, groups);
    return cudaGetLastError();
}

cudaError_t launch_fp8_gather_quant(const std::uint8_t* pool, const std::int64_t* offs, std::uint64_t rows,
                                    std::uint32_t cols, std::uint8_t* q, float* scale, cudaStream_t stream) {
    if (cols % 128) return cudaErrorInvalidValue;
    const std::uint64_t groups = rows * (cols / 128);
    if (!groups) return cudaSuccess;
    gather_quant_kernel<<<grid_for(groups, 148), 256, 0, stream>>>(pool, offs, rows, cols, q, scale);
    return cudaGetLastError();
}

cudaError_t launch_fp8_dequant_scatter(const std::uint8_t* q, const float* scale, std::uint8_t* pool,
                                       const std::int64_t* offs, std::uint64_t rows, std::uint32_t cols,
                                       cudaStream_t stream) {
    if (cols % 128) return cudaErrorInvalidValue;
    const std::uint64_t groups = rows * (cols / 128);
    if (!groups) return cudaSuccess;
    dequant_scatter_kernel<<<grid_for(groups, 148), 256, 0, stream>>>(q, scale, pool, offs, rows, cols);
    return cudaGetLastError();
}

}  // namespace ops
}  // namespace tutti
