// tutti_b200._ops: torch-facing bindings of the sm_100a kernels and the CUDA
// IPC helpers used for NVLink peer access between ranks.
// Parity: reference csrc/kv_transfer/src/mem_kernels.cu:515-543 (the
// tutti_kv_transfer._native module: transfer kernels, replica IPC export and
// import, peer page scatter).

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cuda_runtime.h>

#include "ops_kernels.h"

namespace {

using namespace tutti::ops;

void check_cuda(cudaError_t e, const char* what) {
    TORCH_CHECK(e == cudaSuccess, what, ": ", cudaGetErrorString(e));
}

int sm_count(int dev) {
    static int cached[64] = {0};
    if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
    int n = 148;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (dev >= 0 && dev < 64) cached[dev] = n;
    return n;
}

int dtype_code(const at::Tensor& t) {
    if (t.scalar_type() == at::kBFloat16) return 0;
    if (t.scalar_type() == at::kFloat) return 1;
    if (t.scalar_type() == at::kHalf) return 2;
    TORCH_CHECK(false, "dtype must be bf16, fp16 or fp32");
}

// items: int64 [n, 3] = (src address, dst address, bytes)
void copy_items(const at::Tensor& items, bool tma) {
    TORCH_CHECK(items.is_cuda() && items.scalar_type() == at::kLong && items.dim() == 2 && items.size(1) == 3 &&
                    items.is_contiguous(),
                "items must be a contiguous int64 CUDA tensor [n, 3]");
    const c10::cuda::CUDAGuard guard(items.device());
    auto err = at::zeros({1}, items.options().dtype(at::kInt));
    auto stream = at::cuda::getCurrentCUDAStream();
    check_cuda(launch_copy_items(reinterpret_cast<const CopyItem*>(items.data_ptr<int64_t>()),
                                 static_cast<std::uint32_t>(items.size(0)), tma,
                                 reinterpret_cast<std::uint32_t*>(err.data_ptr<int>()), sm_count(items.get_device()),
                                 stream),
               "copy_items launch");
    if (tma) TORCH_CHECK(err.item<int>() == 0, "bulk copy: an mbarrier wait exceeded its iteration limit");
}

std::tuple<at::Tensor, at::Tensor> fp8_quant(const at::Tensor& x, int64_t group) {
    TORCH_CHECK(x.is_cuda() && x.is_contiguous() && x.dim() == 2, "x must be a contiguous 2-D CUDA tensor");
    TORCH_CHECK(group == 128 && x.size(1) % 128 == 0, "group must be 128 and divide the row");
    const c10::cuda::CUDAGuard guard(x.device());
    auto q = at::empty({x.size(0), x.size(1)}, x.options().dtype(at::kByte));
    auto s = at::empty({x.size(0), x.size(1) / 128}, x.options().dtype(at::kFloat));
    check_cuda(launch_fp8_quant(x.data_ptr(), dtype_code(x), q.data_ptr<uint8_t>(), s.data_ptr<float>(), x.size(0),
                                static_cast<std::uint32_t>(x.size(1)), 128, sm_count(x.get_device()),
                                at::cuda::getCurrentCUDAStream()),
               "fp8_quant");
    return {q, s};
}

at::Tensor fp8_dequant(const at::Tensor& q, const at::Tensor& s, at::ScalarType dtype) {
    TORCH_CHECK(q.is_cuda() && q.is_contiguous() && q.dim() == 2 && q.scalar_type() == at::kByte, "q: uint8 [rows, cols]");
    TORCH_CHECK(s.is_cuda() && s.is_contiguous() && s.scalar_type() == at::kFloat, "scale: fp32");
    const c10::cuda::CUDAGuard guard(q.device());
    auto x = at::empty({q.size(0), q.size(1)}, q.options().dtype(dtype));
    check_cuda(launch_fp8_dequant(q.data_ptr<uint8_t>(), s.data_ptr<float>(), x.data_ptr(), dtype_code(x), q.size(0),
                                  static_cast<std::uint32_t>(q.size(1)), 128, sm_count(q.get_device()),
                                  at::cuda::getCurrentCUDAStream()),
               "fp8_dequant");
    return x;
}

std::tuple<at::Tensor, at::Tensor> fp8_gather_quant(const at::Tensor& pool, const at::Tensor& row_offsets,
                                                     int64_t cols) {
    TORCH_CHECK(pool.is_cuda() && row_offsets.is_cuda() && row_offsets.scalar_type() == at::kLong,
                "pool and int64 row_offsets must be on CUDA");
    const c10::cuda::CUDAGuard guard(pool.device());
    const int64_t rows = row_offsets.numel();
    auto q = at::empty({rows, cols}, pool.options().dtype(at::kByte));
    auto s = at::empty({rows, cols / 128}, pool.options().dtype(at::kFloat));
    check_cuda(launch_fp8_gather_quant(static_cast<const uint8_t*>(pool.data_ptr()), row_offsets.data_ptr<int64_t>(),
                                       rows, static_cast<std::uint32_t>(cols), q.data_ptr<uint8_t>(),
                                       s.data_ptr<float>(), at::cuda::getCurrentCUDAStream()),
               "fp8_gather_quant");
    return {q, s};
}

void fp8_dequant_scatter(const at::Tensor& q, const at::Tensor& s, at::Tensor& pool, const at::Tensor& row_offsets) {
    TORCH_CHECK(q.is_cuda() && s.is_cuda() && pool.is_cuda() && row_offsets.is_cuda(), "CUDA tensors required");
    const c10::cuda::CUDAGuard guard(pool.device());
    check_cuda(launch_fp8_dequant_scatter(q.data_ptr<uint8_t>(), s.data_ptr<float>(),
                                          static_cast<uint8_t*>(pool.data_ptr()), row_offsets.data_ptr<int64_t>(),
                                          row_offsets.numel(), static_cast<std::uint32_t>(q.size(1)),
                                          at::cuda::getCurrentCUDAStream()),
               "fp8_dequant_scatter");
}

at::Tensor prefix_hash(const at::Tensor& tokens, const at::Tensor& starts, const at::Tensor& lengths,
                       const at::Tensor& parents, const at::Tensor& parent_len, const at::Tensor& key_offsets,
                       int64_t total_keys, int64_t chunk_tokens) {
    TORCH_CHECK(tokens.is_cuda() && tokens.scalar_type() == at::kLong, "tokens: int64 CUDA");
    const c10::cuda::CUDAGuard guard(tokens.device());
    auto keys = at::zeros({total_keys, 16}, tokens.options().dtype(at::kByte));
    check_cuda(launch_prefix_hash(tokens.data_ptr<int64_t>(), starts.data_ptr<int64_t>(), lengths.data_ptr<int64_t>(),
                                  parents.data_ptr<uint8_t>(), parent_len.data_ptr<int32_t>(),
                                  key_offsets.data_ptr<int64_t>(), keys.data_ptr<uint8_t>(),
                                  static_cast<std::uint32_t>(starts.numel()), static_cast<std::uint32_t>(chunk_tokens),
                                  at::cuda::getCurrentCUDAStream()),
               "prefix_hash");
    return keys;
}

at::Tensor checksum(const at::Tensor& items, int64_t uniform_bytes) {
    TORCH_CHECK(items.is_cuda() && items.scalar_type() == at::kLong && items.dim() == 2 && items.size(1) == 3,
                "items: int64 CUDA [n, 3]");
    const c10::cuda::CUDAGuard guard(items.device());
    auto out = at::empty({items.size(0)}, items.options());
    const auto* it = reinterpret_cast<const CopyItem*>(items.data_ptr<int64_t>());
    auto* o = reinterpret_cast<std::uint64_t*>(out.data_ptr<int64_t>());
    const auto n = static_cast<std::uint32_t>(items.size(0));
    if (uniform_bytes > 0 && uniform_bytes % 16 == 0)
        check_cuda(launch_checksum_uniform(it, n, static_cast<std::uint64_t>(uniform_bytes), o,
                                           at::cuda::getCurrentCUDAStream()),
                   "checksum");
    else
        check_cuda(launch_checksum(it, n, o, at::cuda::getCurrentCUDAStream()), "checksum");
    return out;
}

// ---- CUDA IPC for NVLink peer access between processes ----
py::tuple ipc_export(const at::Tensor& t) {
    TORCH_CHECK(t.is_cuda(), "tensor must be on CUDA");
    const c10::cuda::CUDAGuard guard(t.device());
    // Allocation base via the driver entry point (no link-time libcuda dependency).
    using GetRange = int (*)(unsigned long long*, size_t*, unsigned long long);
    static GetRange get_range = nullptr;
    if (!get_range) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        check_cuda(cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q),
                   "cudaGetDriverEntryPoint(cuMemGetAddressRange)");
        TORCH_CHECK(fn != nullptr, "cuMemGetAddressRange unavailable");
        get_range = reinterpret_cast<GetRange>(fn);
    }
    unsigned long long base_addr = 0;
    size_t size = 0;
    TORCH_CHECK(get_range(&base_addr, &size, reinterpret_cast<unsigned long long>(t.data_ptr())) == 0,
                "cuMemGetAddressRange failed");
    void* base = reinterpret_cast<void*>(base_addr);
    cudaIpcMemHandle_t h;
    check_cuda(cudaIpcGetMemHandle(&h, base), "cudaIpcGetMemHandle");
    const int64_t offset = static_cast<char*>(t.data_ptr()) - static_cast<char*>(base);
    return py::make_tuple(py::bytes(reinterpret_cast<const char*>(&h), sizeof(h)), offset, static_cast<int64_t>(size));
}

int64_t ipc_open(py::bytes handle, int64_t device) {
    std::string b = handle;
    TORCH_CHECK(b.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, b.data(), sizeof(h));
    const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
    void* p = nullptr;
    check_cuda(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr, int64_t device) {
    const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
    check_cuda(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)), "cudaIpcCloseMemHandle");
}

bool enable_peer_access(int64_t device, int64_t peer) {
    int can = 0;
    cudaDeviceCanAccessPeer(&can, static_cast<int>(device), static_cast<int>(peer));
    if (!can) return false;
    const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
    cudaError_t e = cudaDeviceEnablePeerAccess(static_cast<int>(peer), 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
        return true;
    }
    return e == cudaSuccess;
}

}  // namespace

// Persistent compute stand-in on the current stream; blocks_per_sm CTAs per SM.
void persistent_fma(const at::Tensor& out, int64_t iters, int64_t blocks_per_sm) {
    TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.is_contiguous(), "out: float32 CUDA tensor");
    const c10::cuda::CUDAGuard guard(out.device());
    const std::uint32_t blocks = static_cast<std::uint32_t>(sm_count(out.get_device()) * blocks_per_sm);
    TORCH_CHECK(out.numel() >= static_cast<int64_t>(blocks) * 256, "out needs blocks x 256 floats");
    check_cuda(launch_persistent_fma(out.data_ptr<float>(), static_cast<std::uint64_t>(iters), blocks,
                                     at::cuda::getCurrentCUDAStream()),
               "persistent_fma launch");
}

// Ready flags: `targets` is a uint64 CUDA tensor of word addresses; runs on the current stream.
void ready_signal(const at::Tensor& targets, int64_t value) {
    TORCH_CHECK(targets.is_cuda() && targets.scalar_type() == at::kLong && targets.is_contiguous(),
                "targets: int64 CUDA tensor of addresses");
    const c10::cuda::CUDAGuard guard(targets.device());
    check_cuda(launch_ready_signal(reinterpret_cast<std::uint64_t* const*>(targets.data_ptr<int64_t>()),
                                   static_cast<std::uint32_t>(targets.numel()), static_cast<std::uint64_t>(value),
                                   at::cuda::getCurrentCUDAStream()),
               "ready_signal launch");
}

// Waits on the current stream until words[0..n) >= value (bounded); status: int32 tensor
// (CUDA, or pinned host memory for a host read without a copy).
void ready_wait(int64_t words, int64_t n, int64_t value, int64_t timeout_ns, const at::Tensor& status) {
    TORCH_CHECK(status.scalar_type() == at::kInt && status.numel() >= 1, "status: int32 tensor");
    TORCH_CHECK(n > 0 && n <= 1024 && timeout_ns > 0, "1..1024 words and a positive timeout");
    void* st = status.data_ptr();
    if (!status.is_cuda()) {
        void* dev = nullptr;
        TORCH_CHECK(cudaHostGetDevicePointer(&dev, st, 0) == cudaSuccess, "status: pinned, mapped host memory");
        st = dev;
    }
    check_cuda(launch_ready_wait(reinterpret_cast<const std::uint64_t*>(words), static_cast<std::uint32_t>(n),
                                 static_cast<std::uint64_t>(value), static_cast<std::uint64_t>(timeout_ns),
                                 static_cast<std::uint32_t*>(st), at::cuda::getCurrentCUDAStream()),
               "ready_wait launch");
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.doc() = "tutti_b200 sm_100a kernels: page copy, fp8 block scaling, prefix hashing, checksums, IPC";
    m.def("copy_items", &copy_items, py::arg("items"), py::arg("tma") = true);
    m.def("persistent_fma", &persistent_fma, py::arg("out"), py::arg("iters"), py::arg("blocks_per_sm") = 1);
    m.def("ready_signal", &ready_signal, py::arg("targets"), py::arg("value"));
    m.def("ready_wait", &ready_wait, py::arg("words"), py::arg("n"), py::arg("value"), py::arg("timeout_ns"),
          py::arg("status"));
    m.def("fp8_quant", &fp8_quant, py::arg("x"), py::arg("group") = 128);
    m.def("fp8_dequant", &fp8_dequant, py::arg("q"), py::arg("scale"), py::arg("dtype") = at::kBFloat16);
    m.def("fp8_gather_quant", &fp8_gather_quant);
    m.def("fp8_dequant_scatter", &fp8_dequant_scatter);
    m.def("prefix_hash", &prefix_hash);
    m.def("checksum", &checksum, py::arg("items"), py::arg("uniform_bytes") = 0);
    m.def("ipc_export", &ipc_export);
    m.def("ipc_open", &ipc_open);
    m.def("ipc_close", &ipc_close);
    m.def("enable_peer_access", &enable_peer_access);
}
