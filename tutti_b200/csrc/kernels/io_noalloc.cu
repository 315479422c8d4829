// Allocation-free entry point of the GPU NVMe io path (declared in
// <tutti/noalloc.h>). This entry point has no counterpart in the reference.
//
// Who needs it: callers that cannot allocate GPU memory at the moment they
// move KV, such as engines that give all spare HBM to their KV pool at
// start-up (a cudaMalloc in the middle of a step could then fail) and C-ABI
// embedders that own no CUDA allocator. The runtime's own submit path keeps a
// pool of per-operation arenas obtained with cudaMalloc; this entry point
// instead puts the launch's scratch (command list, piece list, lease ids, work
// cursor, per-command status) in one fixed array below, which every GPU that
// loads the library holds until the process exits.
//
// Limits: TUTTI_NOALLOC_MAX_COMMANDS commands, TUTTI_NOALLOC_MAX_PIECES pieces
// and TUTTI_NOALLOC_MAX_LEASES CTAs per call (about 2.3 MiB in total);
// anything larger is refused before launch. Calls that overlap on the GPU race
// on the shared array. The call is synchronous (it waits for its stream). The
// first call on a device looks up the array's device address with that device
// current; make it before any stream capture. Nothing here calls cudaMalloc,
// cudaFree or any allocating routine.

#include <cstddef>
#include <cstdio>
#include <cstring>
#include <mutex>

#include <cuda_runtime.h>

#include <tutti/noalloc.h>

#include "../datapaths/gpu_nvme_data_path.h"
#include "../runtime/device_guard.h"
#include "io_kernel.h"

namespace {

constexpr std::size_t kAlign = 256;
constexpr std::size_t align_up(std::size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

constexpr std::size_t kOffCmds = 0;
constexpr std::size_t kOffPieces = align_up(kOffCmds + TUTTI_NOALLOC_MAX_COMMANDS * sizeof(tutti::io::IoCommand));
constexpr std::size_t kOffLeases = align_up(kOffPieces + TUTTI_NOALLOC_MAX_PIECES * sizeof(tutti::io::IoPiece));
constexpr std::size_t kOffCursor = align_up(kOffLeases + TUTTI_NOALLOC_MAX_LEASES * sizeof(std::uint32_t));
constexpr std::size_t kOffStatus = align_up(kOffCursor + 16);
constexpr std::size_t kScratchBytes = align_up(kOffStatus + TUTTI_NOALLOC_MAX_COMMANDS * sizeof(std::uint32_t));

// The C structs are copied to the device unchanged, so every field must sit at
// the io kernel's offset with the io kernel's width.
#define TUTTI_SAME_FIELD(a, fa, b, fb)                                                   \
    static_assert(offsetof(a, fa) == offsetof(b, fb) && sizeof(a::fa) == sizeof(b::fb), \
                  #a "." #fa " must match " #b "." #fb)
TUTTI_SAME_FIELD(tutti_noalloc_command, logical, tutti::io::IoCommand, logical);
TUTTI_SAME_FIELD(tutti_noalloc_command, target_row, tutti::io::IoCommand, target);
TUTTI_SAME_FIELD(tutti_noalloc_command, bytes, tutti::io::IoCommand, bytes);
TUTTI_SAME_FIELD(tutti_noalloc_command, first_piece, tutti::io::IoCommand, first_piece);
TUTTI_SAME_FIELD(tutti_noalloc_command, n_pieces, tutti::io::IoCommand, n_pieces);
TUTTI_SAME_FIELD(tutti_noalloc_command, opcode, tutti::io::IoCommand, opcode);
TUTTI_SAME_FIELD(tutti_noalloc_command, transform, tutti::io::IoCommand, transform);
TUTTI_SAME_FIELD(tutti_noalloc_command, replicas, tutti::io::IoCommand, replicas);
TUTTI_SAME_FIELD(tutti_noalloc_piece, mem, tutti::io::IoPiece, mem);
TUTTI_SAME_FIELD(tutti_noalloc_piece, off, tutti::io::IoPiece, off);
TUTTI_SAME_FIELD(tutti_noalloc_piece, bytes, tutti::io::IoPiece, bytes);
#undef TUTTI_SAME_FIELD
static_assert(sizeof(tutti_noalloc_command) == sizeof(tutti::io::IoCommand), "command layout");
static_assert(sizeof(tutti_noalloc_piece) == sizeof(tutti::io::IoPiece), "piece layout");

constexpr int kMaxGpus = 64;

// The fixed scratch array: one copy per GPU that loads this library.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

// Host-side device addresses of g_noalloc_scratch, one per device, looked up
// once. The array's name in host code is only a stand-in, never a device
// address, so it is never handed to a kernel.
void* g_scratch_addr[kMaxGpus] = {};
std::mutex g_setup_mu;
// Per calling thread: calls on different devices may run at the same time.
thread_local char g_last_error[256] = "";

int fail(int code, const char* msg) {
    std::snprintf(g_last_error, sizeof(g_last_error), "%s", msg);
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    std::snprintf(g_last_error, sizeof(g_last_error), "%s: %s", what, cudaGetErrorString(e));
    cudaGetLastError();
    return TUTTI_NOALLOC_E_CUDA;
}

}  // namespace

extern "C" const char* tutti_noalloc_last_error(void) { return g_last_error; }

extern "C" int tutti_nvme_io_noalloc(void* data_path, const tutti_noalloc_command* commands, uint32_t n_commands,
                                     const tutti_noalloc_piece* pieces, uint32_t n_pieces, uint32_t* cmd_status,
                                     cudaStream_t stream) {
    using tutti::GpuNvmeDataPath;
    g_last_error[0] = '\0';
    if (!data_path || (n_commands && (!commands || !cmd_status)) || (n_pieces && !pieces))
        return fail(TUTTI_NOALLOC_E_ARGS, "null argument");
    if (n_commands == 0) return TUTTI_NOALLOC_OK;
    if (n_commands > TUTTI_NOALLOC_MAX_COMMANDS || n_pieces > TUTTI_NOALLOC_MAX_PIECES)
        return fail(TUTTI_NOALLOC_E_TOO_LARGE, "batch exceeds TUTTI_NOALLOC_MAX_COMMANDS / TUTTI_NOALLOC_MAX_PIECES");
    auto* dp = static_cast<GpuNvmeDataPath*>(data_path);

    // Validate everything the kernel will dereference before anything is launched.
    for (uint32_t c = 0; c < n_commands; ++c) {
        const tutti_noalloc_command& k = commands[c];
        if (k.opcode != tutti::nvme::kOpRead && k.opcode != tutti::nvme::kOpWrite)
            return fail(TUTTI_NOALLOC_E_ARGS, "command opcode must be 1 (write) or 2 (read)");
        if (k.transform != 0) return fail(TUTTI_NOALLOC_E_ARGS, "command.transform must be 0 (no stored-format transform)");
        if (k.replicas > 1) return fail(TUTTI_NOALLOC_E_ARGS, "command.replicas must be 0 or 1");
        if (k.bytes == 0 || k.n_pieces == 0 || k.first_piece > n_pieces || k.n_pieces > n_pieces - k.first_piece)
            return fail(TUTTI_NOALLOC_E_ARGS, "command piece range out of bounds");
        if (!dp->noalloc_target_ok(k.target_row, k.logical, k.bytes))
            return fail(TUTTI_NOALLOC_E_ARGS, "command outside an open target");
        uint32_t expect = 0;
        for (uint32_t i = k.first_piece; i < k.first_piece + k.n_pieces; ++i) {
            const tutti_noalloc_piece& p = pieces[i];
            if (p.off != expect || p.bytes == 0 || (p.off | p.bytes) % 16 || p.mem % 16)
                return fail(TUTTI_NOALLOC_E_ARGS, "pieces must tile their command in order, 16-byte aligned");
            if (!dp->noalloc_memory_ok(p.mem, p.bytes))
                return fail(TUTTI_NOALLOC_E_ARGS, "piece outside registered memory");
            expect += p.bytes;
        }
        if (expect != k.bytes) return fail(TUTTI_NOALLOC_E_ARGS, "pieces do not cover their command");
    }

    const int dev = dp->accel_id();
    if (dev < 0 || dev >= kMaxGpus) return fail(TUTTI_NOALLOC_E_SETUP, "data path device out of range");
    tutti::DeviceGuard guard(dev);
    if (!guard.status().ok()) return fail(TUTTI_NOALLOC_E_CUDA, "cannot make the data path's device current");
    {
        std::lock_guard<std::mutex> g(g_setup_mu);
        if (!g_scratch_addr[dev]) {
            void* addr = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&addr, g_noalloc_scratch);
            if (e != cudaSuccess || !addr) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
            g_scratch_addr[dev] = addr;
        }
    }
    char* base = static_cast<char*>(g_scratch_addr[dev]);

    std::uint32_t leases[TUTTI_NOALLOC_MAX_LEASES];
    const std::uint32_t want = n_commands < TUTTI_NOALLOC_MAX_LEASES ? n_commands : TUTTI_NOALLOC_MAX_LEASES;
    const std::uint32_t n_leases = dp->noalloc_acquire_leases(want, leases);
    if (n_leases == 0) return fail(TUTTI_NOALLOC_E_BUSY, "all queue leases are held by in-flight operations");

    int rc = TUTTI_NOALLOC_OK;
    cudaError_t e = cudaMemcpyAsync(base + kOffCmds, commands, n_commands * sizeof(tutti_noalloc_command),
                                    cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess && n_pieces)
        e = cudaMemcpyAsync(base + kOffPieces, pieces, n_pieces * sizeof(tutti_noalloc_piece), cudaMemcpyHostToDevice,
                            stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(base + kOffLeases, leases, n_leases * sizeof(std::uint32_t), cudaMemcpyHostToDevice, stream);
    // The array keeps the previous call's contents: zero the cursor and mark
    // every status word "never ran" before this launch.
    if (e == cudaSuccess) e = cudaMemsetAsync(base + kOffCursor, 0, 16, stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(base + kOffStatus, 0xFF, n_commands * sizeof(std::uint32_t), stream);
    if (e == cudaSuccess) {
        tutti::io::IoKernelParams p{};
        dp->noalloc_fill_params(p);
        p.cmds = reinterpret_cast<const tutti::io::IoCommand*>(base + kOffCmds);
        p.pieces = reinterpret_cast<const tutti::io::IoPiece*>(base + kOffPieces);
        p.n_cmds = n_commands;
        p.cursor = reinterpret_cast<std::uint32_t*>(base + kOffCursor);
        p.cmd_status = reinterpret_cast<std::uint32_t*>(base + kOffStatus);
        p.lease_ids = reinterpret_cast<const std::uint32_t*>(base + kOffLeases);
        e = tutti::io::launch_nvme_io(p, n_leases, stream);
    }
    // Wait for the kernel before copying its statuses back: a copy queued behind
    // a running io kernel could hold up drive DMA that shares its hardware queue.
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(cmd_status, base + kOffStatus, n_commands * sizeof(std::uint32_t), cudaMemcpyDeviceToHost,
                            stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    bool reset = false;
    if (e != cudaSuccess) {
        rc = cuda_fail(e, "io launch");
        cudaStreamSynchronize(stream);
        reset = true;
    } else {
        int failed = 0;
        for (uint32_t c = 0; c < n_commands; ++c) {
            if (cmd_status[c] == 0) continue;
            ++failed;
            const std::uint32_t kind = cmd_status[c] & 0xFFFF0000u;
            if (cmd_status[c] == 0xFFFFFFFFu || kind == tutti::io::kCmdTimeout) reset = true;
        }
        rc = failed;
        if (failed) std::snprintf(g_last_error, sizeof(g_last_error), "%d command(s) failed", failed);
    }
    dp->noalloc_release_leases(leases, n_leases, reset);
    return rc;
}
