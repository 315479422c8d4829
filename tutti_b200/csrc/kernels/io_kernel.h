#pragma once
// Device-side data structures and launch entry points of the GPU NVMe io path.
//
// One launch per submit. Each CTA owns one queue pair per device (its "lease"):
// no SQ/CQ state is shared between CTAs, so the submit/poll path needs no
// global atomics except one work-stealing cursor over the command list.
// A command is a contiguous logical range of one target (<= one staging slot);
// it carries a list of pieces that say where each byte range of the command
// lives in caller memory, so the paged-KV scatter (read) and gather (write)
// happen inside the io kernel, between the staging slot and HBM.
//
// Parity: this replaces the reference's fused_submit_kernel_pool
// (csrc/data_paths/striped_local_nvme/fused_submit_kernel.cuh:171-218) plus its
// separate single_layer_kv_transfer_kernel (csrc/kv_transfer/src/mem_kernels.cu:66-130);
// per-entry status codes follow EntryCompletionStatus (0 ok, 1 resolve,
// 2 timeout, 3 NVMe error) from submit_one.cuh:117-143.

#include <cstdint>

#include <cuda_runtime_api.h>

#include "../nvme/nvme_spec.h"
#include "../nvme/controller.h"

namespace tutti {
namespace io {

constexpr int kMaxSlots = 64;     // staging slots per CTA (slots x kMaxSub must stay under the queue depth)
constexpr int kMaxSub = 8;        // NVMe commands per staging slot (extent/MDTS splits)
constexpr int kMaxDevices = 8;    // devices (controllers) one launch can drive
constexpr int kIoThreads = 512;   // threads per CTA with SIMT movers (host-memory staging)
constexpr int kIoThreadsBulk = 128;  // threads per CTA with bulk-copy movers (HBM staging)

// How the movers copy a slot between staging and caller memory.
//  kMoversSimt: 3 groups x 5 warps of 16-byte loads/stores; hides the latency
//               of zero-copy reads of page-locked host staging over PCIe.
//  kMoversBulk: 3 groups x 1 warp; lane 0 of each group streams the slot
//               through a shared-memory ring with cp.async.bulk (TMA engine),
//               for staging in HBM that the drive fills by DMA.
enum MoverKind : std::uint32_t { kMoversSimt = 0, kMoversBulk = 1 };
constexpr std::uint32_t kBulkStages = 4;
constexpr std::uint32_t kBulkChunk = 8192;
constexpr std::uint32_t kBulkSmemBytes = 3 * kBulkStages * kBulkChunk;  // dynamic smem of a bulk CTA

// Stored-format transforms done by the movers while they move a slot.
// kXformFp8Block128: memory holds bf16; each piece is stored as
// [E4M3 values, n bytes][fp32 scale per 128 values, n/32 bytes] for the
// piece's n bf16 values, i.e. 33/64 of the memory bytes. The scale is
// amax/448 (1 for an all-zero group) and values saturate, as in the
// standalone block-scaling kernels, so both produce identical bytes.
constexpr std::uint16_t kXformNone = 0;
constexpr std::uint16_t kXformFp8Block128 = 1;

struct IoCommand {  // 32 B
    std::uint64_t logical;      // byte offset in the target
    std::uint32_t target;       // row of the device-resident target table
    std::uint32_t bytes;        // <= slot_bytes
    std::uint32_t first_piece;
    std::uint32_t n_pieces;     // pieces per destination group
    std::uint16_t opcode;       // nvme::kOpRead / kOpWrite
    std::uint16_t transform;    // kXformNone / kXformFp8Block128
    // Reads only: number of destination groups (0 or 1: one). Group g's pieces
    // are [first_piece + g*n_pieces, +n_pieces) with the same offsets as group 0;
    // the command's bytes are read once and stored to every group (e.g. the
    // TP ranks that all need a replicated latent cache, over NVLink).
    std::uint32_t replicas;
};

struct IoPiece {  // 16 B
    std::uint64_t mem;     // device-visible address in caller memory
    std::uint32_t off;     // byte offset within the command
    std::uint32_t bytes;
};

struct DevExtent {  // 32 B
    std::uint64_t logical;
    std::uint64_t physical;
    std::uint64_t length;
    std::uint32_t device;
    std::uint32_t pad;
};

struct DevTarget {  // 32 B, device-resident file handle
    const DevExtent* extents;
    std::uint64_t size;
    std::uint32_t n_extents;
    std::uint32_t generation;
    std::uint64_t pad;
};

struct QueueCursor {  // persisted per (device, lease) across launches
    std::uint32_t sq_tail;
    std::uint32_t cq_head;
    std::uint32_t phase;
    std::uint32_t dirty;  // a launch ended with commands still owned by the controller
};

struct DevDevice {
    const nvme::QueuePairView* queues;  // indexed by lease
    QueueCursor* cursors;               // indexed by lease
    std::uint32_t lba_shift;
    std::uint32_t mdts_bytes;
    std::uint32_t n_queues;
    std::uint32_t nsid;
};

// Per-command status words written by the kernel.
enum : std::uint32_t {
    kCmdOk = 0,
    kCmdResolve = 1u << 16,
    kCmdTimeout = 2u << 16,
    kCmdNvme = 3u << 16,      // | raw NVMe status field
    kCmdNotRun = 4u << 16,
    kCmdBadDevice = 5u << 16,
};

// Split completion: a submit-phase launch (one warp per lease) claims commands
// into its slots, writes their SQEs, rings the doorbells and exits; a later
// drain-phase launch of full CTAs on the same leases takes over the slots from
// this hand-over record, polls the CQs, moves the data and enforces the
// deadlines (which run from submission). Reads only.
enum IoPhase : std::uint32_t { kPhaseFull = 0, kPhaseSubmit = 1, kPhaseDrain = 2 };

// A registered memory region the drives may DMA into directly. Addresses in
// [lo, hi) qualify; byte `off = addr - va` of the mapping (which may start
// below lo: the driver pins whole pages) has bus address
// bus[off >> page_shift] + (off & (2^page_shift - 1)), or bus[0] + off when
// page_shift is 0 (one contiguous bus range).
struct DmaRegion {  // 48 B
    std::uint64_t lo;
    std::uint64_t hi;
    std::uint64_t va;
    const std::uint64_t* bus;
    std::uint32_t page_shift;
    std::uint32_t pad[3];
};

struct LeaseCarry {  // one per CTA of a split launch
    int cmd[kMaxSlots];                // -1: slot unused
    std::uint32_t pending[kMaxSlots];  // sub-commands not yet completed
    std::uint32_t status[kMaxSlots];
    unsigned long long t0[kMaxSlots];  // %globaltimer at submission
    std::uint32_t inflight_dev[kMaxDevices];
};

struct IoKernelParams {
    const IoCommand* cmds;
    const IoPiece* pieces;
    std::uint32_t n_cmds;
    std::uint32_t n_devices;
    std::uint32_t* cursor;        // work-stealing index, zero at launch
    std::uint32_t* cmd_status;    // n_cmds words, preset to kCmdNotRun
    const DevTarget* targets;
    const DevDevice* devices;     // n_devices rows (device memory)
    const std::uint32_t* lease_ids;  // gridDim.x leases
    char* staging_dev;            // device address of the staging arena
    // Bus addresses the drives DMA to (device memory): page_bus[k] is the bus
    // address of 4 KiB page k of the staging arena (slot i covers pages
    // [i * slot_bytes / 4 KiB, ...)), list_bus[i] that of slot i's prebuilt
    // PRP-list page. Pages need not be adjacent on the bus.
    const std::uint64_t* page_bus;
    const std::uint64_t* list_bus;
    // Direct reads: a read whose bytes all land in whole 4 KiB pages of these
    // regions (sorted by va) gets PRPs that name those pages, so the drive DMAs
    // into the final memory and no mover touches the data. Its PRP list is
    // written into direct_lists (one 4 KiB page per slot, device address of
    // page-locked host memory) whose bus addresses are direct_list_bus.
    // n_regions == 0: every command is staged.
    const DmaRegion* regions;
    std::uint64_t* direct_lists;
    const std::uint64_t* direct_list_bus;
    std::uint32_t n_regions;
    std::uint32_t direct_pad;
    std::uint32_t slot_bytes;     // <= 2 MiB (one PRP-list page per slot)
    std::uint32_t slots_per_lease;
    std::uint64_t timeout_ns;     // per command, from submission
    std::uint64_t* timing;        // optional: 4 %globaltimer stamps per command
    LeaseCarry* carry;            // split completion: gridDim.x records (else unused)
    std::uint32_t phase;          // IoPhase
    std::uint32_t movers;         // MoverKind (matches where the staging arena lives)
};

// Launches the fused io kernel on `stream` with one CTA per lease (one warp
// per lease for kPhaseSubmit).
cudaError_t launch_nvme_io(const IoKernelParams& p, std::uint32_t n_leases, cudaStream_t stream);

}  // namespace io
}  // namespace tutti
