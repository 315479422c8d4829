#pragma once
// NVMe controller providers behind one queue protocol.
//
// The GPU io kernel always speaks NVMe: it writes 64-byte SQEs into an SQ ring,
// rings the SQ tail doorbell, polls CQE phase bits and rings the CQ head
// doorbell. Which "drive" answers is a provider:
//   * EmulatedNvmeController: host threads own the rings (page-locked, mapped
//     into the GPU), execute READ/WRITE/FLUSH against file-backed namespace
//     ranges and post CQEs. Its media is either the backing files themselves
//     (pread/pwrite) or an in-memory image of them (page-locked host memory,
//     loaded from the files on first touch, written through on WRITE). PRPs
//     may name host memory or GPU memory: GPU destinations are filled by
//     copy-engine DMA on the worker's own CUDA stream, and the CQE of such a
//     command is written by that stream after the copy (the ordering a
//     drive's posted writes give: data before completion). Used where no
//     user-owned NVMe queues exist (no queue-leasing kernel driver, no
//     bindable drives).
//   * SnvmeController (snvme_client.h): a real controller driven through the
//     snvme queue-leasing driver. The rings live in this process's memory, the
//     driver creates the queue pairs over them, the doorbells are the
//     controller's BAR0 (mapped into the process and registered with CUDA as
//     I/O memory) and PRPs carry the bus addresses the driver pinned.
//
// Parity: queue memory layout and doorbell stride follow the reference's
// libnvm queue structs (csrc/device_manager/nvme/libnvm/include/nvm_types.h) and
// NvmeQueueGroup (csrc/data_paths/local_nvme/io/nvme_queue_group.cu:131-217).

#include <atomic>
#include <cstdint>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include <cuda_runtime_api.h>

#include <tutti/status.h>

#include "host_memory.h"
#include "nvme_spec.h"

namespace tutti {
namespace nvme {

// QueuePairView::flags
constexpr std::uint32_t kQueueMmioDoorbells = 1u << 0;  // doorbells are device registers (BAR0)

// Device-visible view of one I/O queue pair; POD, copied into GPU memory.
struct QueuePairView {
    Sqe* sq;                    // SQ ring (depth entries)
    const Cqe* cq;              // CQ ring (depth entries)
    std::uint32_t* sq_doorbell;
    std::uint32_t* cq_doorbell;
    std::uint32_t depth;
    std::uint32_t qid;
    std::uint32_t nsid;
    std::uint32_t flags;        // kQueue*
};

// Bus addresses of a buffer made DMA-reachable by a controller. Behind an
// IOMMU or a GPU peer mapping every page has its own bus address and the
// pages of one buffer need not be adjacent on the bus.
struct DmaMapping {
    std::uint64_t va = 0;          // start of the mapped range (page-aligned when paged)
    std::uint64_t bytes = 0;       // length of the mapped range
    std::uint64_t page_bytes = 0;  // 0: the whole range is one bus range at bus[0]
    std::vector<std::uint64_t> bus;
    int kind = 0;                  // controller-private (which unmap call releases it)

    bool covers(const void* p, std::uint64_t n) const {
        const auto a = reinterpret_cast<std::uint64_t>(p);
        return a >= va && n <= bytes && a - va <= bytes - n;
    }
    // Bus address of virtual address `p` inside the range (0 outside it).
    std::uint64_t bus_at(const void* p) const {
        const auto a = reinterpret_cast<std::uint64_t>(p);
        if (a < va || a - va >= bytes || bus.empty()) return 0;
        const std::uint64_t off = a - va;
        if (page_bytes == 0) return bus[0] + off;
        const std::uint64_t pg = off / page_bytes;
        return pg < bus.size() ? bus[pg] + off % page_bytes : 0;
    }
};

struct ControllerInfo {
    std::string name;
    std::string kind;            // "emulated" | "snvme"
    std::uint32_t lba_bytes = 512;
    std::uint32_t mdts_bytes = 1u << 20;
    std::uint32_t queue_depth = 256;  // CAP.MQES + 1
    std::uint32_t num_io_queues = 0;
    std::uint32_t nsid = 1;
    std::uint64_t namespace_bytes = 0;
    bool device_dma = false;  // PRPs may name GPU memory (the controller DMAs into HBM)
};

// One backing range of an emulated namespace: namespace bytes
// [ns_offset, ns_offset + length) hold file bytes [file_offset, ...).
struct BackingRange {
    std::uint64_t ns_offset;
    std::uint64_t length;
    std::uint64_t file_offset;
};

struct ControllerStats {
    std::uint64_t dma_copies = 0;  // copy-engine transfers issued for GPU-memory PRPs
    std::uint64_t green_streams = 0;  // worker streams in the drives' own (green) context
    std::uint64_t image_bytes = 0; // memory media: bytes of the image loaded so far
    std::uint64_t load_ns = 0;     // time spent loading image chunks from the files
    std::uint64_t file_ns = 0;     // time spent in pread/pwrite of the backing files
    std::uint64_t sync_ns = 0;     // time spent waiting for the workers' own copies
    std::uint64_t max_command_ns = 0;  // longest single command execution
    std::uint64_t commands = 0;
    std::uint64_t read_bytes = 0;
    std::uint64_t write_bytes = 0;
    std::uint64_t errors = 0;
    std::uint64_t injected = 0;
};

// Fault seams for failure-detection tests (host side only; nothing faults a GPU).
enum class InjectKind : std::uint32_t {
    NONE = 0,
    MEDIA_ERROR = 1,    // complete the next N commands with an unrecovered read error
    DROP_COMPLETION = 2,  // execute but never post a CQE for the next N commands
    DELAY = 3,          // delay the next N commands by delay_us
};

class NvmeController {
public:
    virtual ~NvmeController() = default;
    virtual const ControllerInfo& info() const = 0;
    // Device-side pointers (GPU submitter).
    virtual QueuePairView device_queue(std::uint32_t i) const = 0;
    // Host-side pointers (host submitter, tests).
    virtual QueuePairView host_queue(std::uint32_t i) const = 0;
    // Make [ptr, ptr+bytes) (host or GPU memory) DMA-reachable by the controller.
    virtual Result<DmaMapping> map_dma(void* ptr, std::uint64_t bytes) = 0;
    virtual Status unmap_dma(const DmaMapping& m) = 0;
    // Quiesce queue i and reset its head/tail/phase (after a timeout).
    virtual Status reset_queue(std::uint32_t i) = 0;
    virtual ControllerStats stats() const = 0;
    // The emulated drive that answers this controller's queues, if any (its
    // namespace is backed by files and it takes host-side fault injection).
    virtual class EmulatedNvmeController* emulated_drive() { return nullptr; }
    // Makes every completed WRITE durable in the files a host process reads
    // (a drive with a volatile write cache writes it back). A real drive's
    // cache is flushed by the file system's own sync of those files.
    virtual Status flush() { return Status::Ok(); }
};

struct EmulatedControllerConfig {
    std::string name = "emu0";
    std::uint32_t num_io_queues = 64;
    std::uint32_t queue_depth = 256;
    std::uint32_t lba_bytes = 512;
    std::uint32_t mdts_bytes = 1u << 20;
    std::uint32_t worker_threads = 4;
    bool direct_io = false;            // O_DIRECT on backing files
    std::uint64_t namespace_bytes = 1ull << 46;
    std::uint32_t idle_spin_iters = 2000;  // polls before a worker sleeps
    std::uint32_t idle_sleep_us = 20;
    // Diagnostic: complete READ/WRITE commands without moving data (measures
    // the queue protocol and the GPU side alone; payloads are not valid).
    bool skip_data = false;
    // Page-cached mode: serve READs by copying from a shared mapping of the
    // backing file instead of pread (measured no faster on the GPU boxes).
    bool map_reads = false;
    // Media: the backing files (pread/pwrite) or an in-memory image of them.
    // The image is one page-locked arena of `image_budget_bytes` (0: 1 GiB),
    // allocated when the controller is created and handed out in
    // `image_chunk_bytes` pieces, each loaded from its file on first touch;
    // WRITEs update the image and are written through to the file before
    // their CQE, so the files stay the durable copy. Ranges past the arena are
    // served from the files. (Every CUDA allocation of the controller happens
    // at creation: a page-locked allocation while an io kernel waits for this
    // drive would order the drive's copies behind that kernel.)
    enum class Media : std::uint32_t { FILES = 0, MEMORY = 1 };
    Media media = Media::FILES;
    std::uint64_t image_chunk_bytes = 64ull << 20;
    std::uint64_t image_budget_bytes = 0;
    // Memory media only: a volatile write cache. A WRITE completes once its
    // bytes are in the image (for GPU memory: its copy queued on the worker's
    // stream, the CQE written after it); the dirty ranges reach the files on
    // FLUSH, on flush(), when a file is detached and when the drive stops.
    // Off: every WRITE is written through to its file before its CQE.
    bool write_back = false;
    // Queue pairs are created by a driver over rings it was given
    // (create_io_queue_pair) instead of existing from the start on the
    // controller's own rings.
    bool driver_created_queues = false;
    // CUDA device whose memory PRPs may name (-1: the current device at create;
    // ignored without CUDA). GPU destinations are DMA'd by the copy engines.
    int cuda_device = -1;
    // Sustained transfer rate of the emulated drive in GB/s (0: as fast as the
    // host and the copy engines go). Commands start no earlier than the drive
    // could have finished the bytes before them.
    double max_gbps = 0.0;
};

class EmulatedNvmeController final : public NvmeController {
public:
    static Result<std::unique_ptr<EmulatedNvmeController>> create(const EmulatedControllerConfig& cfg);
    ~EmulatedNvmeController() override;

    const ControllerInfo& info() const override { return info_; }
    QueuePairView device_queue(std::uint32_t i) const override;
    QueuePairView host_queue(std::uint32_t i) const override;
    Result<DmaMapping> map_dma(void* ptr, std::uint64_t bytes) override;
    Status unmap_dma(const DmaMapping& m) override;
    Status reset_queue(std::uint32_t i) override;
    ControllerStats stats() const override;
    EmulatedNvmeController* emulated_drive() override { return this; }

    // A DMA window whose memory kind the caller states (true: GPU memory), as
    // a driver that pinned the pages knows it. Returns the identity bus address.
    Result<std::uint64_t> map_window(void* ptr, std::uint64_t bytes, bool device);
    Status unmap_window(std::uint64_t bus);

    // What a queue-owning driver does with admin commands (driver_created_queues):
    // Create I/O CQ + SQ `qid` (1..num_io_queues) over host-memory rings of
    // `depth` entries, and Delete them. The doorbells of `qid` sit at the NVMe
    // offsets of the register file (bar0_host / bar0_device).
    Status create_io_queue_pair(std::uint32_t qid, void* sq, void* cq, std::uint32_t depth);
    Status delete_io_queue_pair(std::uint32_t qid);
    void* bar0_host() const { return bar_mem_.host; }
    void* bar0_device() const { return bar_mem_.device; }
    std::uint64_t bar0_bytes() const { return bar_mem_.bytes; }

    // Back namespace ranges with a file (opened by the controller itself).
    // Idempotent for identical ranges; overlapping ranges of another file fail.
    Status attach_file(const std::string& path, const std::vector<BackingRange>& ranges);
    Status detach_file(const std::string& path);

    // `status`: for MEDIA_ERROR, the CQE status field (type and code) to post; 0: unrecovered read error.
    void inject(InjectKind kind, std::uint32_t count, std::uint32_t delay_us = 0, std::uint32_t status = 0);

    // Stop workers (idempotent). Outstanding SQEs are left unexecuted; a write
    // cache is written back.
    void stop();
    Status flush() override;

private:
    explicit EmulatedNvmeController(const EmulatedControllerConfig& cfg);
    Status start();
    struct WorkerCtx;
    struct Backing;
    struct Seg {
        char* p;
        std::uint64_t n;
        bool device;
    };
    void worker_main(std::uint32_t worker);
    bool service_queue(std::uint32_t q, WorkerCtx& w);
    std::uint32_t execute(const Sqe& sqe, WorkerCtx& w, bool* drop_cqe, bool* on_stream);
    std::uint32_t move_span(bool read, Backing* b, int fd, const char* map, std::uint64_t map_len,
                            std::uint64_t foff, char* buf, std::uint64_t n, bool device, WorkerCtx& w);
    bool collect_iov(std::uint64_t prp1, std::uint64_t prp2, std::uint64_t bytes, std::vector<Seg>& iov) const;
    int window_kind(std::uint64_t addr, std::uint64_t bytes) const;  // -1 none, 0 host, 1 device
    char* image_at(Backing* b, std::uint64_t foff, std::uint64_t* avail);
    void pace(std::uint64_t bytes);

    struct QueueState {
        std::uint32_t sq_head = 0;
        std::uint32_t cq_tail = 0;
        std::uint32_t phase = 1;
        std::atomic<std::uint32_t> reset_request{0};
        std::atomic<std::uint32_t> fatal{0};
        // The rings this queue serves (host view) and the device address of its
        // CQ (completions written by a copy stream); owned by the worker, changed
        // only through a reset request.
        QueuePairView view{};
        char* cq_device = nullptr;
        bool enabled = true;
        // A driver's create/delete, applied by the worker with the next reset.
        QueuePairView pending_view{};
        char* pending_cq_device = nullptr;
        bool pending_enabled = true;
    };
    Status apply_queue_change(std::uint32_t i);
    struct Backing {
        std::string path;
        int fd = -1;
        std::vector<BackingRange> ranges;
        const char* map = nullptr;  // page-cached mode only; unmapped at destruction
        std::uint64_t map_len = 0;
        // memory media: one pointer per image chunk of the file (null until loaded)
        std::uint64_t file_bytes = 0;
        std::unique_ptr<std::atomic<char*>[]> chunks;
        std::size_t n_chunks = 0;
        std::mutex load_mu;
        // write cache: per image chunk the dirty byte range [first, second) within it
        std::unique_ptr<std::pair<std::uint64_t, std::uint64_t>[]> dirty;
        std::mutex dirty_mu;
    };
    void mark_dirty(Backing* b, std::uint64_t foff, std::uint64_t n);
    Status write_back(Backing* b);
    std::mutex streams_mu_;
    std::vector<cudaStream_t> worker_streams_;  // registered while their workers run
    struct Window {
        std::uint64_t base;
        std::uint64_t bytes;
        bool device;
    };

    EmulatedControllerConfig cfg_;
    ControllerInfo info_;
    int cuda_device_ = -1;
    HostMappedBuffer sq_mem_, cq_mem_, bar_mem_;
    std::vector<std::unique_ptr<QueueState>> qstate_;
    std::vector<std::thread> workers_;
    std::atomic<bool> stop_{false};

    mutable std::mutex map_mu_;  // guards backings_ / windows_ (workers take it shared-ish: short)
    std::vector<std::unique_ptr<Backing>> backings_;
    // flattened, sorted by ns_offset: (ns_offset, length, file_offset, fd)
    // map: a read-only shared mapping of the whole backing file (page-cached
    // mode), so READs copy straight from the page cache without a syscall.
    struct Span { std::uint64_t ns, len, foff; int fd; const char* map; std::uint64_t map_len; Backing* b; };
    std::shared_ptr<const std::vector<Span>> spans_;
    std::shared_ptr<const std::vector<Window>> windows_;

    std::atomic<std::uint64_t> image_bytes_{0};
    char* image_arena_ = nullptr;
    std::uint64_t image_arena_bytes_ = 0;
    bool image_arena_pinned_ = false;
    std::vector<char*> bounces_;  // one page-locked bounce buffer per worker (null without CUDA)
    std::atomic<std::uint64_t> st_load_ns_{0}, st_file_ns_{0}, st_sync_ns_{0}, st_max_cmd_ns_{0};
    std::atomic<std::uint64_t> pace_next_ns_{0};

    std::atomic<std::uint32_t> inject_kind_{0};
    std::atomic<std::uint32_t> inject_count_{0};
    std::atomic<std::uint32_t> inject_delay_us_{0};
    std::atomic<std::uint32_t> inject_status_{0};

    std::atomic<std::uint64_t> st_commands_{0}, st_read_{0}, st_write_{0}, st_errors_{0}, st_injected_{0};
    std::atomic<std::uint64_t> st_dma_copies_{0};
    std::atomic<std::uint64_t> st_green_streams_{0};
};

}  // namespace nvme
}  // namespace tutti
