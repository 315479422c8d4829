#pragma once
// GpuNvmeDataPath ("nvme-gpu"): GPU-initiated NVMe IO over one or more
// controllers (striped / RAID0 members are rows of the device table), with the
// paged scatter/gather fused into the io kernel.
//
// Parity with the reference's LocalNvmeDataPath / StripedDataPath
// (csrc/data_paths/local_nvme/local_nvme_data_path.cpp:429-2513,
// csrc/data_paths/striped_local_nvme/striped_data_path.cpp:314-2031):
//   open      -> device-resident file handle (extent table in HBM; no L1/L2
//                handle cache: 180 GB of HBM holds millions of ~100 B handles)
//   register  -> records the caller's buffer; the staging arena's PRP lists are
//                prebuilt once at initialize (register-time precomputation)
//   submit    -> coalesce requests into <= slot-sized commands with piece lists,
//                one H2D of the command blob, one kernel launch on the caller's
//                stream, async D2H of per-command status, one event
//   progress  -> event query; status aggregation into IoCompletionDetail
//   enqueue_wait -> cudaStreamWaitEvent on a consumer stream

#include <atomic>
#include <cstdint>
#include <chrono>
#include <memory>
#include <mutex>
#include <unordered_map>
#include <vector>

#include <tutti/payloads.h>
#include <tutti/spi/data_path.h>
#include <tutti/spi/resolver.h>

#include "../kernels/io_kernel.h"
#include "upload_plan.h"
#include "../nvme/controller.h"

namespace tutti {

struct GpuNvmeConfig {
    std::int32_t accel_id = 0;
    std::uint32_t leases = 64;            // queue pairs used per device (CTAs available)
    std::uint32_t max_ctas_per_op = 64;   // leases one submit may take
    std::uint32_t slots_per_lease = 4;    // staging slots per CTA (<= 64; x 8 below the queue depth)
    std::uint32_t slot_bytes = 1u << 20;  // <= 2 MiB
    std::uint64_t timeout_ns = 5ull * 1000 * 1000 * 1000;
    std::uint32_t max_targets = 1u << 20;
    std::uint32_t max_pieces_per_cmd = 256;
    bool timing = false;                  // per-command %globaltimer stamps
    // Split completion for reads: submit() launches only a one-warp-per-lease
    // kernel that queues the SQEs and exits; the waiting, data movement and
    // deadlines run in a drain launch that enqueue_wait() puts on the consumer's
    // stream, or that progress() launches itself once `async_fallback_us` have
    // passed without one (a host fallback). Off: one kernel does everything.
    bool async_completion = false;
    // Staging slots in write-combined host memory (drives stream into them, the
    // GPU reads them without snoops); writes that the drive reads back are slower.
    bool staging_write_combined = false;
    // A split read's drain is launched by progress() once the drives have posted
    // every CQE of the submitted wave (its data is in place), or after this
    // long, whichever comes first; enqueue_wait() launches it at once.
    std::uint32_t async_fallback_us = 1000;
    // Where the staging slots live. DEVICE: in HBM; the drives DMA into them
    // and the io kernel's bulk-copy movers scatter HBM -> HBM. HOST: page-
    // locked host memory the movers read over PCIe (zero-copy). AUTO: DEVICE
    // when every controller of the table can DMA into GPU memory.
    enum class Staging : std::uint32_t { AUTO = 0, HOST = 1, DEVICE = 2 };
    Staging staging = Staging::AUTO;
    // Per-op arenas (command list, pieces, statuses) created at initialize.
    // A submit that finds none large enough allocates one, and a page-locked
    // or device allocation orders later CUDA work (the drives' copies among
    // it) behind the kernels already running, so keep these sized for the
    // largest op in flight: 8 MiB holds a 32k-token Llama-3.1-8B restore.
    std::uint32_t prealloc_arenas = 4;
    std::uint32_t prealloc_arena_bytes = 8u << 20;
    // Direct reads: device memory registered with this data path is DMA-mapped
    // on every controller, and a read whose bytes land in whole 4 KiB pages of
    // it is served by the drive straight into those pages (PRPs built by the io
    // kernel from the memory's bus addresses); the io kernel moves no data for
    // it. Other reads (partial pages, fp8 transform, replicas, split
    // completion) keep the staged path.
    bool direct_reads = false;
};

// One row of the device table: a controller and the identity string the
// resolver puts into FileExtentPayload::controller / extents' device index.
struct GpuNvmeDevice {
    std::shared_ptr<nvme::NvmeController> controller;
    std::string identity;
};

struct SubmitProfile {
    double coalesce_ms = 0;  // validation + coalescing into commands/pieces
    double launch_ms = 0;    // arena fill, H2D, launch, D2H enqueue
    std::uint64_t commands = 0, requests = 0;
    std::uint64_t h2d_bytes = 0;  // command/piece/lease arena copied to the device
    std::uint64_t d2h_bytes = 0;  // statuses (and timing stamps) copied back
};

struct IoTimingSummary {
    std::uint64_t commands = 0;
    double queue_wait_us_p50 = 0, device_us_p50 = 0, move_us_p50 = 0, total_us_p50 = 0;
    double device_us_p99 = 0, total_us_p99 = 0;
};

class GpuNvmeDataPath final : public DataPath, public AsyncCompletion {
public:
    GpuNvmeDataPath(GpuNvmeConfig config, std::vector<GpuNvmeDevice> devices);
    ~GpuNvmeDataPath() override;

    const DataPathCapabilities& capabilities() const override { return caps_; }
    Status initialize(const DataPathConfig& config, ResourceProvider* resources) override;
    Status shutdown(std::uint64_t timeout_ns) override;
    Result<DataPathTarget> open(const ResolvedTarget& target) override;
    std::vector<Result<DataPathTarget>> open_many(const ResolvedTarget* const* targets, std::size_t count) override;
    Status close(DataPathTarget target) override;
    Result<RegistrationDomainKey> registration_domain(DataPathTarget target) const override;
    Result<DataPathMemory> register_memory(const DataPathMemoryView& view,
                                           const RegistrationDomainKey& domain) override;
    Status unregister_memory(DataPathMemory memory) override;
    SubmitOutcome submit(const DataPathRequest* requests, std::size_t count,
                         const HostSubmitContext& ctx) override;
    Result<ProgressResult> progress(ProgressBudget budget) override;
    Result<DataPathSnapshot> query(DataPathOp op) const override;
    Status release(DataPathOp op) override;
    Status enqueue_wait(const DataPathOp* ops, std::size_t count, cudaStream_t stream) override;

    // Telemetry of the last terminal op with timing enabled.
    IoTimingSummary last_timing() const;
    std::uint32_t free_leases() const;
    bool staging_on_device() const { return staging_on_device_; }
    SubmitProfile last_submit_profile() const {
        std::lock_guard<std::mutex> g(mu_);
        return last_submit_profile_;
    }

    // Support for the allocation-free C entry point (kernels/io_noalloc.cu).
    // None of these allocate: leases come from and return to a vector whose
    // capacity already covers every lease.
    std::int32_t accel_id() const { return cfg_.accel_id; }
    std::uint32_t noalloc_acquire_leases(std::uint32_t max, std::uint32_t* out);
    void noalloc_release_leases(const std::uint32_t* leases, std::uint32_t n, bool reset_dirty);
    void noalloc_fill_params(io::IoKernelParams& p) const;
    // True when [addr, addr+bytes) lies inside one registered memory.
    bool noalloc_memory_ok(std::uint64_t addr, std::uint64_t bytes) const;
    // True when `row` is an open target and [logical, logical+bytes) is inside it.
    bool noalloc_target_ok(std::uint32_t row, std::uint64_t logical, std::uint64_t bytes) const;

    // Test seams, all on the host (nothing faults on the device). Each arms
    // the next `count` occurrences:
    //  LAUNCH_FAILURE        the io kernel launch reports an error and is not
    //                        issued: every request of the submit is rejected;
    //  EVENT_RECORD_FAILURE  the completion event cannot be recorded after the
    //                        kernel was issued: the IO is irreversible, so the
    //                        submit synchronises and the op ends COMPLETED or
    //                        FAILED from its command statuses;
    //  QUERY_ERROR           progress() sees a CUDA error from the event query:
    //                        the op ends FAILED instead of staying IN_FLIGHT.
    enum class TestFault : std::uint32_t { LAUNCH_FAILURE = 0, EVENT_RECORD_FAILURE = 1, QUERY_ERROR = 2 };
    void test_inject(TestFault f, std::uint32_t count) {
        test_faults_[static_cast<std::uint32_t>(f)].store(count, std::memory_order_relaxed);
    }

private:
    bool take_test_fault(TestFault f) {
        auto& c = test_faults_[static_cast<std::uint32_t>(f)];
        std::uint32_t v = c.load(std::memory_order_relaxed);
        while (v && !c.compare_exchange_weak(v, v - 1, std::memory_order_relaxed)) {
        }
        return v != 0;
    }
    std::atomic<std::uint32_t> test_faults_[3]{};

    struct TargetRec {
        std::uint64_t generation = 0;
        std::uint32_t row = 0;
        std::uint64_t size = 0;
        std::string path;
        bool open = false;
    };
    struct MemoryRec {
        std::uint64_t generation = 0;
        char* base = nullptr;
        std::uint64_t size = 0;
        DataPathMemoryKind kind = DataPathMemoryKind::DEVICE;
    };
    struct Arena {
        std::size_t capacity = 0;    // bytes
        char* host = nullptr;        // page-locked, mapped: the status words are written here by the kernel
        char* host_dev = nullptr;    // device address of `host`
        char* dev = nullptr;
        cudaEvent_t event = nullptr;      // after the (drain) kernel and the status copy-back
        cudaEvent_t submitted = nullptr;  // split completion: after the submit-phase kernel
        cudaEvent_t uploaded = nullptr;   // after the command list's upload (on the upload stream)
    };
    struct OpRec {
        std::uint64_t generation = 0;
        IoState state = IoState::IN_FLIGHT;
        Status status;
        std::unique_ptr<Arena> arena;
        std::vector<std::uint32_t> leases;
        std::uint32_t n_cmds = 0;
        std::size_t status_off = 0;
        std::size_t timing_off = 0;
        std::vector<std::uint32_t> cmd_first_req;  // request index range per command
        std::vector<std::uint32_t> piece_req;      // request index per piece
        std::vector<std::uint32_t> cmd_first_piece;
        std::vector<std::uint64_t> req_bytes;       // per accepted request
        std::vector<std::uint32_t> req_input_index; // accepted -> input index
        IoCompletionDetail detail;
        std::uint64_t bytes = 0;
        bool timing = false;
        // split completion: the drain launch still to be issued
        bool drain_pending = false;
        io::IoKernelParams kp{};
        std::uint32_t ctas = 0;
        std::size_t copy_back_bytes = 0;
        std::size_t carry_off = 0;  // split completion: hand-over records in the mapped host half
        cudaStream_t stream = nullptr;
        std::chrono::steady_clock::time_point submitted_at{};
    };

    // Host->device copies an open still owes (extents, a target row).
    Result<DataPathTarget> open_locked(const ResolvedTarget& target, std::vector<DeviceUpload>& uploads);
    Status flush_uploads(std::vector<DeviceUpload>& uploads);
    Status init_device_side();
    Result<std::unique_ptr<Arena>> take_arena(std::size_t bytes);
    void return_arena(std::unique_ptr<Arena> a);
    void finish_op(OpRec& op);
    Status launch_drain(OpRec& op, cudaStream_t stream);
    // Split completion: the submit launch has finished and every CQE it waits
    // for has been posted (read from the host-resident CQs and cursors).
    bool split_data_ready(const OpRec& op) const;
    Status reset_dirty_queues(const std::vector<std::uint32_t>& leases);
    void retire_lease_locked(std::uint32_t lease, const Status& why);
    void return_leases_locked(const std::vector<std::uint32_t>& leases);

    GpuNvmeConfig cfg_;
    std::vector<GpuNvmeDevice> devs_;
    DataPathCapabilities caps_;
    mutable std::mutex mu_;
    bool initialized_ = false;

    // device-side tables
    io::DevTarget* d_targets_ = nullptr;
    io::DevDevice* d_devices_ = nullptr;
    std::vector<nvme::QueuePairView*> d_queue_views_;
    std::vector<io::QueueCursor*> d_cursors_;   // device addresses of cursor_mem_
    std::vector<HostMappedBuffer> cursor_mem_;  // per device: one cursor per lease, in mapped host memory
    std::vector<char*> extent_chunks_;
    std::size_t extent_chunk_used_ = 0;
    static constexpr std::size_t kExtentChunkBytes = 16u << 20;

    // staging arena + PRP-list pages (host mapped), one per lease x slot; with
    // device staging the arena is staging_hbm_ (cudaMalloc) and staging_ is unused
    HostMappedBuffer staging_, prp_;
    char* staging_hbm_ = nullptr;
    // Command lists and target rows go to the device on this stream, never on
    // a stream where an io kernel may be running: a copy waiting behind a
    // kernel that waits for the drives could hold up the drives' own copies.
    cudaStream_t upload_stream_ = nullptr;
    bool staging_on_device_ = false;
    char* staging_base() const { return staging_on_device_ ? staging_hbm_ : static_cast<char*>(staging_.device); }
    // Per controller: the DMA mappings of the staging arena and the PRP-list
    // pages. Every controller must hand out the same bus addresses (one set of
    // prebuilt PRP lists serves all drives).
    std::vector<nvme::DmaMapping> staging_maps_, prp_maps_;
    // Device copies of the bus-address tables the io kernel builds PRPs from:
    // one entry per 4 KiB staging page, one per slot's PRP-list page.
    std::uint64_t* d_page_bus_ = nullptr;
    std::uint64_t* d_list_bus_ = nullptr;
    // Direct reads: per registered device memory, its mapping on every
    // controller and the device copy of its bus table; the device region
    // table the kernels search (a new table per change, the old ones kept
    // until close since ops in flight may hold them); one PRP-list page per
    // staging slot for direct commands.
    struct DirectRegion {
        char* base = nullptr;
        std::uint64_t bytes = 0;
        std::vector<nvme::DmaMapping> maps;  // one per controller
        std::uint64_t* d_bus = nullptr;
    };
    std::unordered_map<std::uint64_t, DirectRegion> direct_regions_;  // memory token ->
    io::DmaRegion* d_regions_ = nullptr;
    std::uint32_t n_regions_ = 0;
    std::vector<void*> retired_device_tables_;
    HostMappedBuffer direct_lists_;
    std::vector<nvme::DmaMapping> direct_list_maps_;
    std::uint64_t* d_direct_list_bus_ = nullptr;
    Status map_direct_region_locked(std::uint64_t token, char* base, std::uint64_t bytes);
    void unmap_direct_region_locked(std::uint64_t token);
    Status publish_regions_locked();
    std::uint32_t lba_ = 512;  // largest LBA size of the device table

    std::vector<TargetRec> targets_;
    std::vector<std::uint32_t> free_target_rows_;
    std::unordered_map<std::string, std::uint32_t> target_by_path_;
    std::unordered_map<std::uint64_t, MemoryRec> memories_;
    std::unordered_map<std::uint64_t, std::unique_ptr<OpRec>> ops_;
    std::vector<std::uint32_t> free_leases_;
    std::vector<bool> retired_;  // leases whose queues could not be reset after a timeout
    std::vector<std::unique_ptr<Arena>> arena_pool_;
    std::uint64_t next_token_ = 1;
    IoTimingSummary last_timing_;
    SubmitProfile last_submit_profile_;
    std::uint32_t cmd_bytes_ = 0;
};

}  // namespace tutti
