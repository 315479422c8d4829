// Host-emulated NVMe controller: the "drive" side of the queue protocol.
//
// Each worker thread owns queues q with q % workers == worker, so a queue's
// head/tail/phase state has exactly one writer and needs no lock. A worker
// observes the SQ tail doorbell (acquire), copies each new SQE, executes it
// against the namespace's file-backed ranges into/out of the PRP-described
// buffers, and posts a CQE whose dword 3 (CID, phase, status) is stored last
// with release semantics, which is the order a PCIe device's posted writes
// give a CQ poller.
//
// GPU-memory PRPs (staging slots or pages in HBM) are served by the copy
// engines: the worker issues cudaMemcpyAsync on its own non-blocking stream
// and, for a READ, has that same stream write the CQE's dword 3
// (cuStreamWriteValue32) after the copy, so the completion cannot overtake
// the data and the worker never waits for the transfer. Measured on B200:
// one 1 MiB host->HBM copy per command runs at the copy engines' 45.6 GB/s,
// and a kernel that spins on a CQ never delays copies issued on the worker's
// stream.

#include "controller.h"

#include <cuda.h>
#include <cuda_runtime_api.h>
#include <fcntl.h>
#include <immintrin.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <sys/uio.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>

namespace tutti {
namespace nvme {

namespace {
inline std::uint32_t load_acquire(const std::uint32_t* p) { return __atomic_load_n(p, __ATOMIC_ACQUIRE); }
inline void store_release(std::uint32_t* p, std::uint32_t v) { __atomic_store_n(p, v, __ATOMIC_RELEASE); }

std::uint64_t now_ns() {
    return static_cast<std::uint64_t>(
        std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now().time_since_epoch())
            .count());
}

// With TUTTI_EMULATOR_STREAMS=green the drives' CUDA streams live in a
// context of their own: a green context over the whole device, which shares
// the application's address space (copies reach its HBM) but not its
// hardware queues, so no stream-ordered wait of the application can sit in
// front of a drive's copies. Off by default: the stalls that first suggested
// it were kernel loads (see the data path's notes), not queue sharing.
// Driver entry points are looked up through the runtime (no libcuda link).
struct GreenDriveStreams {
    using DeviceGet = CUresult (*)(CUdevice*, int);
    using GetResource = CUresult (*)(CUdevice, CUdevResource*, CUdevResourceType);
    using GenerateDesc = CUresult (*)(CUdevResourceDesc*, CUdevResource*, unsigned int);
    using CtxCreate = CUresult (*)(CUgreenCtx*, CUdevResourceDesc, CUdevice, unsigned int);
    using StreamCreate = CUresult (*)(CUstream*, CUgreenCtx, unsigned int, int);
    DeviceGet device_get = nullptr;
    GetResource get_resource = nullptr;
    GenerateDesc generate_desc = nullptr;
    CtxCreate ctx_create = nullptr;
    StreamCreate stream_create = nullptr;
    std::mutex mu;
    std::vector<std::pair<int, CUgreenCtx>> ctx_of_device;

    template <typename F>
    static F lookup(const char* name) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        return reinterpret_cast<F>(p);
    }
    GreenDriveStreams() {
        device_get = lookup<DeviceGet>("cuDeviceGet");
        get_resource = lookup<GetResource>("cuDeviceGetDevResource");
        generate_desc = lookup<GenerateDesc>("cuDevResourceGenerateDesc");
        ctx_create = lookup<CtxCreate>("cuGreenCtxCreate");
        stream_create = lookup<StreamCreate>("cuGreenCtxStreamCreate");
    }
    // A non-blocking stream in the device's drive context (nullptr: unavailable).
    cudaStream_t create(int device) {
        if (!device_get || !get_resource || !generate_desc || !ctx_create || !stream_create) return nullptr;
        std::lock_guard<std::mutex> g(mu);
        CUgreenCtx ctx = nullptr;
        for (auto& kv : ctx_of_device)
            if (kv.first == device) ctx = kv.second;
        if (!ctx) {
            CUdevice dev = 0;
            CUdevResource all{};
            CUdevResourceDesc desc = nullptr;
            if (device_get(&dev, device) != CUDA_SUCCESS || get_resource(dev, &all, CU_DEV_RESOURCE_TYPE_SM) != CUDA_SUCCESS ||
                generate_desc(&desc, &all, 1) != CUDA_SUCCESS ||
                ctx_create(&ctx, desc, dev, CU_GREEN_CTX_DEFAULT_STREAM) != CUDA_SUCCESS)
                return nullptr;
            ctx_of_device.emplace_back(device, ctx);  // lives as long as the process
        }
        CUstream st = nullptr;
        if (stream_create(&st, ctx, CU_STREAM_NON_BLOCKING, 0) != CUDA_SUCCESS) return nullptr;
        return reinterpret_cast<cudaStream_t>(st);
    }
};

// A stream for a drive worker on `device`; *green tells where it lives.
cudaStream_t create_drive_stream(int device, bool* green) {
    static GreenDriveStreams greens;
    *green = false;
    const char* how = std::getenv("TUTTI_EMULATOR_STREAMS");
    if (how && std::strcmp(how, "green") == 0) {
        if (cudaStream_t s = greens.create(device)) {
            *green = true;
            return s;
        }
    }
    cudaStream_t s = nullptr;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return s;
}

// cuStreamWriteValue32, looked up through the runtime so the library does not
// link libcuda (it must import on machines without a driver).
using WriteValue32Fn = CUresult (*)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);
WriteValue32Fn write_value32() {
    static WriteValue32Fn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuStreamWriteValue32", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return static_cast<WriteValue32Fn>(nullptr);
        }
        return reinterpret_cast<WriteValue32Fn>(p);
    }();
    return fn;
}
}  // namespace

// Per worker thread: the CUDA stream its copy-engine transfers and stream-
// posted CQEs go to, and a page-locked bounce buffer for file media <-> GPU
// memory.
struct EmulatedNvmeController::WorkerCtx {
    cudaStream_t stream = nullptr;
    bool cuda = false;
    char* bounce = nullptr;
    std::uint64_t bounce_bytes = 0;
    bool stream_dirty = false;  // work was issued on `stream` since the last synchronize
};

EmulatedNvmeController::EmulatedNvmeController(const EmulatedControllerConfig& cfg) : cfg_(cfg) {
    info_.name = cfg.name;
    info_.kind = "emulated";
    info_.lba_bytes = cfg.lba_bytes;
    info_.mdts_bytes = cfg.mdts_bytes;
    info_.queue_depth = cfg.queue_depth;
    info_.num_io_queues = cfg.num_io_queues;
    info_.nsid = 1;
    info_.namespace_bytes = cfg.namespace_bytes;
    spans_ = std::make_shared<const std::vector<Span>>();
    windows_ = std::make_shared<const std::vector<Window>>();
}

Result<std::unique_ptr<EmulatedNvmeController>> EmulatedNvmeController::create(
    const EmulatedControllerConfig& cfg) {
    using R = Result<std::unique_ptr<EmulatedNvmeController>>;
    if (cfg.num_io_queues == 0 || cfg.num_io_queues > 4096)
        return R::Failure({StatusCode::INVALID_ARGUMENT, "num_io_queues must be in [1, 4096]"});
    if (cfg.queue_depth < 2 || cfg.queue_depth > 65536)
        return R::Failure({StatusCode::INVALID_ARGUMENT, "queue_depth must be in [2, 65536]"});
    if (cfg.lba_bytes != 512 && cfg.lba_bytes != 4096)
        return R::Failure({StatusCode::INVALID_ARGUMENT, "lba_bytes must be 512 or 4096"});
    if (cfg.mdts_bytes < 4096 || (cfg.mdts_bytes % 4096) != 0 ||
        cfg.mdts_bytes / cfg.lba_bytes > 65536)
        return R::Failure({StatusCode::INVALID_ARGUMENT, "mdts_bytes must be a 4 KiB multiple within NLB range"});
    if (cfg.image_chunk_bytes < (1u << 20) || cfg.image_chunk_bytes % 4096)
        return R::Failure({StatusCode::INVALID_ARGUMENT, "image_chunk_bytes must be a 4 KiB multiple >= 1 MiB"});
    if (cfg.max_gbps < 0) return R::Failure({StatusCode::INVALID_ARGUMENT, "max_gbps must be >= 0"});
    std::unique_ptr<EmulatedNvmeController> c(new EmulatedNvmeController(cfg));
    Status st = c->start();
    if (!st.ok()) return R::Failure(st);
    return R(std::move(c));
}

Status EmulatedNvmeController::start() {
    if (cuda_device_present()) {
        int dev = cfg_.cuda_device;
        if (dev < 0 && cudaGetDevice(&dev) != cudaSuccess) {
            cudaGetLastError();
            dev = 0;
        }
        cuda_device_ = dev;
        info_.device_dma = write_value32() != nullptr;
    }
    const std::uint64_t nq = cfg_.num_io_queues, d = cfg_.queue_depth;
    auto sq = host_mapped_alloc(nq * d * sizeof(Sqe));
    if (!sq.ok()) return sq.status();
    sq_mem_ = sq.value();
    auto cq = host_mapped_alloc(nq * d * sizeof(Cqe));
    if (!cq.ok()) return cq.status();
    cq_mem_ = cq.value();
    // Register file: doorbells of the admin queue (0) and I/O queues 1..nq.
    auto bar = host_mapped_alloc(kDoorbellBase + 8 * (nq + 1));
    if (!bar.ok()) return bar.status();
    bar_mem_ = bar.value();
    for (std::uint32_t i = 0; i < nq; ++i) {
        qstate_.emplace_back(new QueueState());
        QueueState& qs = *qstate_.back();
        qs.view = host_queue(i);
        if (cq_mem_.device)
            qs.cq_device = static_cast<char*>(cq_mem_.device) + std::uint64_t(i) * d * sizeof(Cqe);
        qs.enabled = !cfg_.driver_created_queues;
    }
    std::uint32_t nw = std::max<std::uint32_t>(1, std::min(cfg_.worker_threads, cfg_.num_io_queues));
    // All CUDA allocations happen here, before any io kernel can wait on this drive.
    if (cfg_.media == EmulatedControllerConfig::Media::MEMORY) {
        const std::uint64_t cb = cfg_.image_chunk_bytes;
        std::uint64_t want = cfg_.image_budget_bytes ? cfg_.image_budget_bytes : (1ull << 30);
        want = (want + cb - 1) / cb * cb;
        void* p = nullptr;
        if (cuda_device_ >= 0) {
            if (cudaHostAlloc(&p, want, cudaHostAllocPortable) != cudaSuccess) {
                cudaGetLastError();
                return {StatusCode::RESOURCE_EXHAUSTED, "cannot page-lock the emulated drive's image arena"};
            }
            image_arena_pinned_ = true;
        } else if (posix_memalign(&p, 4096, want) != 0) {
            return {StatusCode::RESOURCE_EXHAUSTED, "cannot allocate the emulated drive's image arena"};
        }
        image_arena_ = static_cast<char*>(p);
        image_arena_bytes_ = want;
    }
    bounces_.assign(nw, nullptr);
    if (cuda_device_ >= 0) {
        for (auto& b : bounces_) {
            void* p = nullptr;
            if (cudaHostAlloc(&p, cfg_.mdts_bytes, cudaHostAllocPortable) != cudaSuccess) {
                cudaGetLastError();
                return {StatusCode::RESOURCE_EXHAUSTED, "cannot page-lock the emulated drive's bounce buffers"};
            }
            b = static_cast<char*>(p);
        }
    }
    for (std::uint32_t w = 0; w < nw; ++w) workers_.emplace_back([this, w] { worker_main(w); });
    return Status::Ok();
}

EmulatedNvmeController::~EmulatedNvmeController() {
    stop();
    for (auto& b : backings_) {
        if (b->map) ::munmap(const_cast<char*>(b->map), b->map_len);
        if (b->fd >= 0) ::close(b->fd);
    }
    if (image_arena_) {
        if (image_arena_pinned_)
            cudaFreeHost(image_arena_);
        else
            std::free(image_arena_);
    }
    for (char* b : bounces_)
        if (b) cudaFreeHost(b);
    host_mapped_free(sq_mem_);
    host_mapped_free(cq_mem_);
    host_mapped_free(bar_mem_);
}

void EmulatedNvmeController::stop() {
    stop_.store(true);
    for (auto& t : workers_)
        if (t.joinable()) t.join();
    workers_.clear();
    if (cfg_.write_back) (void)flush();  // the workers drained their streams on exit
}

void EmulatedNvmeController::mark_dirty(Backing* b, std::uint64_t foff, std::uint64_t n) {
    const std::uint64_t cb = cfg_.image_chunk_bytes;
    const std::size_t ci = static_cast<std::size_t>(foff / cb);
    const std::uint64_t lo = foff % cb, hi = lo + n;  // n never crosses the chunk
    std::lock_guard<std::mutex> g(b->dirty_mu);
    auto& d = b->dirty[ci];
    if (d.second <= d.first) {
        d = {lo, hi};
    } else {
        d.first = std::min(d.first, lo);
        d.second = std::max(d.second, hi);
    }
}

Status EmulatedNvmeController::write_back(Backing* b) {
    if (!b->dirty || b->fd < 0) return Status::Ok();
    const std::uint64_t cb = cfg_.image_chunk_bytes;
    std::vector<std::pair<std::size_t, std::pair<std::uint64_t, std::uint64_t>>> todo;
    {
        std::lock_guard<std::mutex> g(b->dirty_mu);
        for (std::size_t ci = 0; ci < b->n_chunks; ++ci) {
            auto& d = b->dirty[ci];
            if (d.second > d.first) todo.push_back({ci, d});
            d = {0, 0};
        }
    }
    Status first;
    for (const auto& t : todo) {
        const char* base = b->chunks[t.first].load(std::memory_order_acquire);
        const std::uint64_t lo = t.second.first, len = t.second.second - t.second.first;
        std::uint64_t done = 0;
        const std::uint64_t t0 = now_ns();
        while (base && done < len) {
            const ssize_t w = ::pwrite(b->fd, base + lo + done, len - done, static_cast<off_t>(t.first * cb + lo + done));
            if (w < 0 && errno == EINTR) continue;
            if (w <= 0) break;
            done += static_cast<std::uint64_t>(w);
        }
        st_file_ns_.fetch_add(now_ns() - t0, std::memory_order_relaxed);
        if (done < len) {
            mark_dirty(b, t.first * cb + lo, len);  // keep it for the next flush
            if (first.ok()) first = {StatusCode::DEVICE_ERROR, "write-back of " + b->path + " failed"};
        }
    }
    if (!todo.empty() && ::fdatasync(b->fd) != 0 && first.ok())
        first = {StatusCode::DEVICE_ERROR, "fdatasync of " + b->path + " failed"};
    return first;
}

Status EmulatedNvmeController::flush() {
    if (!cfg_.write_back) {
        std::lock_guard<std::mutex> g(map_mu_);
        for (auto& b : backings_)
            if (b->fd >= 0) ::fdatasync(b->fd);
        return Status::Ok();
    }
    // Every copy queued so far has landed in the image (the WRITEs that completed
    // posted their CQEs after their copies; this also waits for those in flight).
    {
        std::lock_guard<std::mutex> g(streams_mu_);
        for (cudaStream_t st : worker_streams_)
            if (cudaStreamSynchronize(st) != cudaSuccess) cudaGetLastError();
    }
    std::vector<Backing*> bs;
    {
        std::lock_guard<std::mutex> g(map_mu_);
        for (auto& b : backings_) bs.push_back(b.get());
    }
    Status first;
    for (Backing* b : bs) {
        Status s = write_back(b);
        if (first.ok() && !s.ok()) first = s;
    }
    return first;
}

static QueuePairView make_view(char* sq, char* cq, char* bar, std::uint32_t i, std::uint32_t depth,
                               std::uint32_t nsid) {
    QueuePairView v{};
    v.sq = reinterpret_cast<Sqe*>(sq) + std::uint64_t(i) * depth;
    v.cq = reinterpret_cast<const Cqe*>(cq) + std::uint64_t(i) * depth;
    v.qid = i + 1;  // queue 0 is the admin queue on a real controller
    v.sq_doorbell = reinterpret_cast<std::uint32_t*>(bar + sq_doorbell_offset(v.qid));
    v.cq_doorbell = reinterpret_cast<std::uint32_t*>(bar + cq_doorbell_offset(v.qid));
    v.depth = depth;
    v.nsid = nsid;
    return v;
}

QueuePairView EmulatedNvmeController::device_queue(std::uint32_t i) const {
    if (!sq_mem_.device) return host_queue(i);
    return make_view(static_cast<char*>(sq_mem_.device), static_cast<char*>(cq_mem_.device),
                     static_cast<char*>(bar_mem_.device), i, cfg_.queue_depth, info_.nsid);
}

QueuePairView EmulatedNvmeController::host_queue(std::uint32_t i) const {
    return make_view(static_cast<char*>(sq_mem_.host), static_cast<char*>(cq_mem_.host),
                     static_cast<char*>(bar_mem_.host), i, cfg_.queue_depth, info_.nsid);
}

Result<DmaMapping> EmulatedNvmeController::map_dma(void* ptr, std::uint64_t bytes) {
    using R = Result<DmaMapping>;
    if (!ptr || bytes == 0) return R::Failure({StatusCode::INVALID_ARGUMENT, "empty DMA window"});
    bool device = false;
    if (cuda_device_ >= 0) {
        cudaPointerAttributes a{};
        if (cudaPointerGetAttributes(&a, ptr) == cudaSuccess)
            device = a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
        else
            cudaGetLastError();
    }
    auto bus = map_window(ptr, bytes, device);
    if (!bus.ok()) return R::Failure(bus.status());
    DmaMapping m;
    m.va = reinterpret_cast<std::uint64_t>(ptr);
    m.bytes = bytes;
    m.bus = {bus.value()};
    return R(std::move(m));
}

Status EmulatedNvmeController::unmap_dma(const DmaMapping& m) { return unmap_window(m.va); }

Result<std::uint64_t> EmulatedNvmeController::map_window(void* ptr, std::uint64_t bytes, bool device) {
    using R = Result<std::uint64_t>;
    if (!ptr || bytes == 0) return R::Failure({StatusCode::INVALID_ARGUMENT, "empty DMA window"});
    if (device && !info_.device_dma)
        return R::Failure({StatusCode::UNSUPPORTED, "this controller cannot DMA into GPU memory (no stream memory ops)"});
    std::lock_guard<std::mutex> g(map_mu_);
    auto next = std::make_shared<std::vector<Window>>(*std::atomic_load(&windows_));
    next->push_back({reinterpret_cast<std::uint64_t>(ptr), bytes, device});
    std::atomic_store(&windows_, std::shared_ptr<const std::vector<Window>>(next));
    // The emulator's IOMMU is the identity: bus address == virtual address.
    return R(reinterpret_cast<std::uint64_t>(ptr));
}

Status EmulatedNvmeController::unmap_window(std::uint64_t bus) {
    std::lock_guard<std::mutex> g(map_mu_);
    auto next = std::make_shared<std::vector<Window>>(*std::atomic_load(&windows_));
    auto it = std::find_if(next->begin(), next->end(), [&](const Window& w) { return w.base == bus; });
    if (it == next->end()) return {StatusCode::NOT_FOUND, "no DMA window at that address"};
    next->erase(it);
    std::atomic_store(&windows_, std::shared_ptr<const std::vector<Window>>(next));
    return Status::Ok();
}

Status EmulatedNvmeController::apply_queue_change(std::uint32_t i) {
    QueueState& qs = *qstate_[i];
    if (workers_.empty()) {
        // No worker runs (stopped): apply in place.
        qs.view = qs.pending_view;
        qs.cq_device = qs.pending_cq_device;
        qs.enabled = qs.pending_enabled;
        qs.sq_head = qs.cq_tail = 0;
        qs.phase = 1;
        return Status::Ok();
    }
    qs.reset_request.store(2, std::memory_order_release);
    auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(5);
    while (qs.reset_request.load(std::memory_order_acquire) != 0) {
        if (std::chrono::steady_clock::now() > deadline)
            return {StatusCode::TIMEOUT, "queue change not acknowledged by the drive"};
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    return Status::Ok();
}

Status EmulatedNvmeController::create_io_queue_pair(std::uint32_t qid, void* sq, void* cq, std::uint32_t depth) {
    if (!cfg_.driver_created_queues) return {StatusCode::UNSUPPORTED, "queues are not driver-created"};
    if (qid == 0 || qid > qstate_.size()) return {StatusCode::OUT_OF_RANGE, "invalid queue identifier"};
    if (!sq || !cq) return {StatusCode::INVALID_ARGUMENT, "queue rings are required"};
    if (depth < 2 || depth > info_.queue_depth) return {StatusCode::INVALID_ARGUMENT, "queue size exceeds CAP.MQES"};
    QueueState& qs = *qstate_[qid - 1];
    if (qs.enabled) return {StatusCode::BUSY, "queue identifier in use"};
    char* bar = static_cast<char*>(bar_mem_.host);
    QueuePairView v{};
    v.sq = static_cast<Sqe*>(sq);
    v.cq = static_cast<const Cqe*>(cq);
    v.sq_doorbell = reinterpret_cast<std::uint32_t*>(bar + sq_doorbell_offset(qid));
    v.cq_doorbell = reinterpret_cast<std::uint32_t*>(bar + cq_doorbell_offset(qid));
    v.depth = depth;
    v.qid = qid;
    v.nsid = info_.nsid;
    void* cq_dev = nullptr;
    if (cuda_device_ >= 0 && cudaHostGetDevicePointer(&cq_dev, cq, 0) != cudaSuccess) {
        cudaGetLastError();
        cq_dev = nullptr;  // not device-mapped: completions are posted by the host
    }
    std::memset(cq, 0, std::size_t(depth) * sizeof(Cqe));
    qs.pending_view = v;
    qs.pending_cq_device = static_cast<char*>(cq_dev);
    qs.pending_enabled = true;
    return apply_queue_change(qid - 1);
}

Status EmulatedNvmeController::delete_io_queue_pair(std::uint32_t qid) {
    if (!cfg_.driver_created_queues) return {StatusCode::UNSUPPORTED, "queues are not driver-created"};
    if (qid == 0 || qid > qstate_.size()) return {StatusCode::OUT_OF_RANGE, "invalid queue identifier"};
    QueueState& qs = *qstate_[qid - 1];
    if (!qs.enabled) return {StatusCode::NOT_FOUND, "queue identifier not in use"};
    qs.pending_view = QueuePairView{};
    qs.pending_cq_device = nullptr;
    qs.pending_enabled = false;
    return apply_queue_change(qid - 1);
}

Status EmulatedNvmeController::reset_queue(std::uint32_t i) {
    if (i >= qstate_.size()) return {StatusCode::OUT_OF_RANGE, "queue index"};
    QueueState& qs = *qstate_[i];
    qs.reset_request.store(1);
    auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(5);
    while (qs.reset_request.load() != 0) {
        if (std::chrono::steady_clock::now() > deadline)
            return {StatusCode::TIMEOUT, "queue reset not acknowledged"};
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    return Status::Ok();
}

ControllerStats EmulatedNvmeController::stats() const {
    ControllerStats s;
    s.commands = st_commands_.load();
    s.read_bytes = st_read_.load();
    s.write_bytes = st_write_.load();
    s.errors = st_errors_.load();
    s.injected = st_injected_.load();
    s.dma_copies = st_dma_copies_.load();
    s.green_streams = st_green_streams_.load();
    s.image_bytes = image_bytes_.load();
    s.load_ns = st_load_ns_.load();
    s.file_ns = st_file_ns_.load();
    s.sync_ns = st_sync_ns_.load();
    s.max_command_ns = st_max_cmd_ns_.load();
    return s;
}

Status EmulatedNvmeController::attach_file(const std::string& path, const std::vector<BackingRange>& ranges) {
    std::lock_guard<std::mutex> g(map_mu_);
    Backing* target = nullptr;
    for (auto& b : backings_) {
        if (b->path == path) {
            // Same file: accept ranges already present, add new ones.
            for (const auto& r : ranges) {
                bool have = std::any_of(b->ranges.begin(), b->ranges.end(), [&](const BackingRange& x) {
                    return x.ns_offset == r.ns_offset && x.length == r.length && x.file_offset == r.file_offset;
                });
                if (!have) b->ranges.push_back(r);
            }
            target = b.get();
            break;
        }
    }
    if (!target) {
        int flags = O_RDWR | O_CLOEXEC;
        int fd = ::open(path.c_str(), flags | (cfg_.direct_io ? O_DIRECT : 0));
        if (fd < 0 && cfg_.direct_io) fd = ::open(path.c_str(), flags);  // e.g. tmpfs rejects O_DIRECT
        if (fd < 0) return {StatusCode::NOT_FOUND, "emulated namespace cannot open " + path};
        auto nb = std::make_unique<Backing>();
        nb->path = path;
        nb->fd = fd;
        nb->ranges = ranges;
        struct stat st {};
        if (::fstat(fd, &st) == 0 && st.st_size > 0) nb->file_bytes = static_cast<std::uint64_t>(st.st_size);
        if (!cfg_.direct_io && cfg_.map_reads && nb->file_bytes) {
            // Page-cached mode: READs copy from a shared read-only mapping (the page
            // cache itself) instead of pread; WRITEs keep pwrite, which the mapping sees.
            void* m = ::mmap(nullptr, static_cast<std::size_t>(nb->file_bytes), PROT_READ, MAP_SHARED, fd, 0);
            if (m != MAP_FAILED) {
                nb->map = static_cast<const char*>(m);
                nb->map_len = nb->file_bytes;
            }
        }
        if (cfg_.media == EmulatedControllerConfig::Media::MEMORY && nb->file_bytes) {
            nb->n_chunks = static_cast<std::size_t>((nb->file_bytes + cfg_.image_chunk_bytes - 1) / cfg_.image_chunk_bytes);
            nb->chunks.reset(new std::atomic<char*>[nb->n_chunks]);
            for (std::size_t i = 0; i < nb->n_chunks; ++i) nb->chunks[i].store(nullptr);
            nb->dirty.reset(new std::pair<std::uint64_t, std::uint64_t>[nb->n_chunks]());
        }
        target = nb.get();
        backings_.push_back(std::move(nb));
    }
    (void)target;
    auto spans = std::make_shared<std::vector<Span>>();
    for (auto& b : backings_)
        for (auto& r : b->ranges)
            spans->push_back({r.ns_offset, r.length, r.file_offset, b->fd, b->map, b->map_len, b.get()});
    std::sort(spans->begin(), spans->end(), [](const Span& a, const Span& b) { return a.ns < b.ns; });
    for (std::size_t i = 1; i < spans->size(); ++i) {
        const Span& p = (*spans)[i - 1];
        const Span& c = (*spans)[i];
        if (p.ns + p.len > c.ns && !(p.ns == c.ns && p.fd == c.fd && p.foff == c.foff))
            return {StatusCode::INVALID_ARGUMENT, "namespace ranges overlap"};
    }
    spans->erase(std::unique(spans->begin(), spans->end(),
                             [](const Span& a, const Span& b) { return a.ns == b.ns && a.fd == b.fd; }),
                 spans->end());
    std::atomic_store(&spans_, std::shared_ptr<const std::vector<Span>>(spans));
    return Status::Ok();
}

Status EmulatedNvmeController::detach_file(const std::string& path) {
    std::lock_guard<std::mutex> g(map_mu_);
    auto it = std::find_if(backings_.begin(), backings_.end(), [&](const std::unique_ptr<Backing>& b) {
        return b->path == path;
    });
    if (it == backings_.end()) return {StatusCode::NOT_FOUND, "not attached: " + path};
    if (cfg_.write_back) {
        {
            std::lock_guard<std::mutex> sg(streams_mu_);
            for (cudaStream_t st : worker_streams_)
                if (cudaStreamSynchronize(st) != cudaSuccess) cudaGetLastError();
        }
        TUTTI_RETURN_IF_ERROR(write_back(it->get()));  // the file holds every completed WRITE
    }
    // Keep the fd and the image open (a worker may hold a span snapshot); clear its ranges.
    (*it)->ranges.clear();
    auto spans = std::make_shared<std::vector<Span>>();
    for (auto& b : backings_)
        for (auto& r : b->ranges)
            spans->push_back({r.ns_offset, r.length, r.file_offset, b->fd, b->map, b->map_len, b.get()});
    std::sort(spans->begin(), spans->end(), [](const Span& a, const Span& b) { return a.ns < b.ns; });
    std::atomic_store(&spans_, std::shared_ptr<const std::vector<Span>>(spans));
    return Status::Ok();
}

void EmulatedNvmeController::inject(InjectKind kind, std::uint32_t count, std::uint32_t delay_us,
                                    std::uint32_t status) {
    inject_delay_us_.store(delay_us);
    inject_status_.store(status);
    inject_count_.store(count);
    inject_kind_.store(static_cast<std::uint32_t>(kind));
}

int EmulatedNvmeController::window_kind(std::uint64_t addr, std::uint64_t bytes) const {
    auto w = std::atomic_load(&windows_);
    for (const auto& x : *w)
        if (addr >= x.base && addr + bytes <= x.base + x.bytes) return x.device ? 1 : 0;
    return -1;
}

bool EmulatedNvmeController::collect_iov(std::uint64_t prp1, std::uint64_t prp2, std::uint64_t bytes,
                                         std::vector<Seg>& iov) const {
    iov.clear();
    auto push = [&](std::uint64_t addr, std::uint64_t len) -> bool {
        const int kind = window_kind(addr, len);
        if (kind < 0) return false;
        char* p = reinterpret_cast<char*>(addr);
        if (!iov.empty() && iov.back().p + iov.back().n == p && iov.back().device == (kind == 1))
            iov.back().n += len;
        else
            iov.push_back({p, len, kind == 1});
        return true;
    };
    const std::uint64_t P = kMemoryPageBytes;
    std::uint64_t first = std::min<std::uint64_t>(bytes, P - (prp1 & (P - 1)));
    if (!push(prp1, first)) return false;
    std::uint64_t remaining = bytes - first;
    if (remaining == 0) return true;
    if (remaining <= P) {
        if (prp2 & (P - 1)) return false;  // second page must be page aligned
        return push(prp2, remaining);
    }
    // PRP list: 8-byte entries in host memory; the last slot of a list page chains to the next page.
    if (prp2 & 7) return false;
    std::uint64_t list = prp2;
    std::uint64_t slots = (P - (list & (P - 1))) / 8;
    while (remaining > 0) {
        if (window_kind(list, 8) != 0) return false;
        std::uint64_t entry = *reinterpret_cast<volatile std::uint64_t*>(list);
        if (slots == 1 && remaining > P) {
            if (entry & (P - 1)) return false;
            list = entry;
            slots = P / 8;
            continue;
        }
        if (entry & (P - 1)) return false;
        std::uint64_t len = std::min<std::uint64_t>(remaining, P);
        if (!push(entry, len)) return false;
        remaining -= len;
        list += 8;
        --slots;
    }
    return true;
}

// Memory media: the image bytes at file offset `foff` (loading their chunk
// from the file on first touch); *avail = bytes usable from there within the
// chunk. Null when the offset is past the file or the image budget is spent.
char* EmulatedNvmeController::image_at(Backing* b, std::uint64_t foff, std::uint64_t* avail) {
    const std::uint64_t cb = cfg_.image_chunk_bytes;
    const std::size_t ci = static_cast<std::size_t>(foff / cb);
    if (!b || ci >= b->n_chunks) return nullptr;
    char* base = b->chunks[ci].load(std::memory_order_acquire);
    if (!base) {
        std::lock_guard<std::mutex> g(b->load_mu);
        base = b->chunks[ci].load(std::memory_order_relaxed);
        if (!base) {
            // carve the next chunk out of the arena allocated at creation
            if (!image_arena_) return nullptr;
            const std::uint64_t at = image_bytes_.fetch_add(cb);
            if (at + cb > image_arena_bytes_) {
                image_bytes_.fetch_sub(cb);
                return nullptr;  // arena spent: the caller serves this range from the file
            }
            void* p = image_arena_ + at;
            char* c = static_cast<char*>(p);
            const std::uint64_t t0 = now_ns();
            const std::uint64_t start = static_cast<std::uint64_t>(ci) * cb;
            std::uint64_t done = 0;
            while (done < cb) {
                ssize_t r = ::pread(b->fd, c + done, cb - done, start + done);
                if (r < 0 && errno == EINTR) continue;
                if (r <= 0) break;
                done += static_cast<std::uint64_t>(r);
            }
            if (done < cb) std::memset(c + done, 0, cb - done);  // past EOF: zeros
            st_load_ns_.fetch_add(now_ns() - t0, std::memory_order_relaxed);
            b->chunks[ci].store(c, std::memory_order_release);
            base = c;
        }
    }
    *avail = cb - foff % cb;
    return base + foff % cb;
}

// Drive bandwidth cap: reserve the transfer time of `bytes` on the drive's
// timeline and wait until the reservation starts.
void EmulatedNvmeController::pace(std::uint64_t bytes) {
    if (cfg_.max_gbps <= 0) return;
    const std::uint64_t cost = static_cast<std::uint64_t>(static_cast<double>(bytes) / cfg_.max_gbps);  // ns
    std::uint64_t now = now_ns();
    std::uint64_t prev = pace_next_ns_.load();
    std::uint64_t start;
    do {
        start = std::max(prev, now);
    } while (!pace_next_ns_.compare_exchange_weak(prev, start + cost));
    while (now_ns() < start) {
        if (start - now_ns() > 50000)
            std::this_thread::sleep_for(std::chrono::microseconds(20));
        else
            _mm_pause();
    }
}

// Moves `n` bytes between file offset `foff` of a backing file and `buf`
// (host memory, or GPU memory when `device`). Returns 0 or an NVMe status.
std::uint32_t EmulatedNvmeController::move_span(bool read, Backing* b, int fd, const char* map,
                                                std::uint64_t map_len, std::uint64_t foff, char* buf,
                                                std::uint64_t n, bool device, WorkerCtx& w) {
    const std::uint32_t xfer_error = make_status(0, kScDataTransferError);
    const std::uint32_t media_error = make_status(kSctMedia, kScUnrecoveredRead);
    if (device && !w.cuda) return xfer_error;
    auto file_io = [&](char* p, std::uint64_t len, std::uint64_t off) -> bool {
        struct Timer {
            std::atomic<std::uint64_t>& acc;
            std::uint64_t t0 = now_ns();
            ~Timer() { acc.fetch_add(now_ns() - t0, std::memory_order_relaxed); }
        } timer{st_file_ns_};
        std::uint64_t done = 0;
        if (read && map && off + len <= map_len) {
            std::memcpy(p, map + off, len);
            return true;
        }
        while (done < len) {
            ssize_t r = read ? ::pread(fd, p + done, len - done, off + done)
                             : ::pwrite(fd, p + done, len - done, off + done);
            if (r < 0 && errno == EINTR) continue;
            if (r <= 0) {
                if (read && r == 0) {  // past EOF of a backing file: zero fill
                    std::memset(p + done, 0, len - done);
                    return true;
                }
                return false;
            }
            done += static_cast<std::uint64_t>(r);
        }
        return true;
    };
    auto sync_stream = [&]() -> bool {
        if (!w.stream_dirty) return true;
        w.stream_dirty = false;
        const std::uint64_t t0 = now_ns();
        const cudaError_t e = cudaStreamSynchronize(w.stream);
        st_sync_ns_.fetch_add(now_ns() - t0, std::memory_order_relaxed);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        return true;
    };
    while (n > 0) {
        std::uint64_t avail = 0;
        char* img = cfg_.media == EmulatedControllerConfig::Media::MEMORY ? image_at(b, foff, &avail) : nullptr;
        if (img) {
            const std::uint64_t k = std::min(n, avail);
            if (read) {
                if (device) {
                    if (cudaMemcpyAsync(buf, img, k, cudaMemcpyHostToDevice, w.stream) != cudaSuccess) {
                        cudaGetLastError();
                        return xfer_error;
                    }
                    st_dma_copies_.fetch_add(1, std::memory_order_relaxed);
                    w.stream_dirty = true;
                } else {
                    std::memcpy(buf, img, k);
                }
            } else {
                if (device) {
                    if (cudaMemcpyAsync(img, buf, k, cudaMemcpyDeviceToHost, w.stream) != cudaSuccess) {
                        cudaGetLastError();
                        return xfer_error;
                    }
                    st_dma_copies_.fetch_add(1, std::memory_order_relaxed);
                    w.stream_dirty = true;
                    // write cache: the CQE follows the copy on the stream; else the file first
                    if (!cfg_.write_back && !sync_stream()) return xfer_error;
                } else {
                    std::memcpy(img, buf, k);
                }
                if (cfg_.write_back)
                    mark_dirty(b, foff, k);
                else if (!file_io(img, k, foff))
                    return media_error;  // write-through: the file stays durable
            }
            buf += k;
            foff += k;
            n -= k;
            continue;
        }
        if (!device) {
            if (!file_io(buf, n, foff)) return media_error;
            return 0;
        }
        // File media and GPU memory: through the worker's page-locked bounce buffer.
        if (!w.bounce) return xfer_error;
        const std::uint64_t k = std::min(n, w.bounce_bytes);
        if (!sync_stream()) return xfer_error;  // the bounce may still feed an earlier copy
        if (read) {
            if (!file_io(w.bounce, k, foff)) return media_error;
            if (cudaMemcpyAsync(buf, w.bounce, k, cudaMemcpyHostToDevice, w.stream) != cudaSuccess) {
                cudaGetLastError();
                return xfer_error;
            }
            w.stream_dirty = true;
        } else {
            if (cudaMemcpyAsync(w.bounce, buf, k, cudaMemcpyDeviceToHost, w.stream) != cudaSuccess) {
                cudaGetLastError();
                return xfer_error;
            }
            w.stream_dirty = true;
            if (!sync_stream()) return xfer_error;
            if (!file_io(w.bounce, k, foff)) return media_error;
        }
        st_dma_copies_.fetch_add(1, std::memory_order_relaxed);
        buf += k;
        foff += k;
        n -= k;
    }
    return 0;
}

std::uint32_t EmulatedNvmeController::execute(const Sqe& sqe, WorkerCtx& w, bool* drop_cqe, bool* on_stream) {
    *drop_cqe = false;
    *on_stream = false;
    st_commands_.fetch_add(1, std::memory_order_relaxed);
    const std::uint8_t op = sqe_opcode(sqe);

    // Injected faults consume one unit each.
    std::uint32_t ik = inject_kind_.load(std::memory_order_relaxed);
    if (ik != 0) {
        std::uint32_t c = inject_count_.load();
        while (c > 0 && !inject_count_.compare_exchange_weak(c, c - 1)) {
        }
        if (c > 0) {
            st_injected_.fetch_add(1);
            if (c == 1) inject_kind_.store(0);
            switch (static_cast<InjectKind>(ik)) {
                case InjectKind::MEDIA_ERROR: {
                    st_errors_.fetch_add(1);
                    const std::uint32_t raw = inject_status_.load();
                    return raw ? raw : make_status(kSctMedia, kScUnrecoveredRead);
                }
                case InjectKind::DROP_COMPLETION:
                    *drop_cqe = true;
                    return 0;
                case InjectKind::DELAY:
                    std::this_thread::sleep_for(std::chrono::microseconds(inject_delay_us_.load()));
                    break;
                default:
                    break;
            }
        }
    }

    if (op == kOpFlush) {
        // this worker's own copies first (flush() waits for every worker's stream)
        if (w.stream_dirty && cudaStreamSynchronize(w.stream) != cudaSuccess) cudaGetLastError();
        w.stream_dirty = false;
        return flush().ok() ? 0u : make_status(0, kScDataTransferError);
    }
    if (op != kOpRead && op != kOpWrite) {
        st_errors_.fetch_add(1);
        return make_status(0, kScInvalidOpcode);
    }
    if (sqe.nsid != info_.nsid) {
        st_errors_.fetch_add(1);
        return make_status(0, kScInvalidNamespace);
    }
    const std::uint64_t lba = info_.lba_bytes;
    const std::uint64_t off = sqe_slba(sqe) * lba;
    const std::uint64_t bytes = std::uint64_t(sqe_nlb(sqe)) * lba;
    if (bytes > info_.mdts_bytes) {
        st_errors_.fetch_add(1);
        return make_status(0, kScInvalidField);
    }
    if (off + bytes > info_.namespace_bytes) {
        st_errors_.fetch_add(1);
        return make_status(0, kScLbaOutOfRange);
    }
    thread_local std::vector<Seg> iov;
    if (!collect_iov(sqe.prp1, sqe.prp2, bytes, iov)) {
        st_errors_.fetch_add(1);
        return make_status(0, kScDataTransferError);
    }
    const bool read = op == kOpRead;
    if (cfg_.skip_data) {
        (read ? st_read_ : st_write_).fetch_add(bytes, std::memory_order_relaxed);
        return 0;
    }
    pace(bytes);
    const std::uint64_t t_cmd = now_ns();
    struct MaxTimer {
        std::atomic<std::uint64_t>& mx;
        std::uint64_t t0;
        ~MaxTimer() {
            const std::uint64_t d = now_ns() - t0;
            std::uint64_t cur = mx.load(std::memory_order_relaxed);
            while (d > cur && !mx.compare_exchange_weak(cur, d)) {
            }
        }
    } max_timer{st_max_cmd_ns_, t_cmd};
    auto spans = std::atomic_load(&spans_);
    // Walk namespace spans and iov segments together.
    std::uint64_t pos = off, end = off + bytes;
    std::size_t seg = 0;
    std::uint64_t seg_off = 0;
    auto it = std::upper_bound(spans->begin(), spans->end(), pos,
                               [](std::uint64_t v, const Span& s) { return v < s.ns; });
    if (it != spans->begin()) --it;
    while (pos < end) {
        if (it == spans->end() || pos < it->ns || pos >= it->ns + it->len) {
            st_errors_.fetch_add(1);
            return make_status(0, kScLbaOutOfRange);  // unbacked namespace range
        }
        std::uint64_t chunk = std::min(it->ns + it->len - pos, end - pos);
        std::uint64_t foff = it->foff + (pos - it->ns);
        while (chunk > 0) {
            const Seg& s = iov[seg];
            const std::uint64_t n = std::min(chunk, s.n - seg_off);
            const std::uint32_t st =
                move_span(read, it->b, it->fd, it->map, it->map_len, foff, s.p + seg_off, n, s.device, w);
            if (st != 0) {
                st_errors_.fetch_add(1);
                return st;
            }
            // the CQE follows the copy on the stream (a cached WRITE's slot is reused only after it)
            if (s.device && (read || cfg_.write_back)) *on_stream = true;
            chunk -= n;
            pos += n;
            foff += n;
            seg_off += n;
            if (seg_off == s.n) {
                ++seg;
                seg_off = 0;
            }
        }
        ++it;
    }
    (read ? st_read_ : st_write_).fetch_add(bytes, std::memory_order_relaxed);
    return 0;
}

bool EmulatedNvmeController::service_queue(std::uint32_t q, WorkerCtx& w) {
    QueueState& qs = *qstate_[q];
    auto drain_stream = [&] {
        if (w.stream_dirty) {
            w.stream_dirty = false;
            if (cudaStreamSynchronize(w.stream) != cudaSuccess) cudaGetLastError();
        }
    };
    if (const std::uint32_t req = qs.reset_request.load(std::memory_order_acquire)) {
        drain_stream();  // no CQE write of this queue may land after the reset
        qs.sq_head = 0;
        qs.cq_tail = 0;
        qs.phase = 1;
        if (req == 2) {  // a driver created or deleted the queue pair
            qs.view = qs.pending_view;
            qs.cq_device = qs.pending_cq_device;
            qs.enabled = qs.pending_enabled;
        }
        if (qs.enabled) {
            const QueuePairView& v = qs.view;
            std::memset(const_cast<Cqe*>(v.cq), 0, sizeof(Cqe) * v.depth);
            store_release(v.sq_doorbell, 0);
            store_release(v.cq_doorbell, 0);
        }
        qs.fatal.store(0);
        qs.reset_request.store(0, std::memory_order_release);
        return true;
    }
    if (!qs.enabled || qs.fatal.load(std::memory_order_relaxed)) return false;
    const QueuePairView v = qs.view;
    std::uint32_t tail = load_acquire(v.sq_doorbell);
    if (tail >= v.depth) {
        qs.fatal.store(1);  // protocol violation: invalid doorbell value
        return false;
    }
    bool any = false;
    int budget = 64;
    while (qs.sq_head != tail && budget-- > 0) {
        Sqe sqe;
        std::memcpy(&sqe, const_cast<const Sqe*>(&v.sq[qs.sq_head]), sizeof(Sqe));
        qs.sq_head = (qs.sq_head + 1) % v.depth;
        bool drop = false, on_stream = false;
        const std::uint32_t status = execute(sqe, w, &drop, &on_stream);
        any = true;
        if (drop) {
            drain_stream();  // a dropped completion must not leave its data landing later
            continue;
        }
        // CQ full: the next tail would meet the consumer's head.
        std::uint32_t next = (qs.cq_tail + 1) % v.depth;
        while (next == load_acquire(v.cq_doorbell)) {
            if (stop_.load(std::memory_order_relaxed) || qs.reset_request.load()) return true;
            _mm_pause();
        }
        Cqe* slot = const_cast<Cqe*>(&v.cq[qs.cq_tail]);
        slot->dw0 = 0;
        slot->dw1 = 0;
        slot->dw2 = (qs.sq_head & 0xFFFFu) | ((v.qid & 0xFFFFu) << 16);
        const std::uint32_t dw3 = make_cqe_dw3(sqe_cid(sqe), qs.phase, status);
        bool posted = false;
        if (on_stream && status == 0 && qs.cq_device) {
            // After the copies on the same stream: the completion follows the data.
            const std::uint64_t dev_dw3 =
                reinterpret_cast<std::uint64_t>(qs.cq_device) + std::uint64_t(qs.cq_tail) * sizeof(Cqe) + 12;
            posted = write_value32()(reinterpret_cast<CUstream>(w.stream), static_cast<CUdeviceptr>(dev_dw3), dw3,
                                     0) == CUDA_SUCCESS;
        }
        if (!posted) {
            // Host-posted completion: no earlier transfer of this worker may still be in flight
            // (a failed command's slot is reused at once).
            drain_stream();
            store_release(&slot->dw3, dw3);
        }
        qs.cq_tail = next;
        if (qs.cq_tail == 0) qs.phase ^= 1u;
        if (qs.sq_head == tail) tail = load_acquire(v.sq_doorbell);
    }
    return any;
}

void EmulatedNvmeController::worker_main(std::uint32_t worker) {
    const std::uint32_t nw = static_cast<std::uint32_t>(
        std::max<std::size_t>(1, std::min<std::size_t>(cfg_.worker_threads, cfg_.num_io_queues)));
    WorkerCtx w;
    w.bounce = worker < bounces_.size() ? bounces_[worker] : nullptr;
    w.bounce_bytes = cfg_.mdts_bytes;
    if (cuda_device_ >= 0 && cudaSetDevice(cuda_device_) == cudaSuccess) {
        bool green = false;
        w.stream = create_drive_stream(cuda_device_, &green);
        w.cuda = w.stream != nullptr;
        if (green) st_green_streams_.fetch_add(1, std::memory_order_relaxed);
        if (w.stream) {
            std::lock_guard<std::mutex> g(streams_mu_);
            worker_streams_.push_back(w.stream);
        }
    } else {
        cudaGetLastError();
    }
    std::uint32_t idle = 0;
    while (!stop_.load(std::memory_order_relaxed)) {
        bool any = false;
        for (std::uint32_t q = worker; q < cfg_.num_io_queues; q += nw) any |= service_queue(q, w);
        if (any) {
            idle = 0;
            continue;
        }
        if (++idle < cfg_.idle_spin_iters) {
            _mm_pause();
        } else {
            std::this_thread::sleep_for(std::chrono::microseconds(cfg_.idle_sleep_us));
        }
    }
    if (w.stream) {
        cudaStreamSynchronize(w.stream);
        {
            std::lock_guard<std::mutex> g(streams_mu_);
            worker_streams_.erase(std::remove(worker_streams_.begin(), worker_streams_.end(), w.stream),
                                  worker_streams_.end());
        }
        cudaStreamDestroy(w.stream);
    }
    cudaGetLastError();
}

}  // namespace nvme
}  // namespace tutti
