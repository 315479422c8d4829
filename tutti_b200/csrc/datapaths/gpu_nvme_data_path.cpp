#include "gpu_nvme_data_path.h"

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include "../runtime/device_guard.h"

namespace tutti {

namespace {
constexpr std::uint32_t kApiVersion = 1;

std::size_t align_up(std::size_t v, std::size_t a) { return (v + a - 1) / a * a; }

Status cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return Status::Ok();
    cudaGetLastError();
    return {StatusCode::DEVICE_ERROR, std::string(what) + ": " + cudaGetErrorString(e)};
}

// Reads of the same target range into several memories (same piece tiling)
// become one command with replica groups: the bytes cross PCIe once and the
// kernel stores them to every destination (e.g. each TP rank's pool).
void merge_replicas(std::vector<io::IoCommand>& cmds, std::vector<io::IoPiece>& pieces,
                    std::vector<std::uint32_t>& cmd_first_piece, std::vector<std::uint32_t>& piece_req) {
    struct Key {
        std::uint64_t logical;
        std::uint32_t target, bytes, n;
        bool operator==(const Key& o) const {
            return logical == o.logical && target == o.target && bytes == o.bytes && n == o.n;
        }
    };
    struct KeyHash {
        std::size_t operator()(const Key& k) const {
            return std::hash<std::uint64_t>()(k.logical * 0x9E3779B97F4A7C15ull ^ (std::uint64_t(k.target) << 32 | k.bytes) ^ k.n);
        }
    };
    std::unordered_map<Key, std::uint32_t, KeyHash> group_of;
    std::vector<std::vector<std::uint32_t>> groups;
    bool merged = false;
    auto same_tiling = [&](const io::IoCommand& a, const io::IoCommand& b) {
        for (std::uint32_t i = 0; i < a.n_pieces; ++i) {
            const auto& x = pieces[a.first_piece + i];
            const auto& y = pieces[b.first_piece + i];
            if (x.off != y.off || x.bytes != y.bytes) return false;
        }
        return true;
    };
    groups.reserve(cmds.size());
    for (std::uint32_t i = 0; i < cmds.size(); ++i) {
        const auto& c = cmds[i];
        if (c.opcode == nvme::kOpRead) {
            const Key k{c.logical, c.target | (std::uint32_t(c.transform) << 31), c.bytes, c.n_pieces};
            auto it = group_of.find(k);
            if (it != group_of.end() && same_tiling(cmds[groups[it->second][0]], c)) {
                groups[it->second].push_back(i);
                merged = true;
                continue;
            }
            group_of[k] = static_cast<std::uint32_t>(groups.size());
        }
        groups.push_back({i});
    }
    if (!merged) return;
    std::vector<io::IoCommand> nc;
    std::vector<io::IoPiece> np;
    std::vector<std::uint32_t> nfirst, nreq;
    nc.reserve(groups.size());
    np.reserve(pieces.size());
    nreq.reserve(piece_req.size());
    for (const auto& g : groups) {
        io::IoCommand c = cmds[g[0]];
        c.first_piece = static_cast<std::uint32_t>(np.size());
        c.replicas = g.size() > 1 ? static_cast<std::uint32_t>(g.size()) : 0u;
        nfirst.push_back(c.first_piece);
        for (auto idx : g) {
            const auto& o = cmds[idx];
            for (std::uint32_t p = 0; p < o.n_pieces; ++p) {
                np.push_back(pieces[o.first_piece + p]);
                nreq.push_back(piece_req[o.first_piece + p]);
            }
        }
        nc.push_back(c);
    }
    cmds.swap(nc);
    pieces.swap(np);
    cmd_first_piece.swap(nfirst);
    piece_req.swap(nreq);
}

// NVTX ranges around each submit, opt-in with TUTTI_NVTX=1 (read once).
bool nvtx_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("TUTTI_NVTX");
        return e && *e && std::strcmp(e, "0") != 0;
    }();
    return on;
}

double percentile(std::vector<double>& v, double q) {
    if (v.empty()) return 0.0;
    std::size_t k = static_cast<std::size_t>(q * (v.size() - 1));
    std::nth_element(v.begin(), v.begin() + k, v.end());
    return v[k];
}
}  // namespace

GpuNvmeDataPath::GpuNvmeDataPath(GpuNvmeConfig config, std::vector<GpuNvmeDevice> devices)
    : cfg_(config), devs_(std::move(devices)) {
    caps_.name = "nvme-gpu";
    caps_.source_api_version = kApiVersion;
    caps_.supports_device_execution = true;
    caps_.supports_host_execution = false;
    caps_.supports_device_memory = true;
    caps_.supports_host_memory = true;  // page-locked, device-mapped host memory
    caps_.supports_direct = false;
    caps_.supports_staged = true;
    caps_.supports_read = true;
    caps_.supports_write = true;
    caps_.supports_fp8_block_transform = true;  // fused into the movers
    std::uint32_t lba = 512;
    for (auto& d : devs_)
        if (d.controller) lba = std::max(lba, d.controller->info().lba_bytes);
    // Requests need only 16-byte alignment: sub-sector pieces (e.g. 8,448-byte
    // index-cache pages) are packed into commands, and it is the commands that
    // must start and end on LBA boundaries (checked per submit).
    lba_ = lba;
    caps_.target_alignment_bytes = 16;
    caps_.memory_alignment_bytes = 16;
    caps_.length_alignment_bytes = 16;
    caps_.max_single_io_bytes = 0;
    caps_.max_batch_requests = 1u << 26;
    caps_.supports_scatter_gather = true;
    caps_.max_scatter_gather_entries = cfg_.max_pieces_per_cmd;
    caps_.registration_scope = RegistrationScope::GLOBAL;
    caps_.progress_model = ProgressModel::HOST_POLL;
    caps_.device_completion_fence_on_caller_stream = true;
    caps_.device_execution_autonomous = true;
    caps_.supports_multi_stream = true;
    caps_.max_concurrent_streams = 0;
    caps_.bound_accel_id = cfg_.accel_id;
    caps_.supports_multi_gpu = false;
    caps_.optional_target_features = {"fused-paged-scatter", "striped", "raid0-members"};
}

GpuNvmeDataPath::~GpuNvmeDataPath() { shutdown(0); }

Status GpuNvmeDataPath::initialize(const DataPathConfig&, ResourceProvider*) {
    std::lock_guard<std::mutex> g(mu_);
    if (initialized_) return {StatusCode::INVALID_ARGUMENT, "already initialized"};
    if (devs_.empty() || devs_.size() > io::kMaxDevices)
        return {StatusCode::INVALID_ARGUMENT, "device table must hold 1..8 controllers"};
    if (cfg_.slots_per_lease == 0 || cfg_.slots_per_lease > io::kMaxSlots)
        return {StatusCode::INVALID_ARGUMENT, "slots_per_lease must be in [1, 64]"};
    if (cfg_.slot_bytes < 4096 || cfg_.slot_bytes > (2u << 20) || cfg_.slot_bytes % 4096)
        return {StatusCode::INVALID_ARGUMENT, "slot_bytes must be a 4 KiB multiple <= 2 MiB"};
    if (cfg_.leases == 0) return {StatusCode::INVALID_ARGUMENT, "leases must be > 0"};
    for (auto& d : devs_) {
        if (!d.controller) return {StatusCode::INVALID_ARGUMENT, "null controller"};
        const auto& inf = d.controller->info();
        if (inf.num_io_queues < cfg_.leases)
            return {StatusCode::RESOURCE_EXHAUSTED,
                    inf.name + " has " + std::to_string(inf.num_io_queues) + " queues < leases"};
        if (cfg_.slots_per_lease * io::kMaxSub >= inf.queue_depth)
            return {StatusCode::INVALID_ARGUMENT, "slots_per_lease x 8 must be < queue depth"};
    }
    // A command must split into <= kMaxSub NVMe commands: half the budget for
    // MDTS splits, half for extent boundaries.
    cmd_bytes_ = cfg_.slot_bytes;
    for (auto& d : devs_)
        cmd_bytes_ = std::min<std::uint32_t>(cmd_bytes_, d.controller->info().mdts_bytes * (io::kMaxSub / 2));
    DeviceGuard guard(cfg_.accel_id);
    TUTTI_RETURN_IF_ERROR(guard.status());
    TUTTI_RETURN_IF_ERROR(init_device_side());
    initialized_ = true;
    return Status::Ok();
}

Status GpuNvmeDataPath::init_device_side() {
    const std::uint64_t nslots = std::uint64_t(cfg_.leases) * cfg_.slots_per_lease;
    bool all_dma = true;
    for (auto& d : devs_) all_dma = all_dma && d.controller->info().device_dma;
    if (cfg_.staging == GpuNvmeConfig::Staging::DEVICE && !all_dma)
        return {StatusCode::UNSUPPORTED, "device staging needs controllers that DMA into GPU memory"};
    staging_on_device_ = cfg_.staging == GpuNvmeConfig::Staging::DEVICE ||
                         (cfg_.staging == GpuNvmeConfig::Staging::AUTO && all_dma);
    if (staging_on_device_) {
        // The drives' copies are CUDA work in this process, so two process-wide
        // settings decide whether they can stall behind a running io kernel.
        // Eager loading covers the kernels of modules loaded at startup; a
        // library that loads kernels on first use (cuBLAS on a new GEMM shape)
        // takes the same lock, so an application runs its shapes once before
        // restores start (measured: the first 4096 x 4096 GEMM of a prefill
        // held the host for 10 s while the drives' copies waited).
        const char* loading = std::getenv("CUDA_MODULE_LOADING");
        const char* conns = std::getenv("CUDA_DEVICE_MAX_CONNECTIONS");
        if (!loading || std::strcmp(loading, "EAGER") != 0)
            std::fprintf(stderr,
                         "[tutti] nvme-gpu: drives DMA into HBM staging but CUDA_MODULE_LOADING is not EAGER: a kernel "
                         "loaded lazily while a restore runs stalls the drives until the io deadline\n");
        if (!conns || std::atoi(conns) < 16)
            std::fprintf(stderr,
                         "[tutti] nvme-gpu: drives DMA into HBM staging with CUDA_DEVICE_MAX_CONNECTIONS < 16: a copy "
                         "that waits behind an io kernel can share a hardware queue with a drive's copies\n");
    }
    void* arena = nullptr;
    std::uint64_t arena_bytes = nslots * cfg_.slot_bytes;
    if (staging_on_device_) {
        TUTTI_RETURN_IF_ERROR(cuda_status(cudaMalloc(&staging_hbm_, arena_bytes), "cudaMalloc staging"));
        arena = staging_hbm_;
    } else {
        auto st = host_mapped_alloc(arena_bytes, cfg_.staging_write_combined);
        if (!st.ok()) return st.status();
        staging_ = st.value();
        if (!staging_.device)
            return {StatusCode::UNSUPPORTED, "nvme-gpu needs a CUDA device (device-mapped host memory)"};
        arena = staging_.host;
        arena_bytes = staging_.bytes;
    }
    auto pr = host_mapped_alloc(nslots * nvme::kMemoryPageBytes);
    if (!pr.ok()) return pr.status();
    prp_ = pr.value();
    if (!prp_.device) return {StatusCode::UNSUPPORTED, "nvme-gpu needs a CUDA device (device-mapped host memory)"};
    // Map both regions on every controller. The prebuilt PRP lists are shared by
    // all drives, so every controller must report the same bus address for
    // every page (an identity or pass-through IOMMU does).
    const std::uint64_t pages_per_slot = cfg_.slot_bytes / nvme::kMemoryPageBytes;
    std::vector<std::uint64_t> page_bus(nslots * pages_per_slot), list_bus(nslots);
    char* const arena_va = static_cast<char*>(arena);
    char* const prp_va = static_cast<char*>(prp_.host);
    for (std::size_t d = 0; d < devs_.size(); ++d) {
        auto a = devs_[d].controller->map_dma(arena, arena_bytes);
        if (!a.ok()) return a.status();
        staging_maps_.push_back(std::move(a).value());
        auto b = devs_[d].controller->map_dma(prp_.host, prp_.bytes);
        if (!b.ok()) return b.status();
        prp_maps_.push_back(std::move(b).value());
        const nvme::DmaMapping& sm = staging_maps_.back();
        const nvme::DmaMapping& pm = prp_maps_.back();
        if (!sm.covers(arena, nslots * cfg_.slot_bytes) || !pm.covers(prp_.host, nslots * nvme::kMemoryPageBytes))
            return {StatusCode::INTERNAL, devs_[d].identity + ": DMA mapping does not cover the buffer"};
        for (std::uint64_t k = 0; k < page_bus.size(); ++k) {
            const std::uint64_t bus = sm.bus_at(arena_va + k * nvme::kMemoryPageBytes);
            if (bus == 0 || (bus & (nvme::kMemoryPageBytes - 1)) != 0)
                return {StatusCode::UNSUPPORTED, devs_[d].identity + ": staging page without a 4 KiB-aligned bus address"};
            if (d > 0 && bus != page_bus[k])
                return {StatusCode::UNSUPPORTED, "controllers disagree on the bus addresses of the staging arena"};
            page_bus[k] = bus;
        }
        for (std::uint64_t i = 0; i < nslots; ++i) {
            const std::uint64_t bus = pm.bus_at(prp_va + i * nvme::kMemoryPageBytes);
            if (bus == 0 || (d > 0 && bus != list_bus[i]))
                return {StatusCode::UNSUPPORTED, "controllers disagree on the bus addresses of the PRP lists"};
            list_bus[i] = bus;
        }
    }
    // Prebuilt PRP lists: entry j of slot i's page is the bus address of the
    // slot's page j (a command starting at page j0 points PRP2 at entry j0 + 1).
    auto* lists = static_cast<std::uint64_t*>(prp_.host);
    for (std::uint64_t i = 0; i < nslots; ++i)
        for (std::uint64_t j = 0; j < pages_per_slot; ++j) lists[i * 512 + j] = page_bus[i * pages_per_slot + j];
    if (cfg_.direct_reads) {
        // One PRP-list page per slot for direct commands (the io kernel writes it).
        auto dl = host_mapped_alloc(nslots * nvme::kMemoryPageBytes);
        if (!dl.ok()) return dl.status();
        direct_lists_ = dl.value();
        if (!direct_lists_.device) return {StatusCode::UNSUPPORTED, "direct reads need device-mapped host memory"};
        std::vector<std::uint64_t> dbus(nslots);
        for (std::size_t d = 0; d < devs_.size(); ++d) {
            auto m = devs_[d].controller->map_dma(direct_lists_.host, direct_lists_.bytes);
            if (!m.ok()) return m.status();
            direct_list_maps_.push_back(std::move(m).value());
            for (std::uint64_t i = 0; i < nslots; ++i) {
                const std::uint64_t bus =
                    direct_list_maps_.back().bus_at(static_cast<char*>(direct_lists_.host) + i * nvme::kMemoryPageBytes);
                if (bus == 0 || (d > 0 && bus != dbus[i]))
                    return {StatusCode::UNSUPPORTED, "controllers disagree on the bus addresses of the direct PRP lists"};
                dbus[i] = bus;
            }
        }
        TUTTI_RETURN_IF_ERROR(cuda_status(cudaMalloc(&d_direct_list_bus_, nslots * 8), "cudaMalloc direct lists"));
        TUTTI_RETURN_IF_ERROR(cuda_status(
            cudaMemcpy(d_direct_list_bus_, dbus.data(), nslots * 8, cudaMemcpyHostToDevice), "upload direct lists"));
    }
    TUTTI_RETURN_IF_ERROR(cuda_status(cudaMalloc(&d_page_bus_, page_bus.size() * 8), "cudaMalloc page table"));
    TUTTI_RETURN_IF_ERROR(cuda_status(cudaMalloc(&d_list_bus_, list_bus.size() * 8), "cudaMalloc list table"));
    TUTTI_RETURN_IF_ERROR(cuda_status(
        cudaMemcpy(d_page_bus_, page_bus.data(), page_bus.size() * 8, cudaMemcpyHostToDevice), "upload page table"));
    TUTTI_RETURN_IF_ERROR(cuda_status(
        cudaMemcpy(d_list_bus_, list_bus.data(), list_bus.size() * 8, cudaMemcpyHostToDevice), "upload list table"));

    std::vector<io::DevDevice> rows(devs_.size());
    for (std::size_t d = 0; d < devs_.size(); ++d) {
        auto& ctl = *devs_[d].controller;
        std::vector<nvme::QueuePairView> views(cfg_.leases);
        for (std::uint32_t l = 0; l < cfg_.leases; ++l) views[l] = ctl.device_queue(l);
        nvme::QueuePairView* dv = nullptr;
        TUTTI_RETURN_IF_ERROR(cuda_status(cudaMalloc(&dv, views.size() * sizeof(views[0])), "cudaMalloc queues"));
        TUTTI_RETURN_IF_ERROR(cuda_status(
            cudaMemcpy(dv, views.data(), views.size() * sizeof(views[0]), cudaMemcpyHostToDevice), "upload queues"));
        d_queue_views_.push_back(dv);
        // Cursors live in mapped host memory: the kernel reads them when a CTA
        // starts and writes them when it ends; the host reads them without a copy.
        auto cm = host_mapped_alloc(std::size_t(cfg_.leases) * sizeof(io::QueueCursor));
        if (!cm.ok()) return cm.status();
        cursor_mem_.push_back(cm.value());
        auto* hc = cursor_mem_.back().host_as<io::QueueCursor>();
        for (std::uint32_t l = 0; l < cfg_.leases; ++l) hc[l] = io::QueueCursor{0, 0, 1, 0};
        d_cursors_.push_back(cursor_mem_.back().device_as<io::QueueCursor>());
        std::uint32_t lba = ctl.info().lba_bytes, shift = 0;
        while ((1u << shift) < lba) ++shift;
        rows[d] = io::DevDevice{dv, d_cursors_.back(), shift, ctl.info().mdts_bytes, cfg_.leases, ctl.info().nsid};
    }
    TUTTI_RETURN_IF_ERROR(cuda_status(cudaMalloc(&d_devices_, rows.size() * sizeof(rows[0])), "cudaMalloc devices"));
    TUTTI_RETURN_IF_ERROR(cuda_status(
        cudaMemcpy(d_devices_, rows.data(), rows.size() * sizeof(rows[0]), cudaMemcpyHostToDevice), "upload devices"));
    TUTTI_RETURN_IF_ERROR(cuda_status(cudaMalloc(&d_targets_, std::size_t(cfg_.max_targets) * sizeof(io::DevTarget)),
                                      "cudaMalloc targets"));
    TUTTI_RETURN_IF_ERROR(cuda_status(
        cudaMemset(d_targets_, 0, std::size_t(cfg_.max_targets) * sizeof(io::DevTarget)), "memset targets"));
    for (std::uint32_t l = cfg_.leases; l-- > 0;) free_leases_.push_back(l);
    retired_.assign(cfg_.leases, false);
    TUTTI_RETURN_IF_ERROR(
        cuda_status(cudaStreamCreateWithFlags(&upload_stream_, cudaStreamNonBlocking), "cudaStreamCreate upload"));
    for (std::uint32_t i = 0; i < cfg_.prealloc_arenas; ++i) {
        auto a = take_arena(cfg_.prealloc_arena_bytes);
        if (!a.ok()) return a.status();
        return_arena(std::move(a).value());
    }
    if (const char* v = std::getenv("TUTTI_VERBOSE"); v && *v && std::strcmp(v, "0") != 0)
        std::fprintf(stderr,
                     "[tutti] nvme-gpu accel %d: %zu controller(s), %u leases x %u slots x %u KiB %s staging, "
                     "commands up to %u KiB, LBA %u, timeout %.1f s\n",
                     cfg_.accel_id, devs_.size(), cfg_.leases, cfg_.slots_per_lease, cfg_.slot_bytes >> 10,
                     staging_on_device_ ? "HBM" : "host",
                     cmd_bytes_ >> 10, lba_, cfg_.timeout_ns / 1e9);
    return Status::Ok();
}

Status GpuNvmeDataPath::shutdown(std::uint64_t) {
    std::lock_guard<std::mutex> g(mu_);
    if (!initialized_) return Status::Ok();
    DeviceGuard guard(cfg_.accel_id);
    for (auto& kv : ops_)
        if (kv.second->drain_pending) launch_drain(*kv.second, kv.second->stream);
    for (auto& kv : ops_)
        if (kv.second->arena && kv.second->arena->event) cudaEventSynchronize(kv.second->arena->event);
    for (auto& kv : ops_)
        if (kv.second->arena) arena_pool_.push_back(std::move(kv.second->arena));
    ops_.clear();
    for (auto& a : arena_pool_) {
        if (a->event) cudaEventDestroy(a->event);
        if (a->submitted) cudaEventDestroy(a->submitted);
        if (a->uploaded) cudaEventDestroy(a->uploaded);
        if (a->host) cudaFreeHost(a->host);
        if (a->dev) cudaFree(a->dev);
    }
    arena_pool_.clear();
    if (upload_stream_) {
        cudaStreamSynchronize(upload_stream_);
        cudaStreamDestroy(upload_stream_);
        upload_stream_ = nullptr;
    }
    for (auto* p : d_queue_views_) cudaFree(p);
    for (auto& m : cursor_mem_) host_mapped_free(m);
    cursor_mem_.clear();
    for (auto* p : extent_chunks_) cudaFree(p);
    d_queue_views_.clear();
    d_cursors_.clear();
    extent_chunks_.clear();
    if (d_devices_) cudaFree(d_devices_);
    if (d_targets_) cudaFree(d_targets_);
    d_devices_ = nullptr;
    d_targets_ = nullptr;
    for (std::size_t d = 0; d < devs_.size(); ++d) {
        if (d < staging_maps_.size()) devs_[d].controller->unmap_dma(staging_maps_[d]);
        if (d < prp_maps_.size()) devs_[d].controller->unmap_dma(prp_maps_[d]);
    }
    staging_maps_.clear();
    prp_maps_.clear();
    if (d_page_bus_) cudaFree(d_page_bus_);
    if (d_list_bus_) cudaFree(d_list_bus_);
    d_page_bus_ = d_list_bus_ = nullptr;
    for (auto& kv : direct_regions_) {
        for (std::size_t d = 0; d < kv.second.maps.size() && d < devs_.size(); ++d)
            devs_[d].controller->unmap_dma(kv.second.maps[d]);
        if (kv.second.d_bus) cudaFree(kv.second.d_bus);
    }
    direct_regions_.clear();
    for (void* t : retired_device_tables_) cudaFree(t);
    retired_device_tables_.clear();
    if (d_regions_) cudaFree(d_regions_);
    d_regions_ = nullptr;
    n_regions_ = 0;
    for (std::size_t d = 0; d < direct_list_maps_.size() && d < devs_.size(); ++d)
        devs_[d].controller->unmap_dma(direct_list_maps_[d]);
    direct_list_maps_.clear();
    host_mapped_free(direct_lists_);
    if (d_direct_list_bus_) cudaFree(d_direct_list_bus_);
    d_direct_list_bus_ = nullptr;
    host_mapped_free(staging_);
    host_mapped_free(prp_);
    if (staging_hbm_) cudaFree(staging_hbm_);
    staging_hbm_ = nullptr;
    initialized_ = false;
    return Status::Ok();
}

Result<DataPathTarget> GpuNvmeDataPath::open(const ResolvedTarget& target) {
    std::lock_guard<std::mutex> g(mu_);
    std::vector<DeviceUpload> uploads;
    auto r = open_locked(target, uploads);
    if (!r.ok()) return r;
    Status s = flush_uploads(uploads);
    if (!s.ok()) return Result<DataPathTarget>::Failure(s);
    return r;
}

std::vector<Result<DataPathTarget>> GpuNvmeDataPath::open_many(const ResolvedTarget* const* targets, std::size_t count) {
    std::lock_guard<std::mutex> g(mu_);
    std::vector<Result<DataPathTarget>> out;
    out.reserve(count);
    std::vector<DeviceUpload> uploads;
    for (std::size_t i = 0; i < count; ++i) out.push_back(open_locked(*targets[i], uploads));
    Status s = flush_uploads(uploads);
    if (!s.ok())  // no target of the batch is usable without its device rows
        for (auto& r : out)
            if (r.ok()) r = Result<DataPathTarget>::Failure(s);
    return out;
}

Status GpuNvmeDataPath::flush_uploads(std::vector<DeviceUpload>& uploads) {
    // Caller holds mu_. One copy per run of nearby destinations in one allocation
    // (bump-allocated extent arrays, consecutive target rows); see upload_plan.h.
    if (uploads.empty()) return Status::Ok();
    DeviceGuard guard(cfg_.accel_id);
    const auto runs = coalesce_uploads(std::move(uploads), 255);
    for (const UploadRun& r : runs)
        TUTTI_RETURN_IF_ERROR(cuda_status(
            cudaMemcpyAsync(r.dst, r.bytes.data(), r.bytes.size(), cudaMemcpyHostToDevice, upload_stream_),
            "upload target rows"));
    TUTTI_RETURN_IF_ERROR(cuda_status(cudaStreamSynchronize(upload_stream_), "upload target rows"));
    uploads.clear();
    return Status::Ok();
}

Result<DataPathTarget> GpuNvmeDataPath::open_locked(const ResolvedTarget& target,
                                                     std::vector<DeviceUpload>& uploads) {
    // Caller holds mu_. Host-side work of an open; the device copies it owes are
    // appended to `uploads` (flush_uploads).
    using R = Result<DataPathTarget>;
    auto pv = target.view<FileExtentPayload>(kFileExtentPayloadType, kFileExtentPayloadVersion);
    if (!pv.ok()) return R::Failure(pv.status());
    const FileExtentPayload& p = *pv.value();
    if (!initialized_) return R::Failure({StatusCode::NOT_READY, "not initialized"});
    if (p.extents.empty() && p.file_size > 0) return R::Failure({StatusCode::INVALID_ARGUMENT, "no extents"});
    for (const auto& e : p.extents)
        if (e.device >= devs_.size())
            return R::Failure({StatusCode::INVALID_ARGUMENT, "extent names device " + std::to_string(e.device) +
                                                                 " beyond the device table"});
    DeviceGuard guard(cfg_.accel_id);
    // Back the namespace ranges on emulated controllers.
    for (std::size_t d = 0; d < devs_.size(); ++d) {
        nvme::EmulatedNvmeController* emu = devs_[d].controller->emulated_drive();
        if (!emu) continue;  // a real drive: the file system already sits on its namespace
        std::vector<nvme::BackingRange> ranges;
        for (const auto& e : p.extents)
            if (e.device == d) ranges.push_back({e.physical, e.length, e.logical});
        if (!ranges.empty()) TUTTI_RETURN_IF_ERROR_R(R, emu->attach_file(p.path, ranges));
    }
    std::uint32_t row;
    if (!free_target_rows_.empty()) {
        row = free_target_rows_.back();
        free_target_rows_.pop_back();
    } else {
        if (targets_.size() >= cfg_.max_targets) return R::Failure({StatusCode::RESOURCE_EXHAUSTED, "target table full"});
        row = static_cast<std::uint32_t>(targets_.size());
        targets_.emplace_back();
    }
    // Extents into the HBM pool (bump allocation in 16 MiB chunks).
    std::vector<io::DevExtent> ex(p.extents.size());
    for (std::size_t i = 0; i < ex.size(); ++i)
        ex[i] = io::DevExtent{p.extents[i].logical, p.extents[i].physical, p.extents[i].length, p.extents[i].device, 0};
    const std::size_t need = align_up(std::max<std::size_t>(1, ex.size()) * sizeof(io::DevExtent), 256);
    if (need > kExtentChunkBytes) return R::Failure({StatusCode::RESOURCE_EXHAUSTED, "too many extents"});
    if (extent_chunks_.empty() || extent_chunk_used_ + need > kExtentChunkBytes) {
        char* c = nullptr;
        Status s = cuda_status(cudaMalloc(&c, kExtentChunkBytes), "cudaMalloc extents");
        if (!s.ok()) return R::Failure(s);
        extent_chunks_.push_back(c);
        extent_chunk_used_ = 0;
    }
    auto* dex = reinterpret_cast<io::DevExtent*>(extent_chunks_.back() + extent_chunk_used_);
    extent_chunk_used_ += need;
    if (!ex.empty()) {
        const char* b = reinterpret_cast<const char*>(ex.data());
        uploads.push_back({extent_chunks_.back(), reinterpret_cast<char*>(dex),
                           std::vector<char>(b, b + ex.size() * sizeof(ex[0]))});
    }
    TargetRec& tr = targets_[row];
    tr.generation = next_token_++;
    tr.row = row;
    tr.size = p.file_size;
    tr.path = p.path;
    tr.open = true;
    io::DevTarget dt{dex, p.file_size, static_cast<std::uint32_t>(ex.size()),
                     static_cast<std::uint32_t>(tr.generation), 0};
    const char* b = reinterpret_cast<const char*>(&dt);
    uploads.push_back({reinterpret_cast<const char*>(d_targets_), reinterpret_cast<char*>(d_targets_ + row),
                       std::vector<char>(b, b + sizeof(dt))});
    return DataPathTarget{row, tr.generation};
}

Status GpuNvmeDataPath::close(DataPathTarget t) {
    std::lock_guard<std::mutex> g(mu_);
    if (t.token >= targets_.size() || targets_[t.token].generation != t.generation || !targets_[t.token].open)
        return {StatusCode::NOT_FOUND, "unknown target"};
    targets_[t.token].open = false;
    targets_[t.token].generation = 0;
    free_target_rows_.push_back(static_cast<std::uint32_t>(t.token));
    DeviceGuard guard(cfg_.accel_id);
    io::DevTarget zero{};
    Status cs = cuda_status(cudaMemcpyAsync(d_targets_ + t.token, &zero, sizeof(zero), cudaMemcpyHostToDevice,
                                            upload_stream_), "clear target");
    if (cs.ok()) cs = cuda_status(cudaStreamSynchronize(upload_stream_), "clear target");
    return cs;
}

Result<RegistrationDomainKey> GpuNvmeDataPath::registration_domain(DataPathTarget) const {
    return RegistrationDomainKey{"nvme-gpu:" + std::to_string(cfg_.accel_id)};
}

Result<DataPathMemory> GpuNvmeDataPath::register_memory(const DataPathMemoryView& v, const RegistrationDomainKey&) {
    using R = Result<DataPathMemory>;
    if (!v.base || v.size_bytes == 0) return R::Failure({StatusCode::INVALID_ARGUMENT, "empty memory"});
    if (reinterpret_cast<std::uintptr_t>(v.base) % 16)
        return R::Failure({StatusCode::INVALID_ARGUMENT, "memory base must be 16-byte aligned"});
    std::lock_guard<std::mutex> g(mu_);
    if (v.kind == DataPathMemoryKind::DEVICE && v.expected_accel_id >= 0 && v.expected_accel_id != cfg_.accel_id) {
        // Another GPU's memory (e.g. a TP peer's KV pool mapped through CUDA IPC):
        // usable when this GPU can reach it over NVLink/P2P.
        int can = 0;
        if (cudaDeviceCanAccessPeer(&can, cfg_.accel_id, v.expected_accel_id) != cudaSuccess || !can) {
            cudaGetLastError();
            return R::Failure({StatusCode::INVALID_ARGUMENT, "memory belongs to an accelerator without peer access"});
        }
    }
    std::uint64_t tok = next_token_++;
    memories_[tok] = MemoryRec{tok, static_cast<char*>(v.base), v.size_bytes, v.kind};
    if (cfg_.direct_reads && initialized_ && v.kind == DataPathMemoryKind::DEVICE &&
        (v.expected_accel_id < 0 || v.expected_accel_id == cfg_.accel_id)) {
        // This GPU's own memory: the drives may DMA into it. A region that
        // cannot be mapped stays registered and is served through staging.
        Status ms = map_direct_region_locked(tok, static_cast<char*>(v.base), v.size_bytes);
        if (!ms.ok())
            std::fprintf(stderr, "[tutti] nvme-gpu accel %d: memory served through staging (%s)\n", cfg_.accel_id,
                         ms.message().c_str());
    }
    return DataPathMemory{tok, tok};
}

Status GpuNvmeDataPath::unregister_memory(DataPathMemory m) {
    std::lock_guard<std::mutex> g(mu_);
    auto it = memories_.find(m.token);
    if (it == memories_.end() || it->second.generation != m.generation) return {StatusCode::NOT_FOUND, "unknown memory"};
    memories_.erase(it);
    if (direct_regions_.count(m.token)) unmap_direct_region_locked(m.token);
    return Status::Ok();
}

Status GpuNvmeDataPath::map_direct_region_locked(std::uint64_t token, char* base, std::uint64_t bytes) {
    DeviceGuard guard(cfg_.accel_id);
    DirectRegion r;
    r.base = base;
    r.bytes = bytes;
    for (std::size_t d = 0; d < devs_.size(); ++d) {
        auto m = devs_[d].controller->map_dma(base, bytes);
        if (!m.ok() || !m.value().covers(base, bytes)) {
            for (std::size_t k = 0; k < r.maps.size(); ++k) devs_[k].controller->unmap_dma(r.maps[k]);
            return m.ok() ? Status{StatusCode::INTERNAL, "DMA mapping does not cover the memory"} : m.status();
        }
        r.maps.push_back(std::move(m).value());
        const nvme::DmaMapping& a = r.maps.front();
        const nvme::DmaMapping& b = r.maps.back();
        const bool pow2 = a.page_bytes == 0 || (a.page_bytes >= 4096 && (a.page_bytes & (a.page_bytes - 1)) == 0);
        if (!pow2 || a.va != b.va || a.page_bytes != b.page_bytes || a.bus != b.bus) {
            for (std::size_t k = 0; k < r.maps.size(); ++k) devs_[k].controller->unmap_dma(r.maps[k]);
            return {StatusCode::UNSUPPORTED, "controllers disagree on the memory's bus addresses"};
        }
    }
    const nvme::DmaMapping& m = r.maps.front();
    Status st = cuda_status(cudaMalloc(&r.d_bus, m.bus.size() * 8), "cudaMalloc bus table");
    if (st.ok())
        st = cuda_status(cudaMemcpyAsync(r.d_bus, m.bus.data(), m.bus.size() * 8, cudaMemcpyHostToDevice, upload_stream_),
                         "upload bus table");
    if (st.ok()) st = cuda_status(cudaStreamSynchronize(upload_stream_), "upload bus table");
    if (!st.ok()) {
        for (std::size_t k = 0; k < r.maps.size(); ++k) devs_[k].controller->unmap_dma(r.maps[k]);
        if (r.d_bus) cudaFree(r.d_bus);
        return st;
    }
    direct_regions_[token] = std::move(r);
    return publish_regions_locked();
}

void GpuNvmeDataPath::unmap_direct_region_locked(std::uint64_t token) {
    auto it = direct_regions_.find(token);
    if (it == direct_regions_.end()) return;
    DirectRegion r = std::move(it->second);
    direct_regions_.erase(it);
    (void)publish_regions_locked();
    for (std::size_t d = 0; d < r.maps.size() && d < devs_.size(); ++d) devs_[d].controller->unmap_dma(r.maps[d]);
    retired_device_tables_.push_back(r.d_bus);  // an op in flight may still hold the old table
}

Status GpuNvmeDataPath::publish_regions_locked() {
    // A new device table per change: ops in flight keep reading the one they
    // were launched with.
    std::vector<io::DmaRegion> rows;
    for (const auto& kv : direct_regions_) {
        const DirectRegion& r = kv.second;
        const nvme::DmaMapping& m = r.maps.front();
        io::DmaRegion row{};
        row.lo = reinterpret_cast<std::uint64_t>(r.base);
        row.hi = row.lo + r.bytes;
        row.va = m.va;
        row.bus = r.d_bus;
        row.page_shift = m.page_bytes ? static_cast<std::uint32_t>(__builtin_ctzll(m.page_bytes)) : 0u;
        rows.push_back(row);
    }
    std::sort(rows.begin(), rows.end(), [](const io::DmaRegion& a, const io::DmaRegion& b) { return a.lo < b.lo; });
    io::DmaRegion* table = nullptr;
    if (!rows.empty()) {
        TUTTI_RETURN_IF_ERROR(cuda_status(cudaMalloc(&table, rows.size() * sizeof(io::DmaRegion)), "cudaMalloc regions"));
        TUTTI_RETURN_IF_ERROR(cuda_status(cudaMemcpyAsync(table, rows.data(), rows.size() * sizeof(io::DmaRegion),
                                                          cudaMemcpyHostToDevice, upload_stream_),
                                          "upload regions"));
        TUTTI_RETURN_IF_ERROR(cuda_status(cudaStreamSynchronize(upload_stream_), "upload regions"));
    }
    if (d_regions_) retired_device_tables_.push_back(d_regions_);
    d_regions_ = table;
    n_regions_ = static_cast<std::uint32_t>(rows.size());
    return Status::Ok();
}

Result<std::unique_ptr<GpuNvmeDataPath::Arena>> GpuNvmeDataPath::take_arena(std::size_t bytes) {
    using R = Result<std::unique_ptr<Arena>>;
    for (std::size_t i = 0; i < arena_pool_.size(); ++i) {
        if (arena_pool_[i]->capacity >= bytes) {
            auto a = std::move(arena_pool_[i]);
            arena_pool_.erase(arena_pool_.begin() + i);
            return R(std::move(a));
        }
    }
    auto a = std::make_unique<Arena>();
    a->capacity = align_up(std::max<std::size_t>(bytes, 1u << 20), 1u << 20);
    Status s = cuda_status(cudaHostAlloc(reinterpret_cast<void**>(&a->host), a->capacity, cudaHostAllocMapped),
                           "cudaHostAlloc arena");
    if (!s.ok()) return R::Failure(s);
    s = cuda_status(cudaHostGetDevicePointer(reinterpret_cast<void**>(&a->host_dev), a->host, 0),
                    "cudaHostGetDevicePointer arena");
    if (!s.ok()) {
        cudaFreeHost(a->host);
        return R::Failure(s);
    }
    s = cuda_status(cudaMalloc(&a->dev, a->capacity), "cudaMalloc arena");
    if (!s.ok()) {
        cudaFreeHost(a->host);
        return R::Failure(s);
    }
    s = cuda_status(cudaEventCreateWithFlags(&a->event, cudaEventDisableTiming), "cudaEventCreate");
    if (s.ok()) s = cuda_status(cudaEventCreateWithFlags(&a->submitted, cudaEventDisableTiming), "cudaEventCreate");
    if (s.ok()) s = cuda_status(cudaEventCreateWithFlags(&a->uploaded, cudaEventDisableTiming), "cudaEventCreate");
    if (!s.ok()) {
        if (a->event) cudaEventDestroy(a->event);
        if (a->submitted) cudaEventDestroy(a->submitted);
        cudaFreeHost(a->host);
        cudaFree(a->dev);
        return R::Failure(s);
    }
    return R(std::move(a));
}

void GpuNvmeDataPath::return_arena(std::unique_ptr<Arena> a) {
    if (a) arena_pool_.push_back(std::move(a));
}

SubmitOutcome GpuNvmeDataPath::submit(const DataPathRequest* reqs, std::size_t count, const HostSubmitContext& ctx) {
    SubmitOutcome out;
    const auto t_start = std::chrono::steady_clock::now();
    out.initial_states.resize(count);
    if (count == 0) return out;
    std::lock_guard<std::mutex> g(mu_);
    auto reject_all = [&](Status s) {
        for (auto& st : out.initial_states) st = {IoRequestState::REJECTED, s};
        out.status = s;
        return out;
    };
    if (!initialized_) return reject_all({StatusCode::NOT_READY, "not initialized"});
    if (ctx.execution_domain != ExecutionDomain::DEVICE_EXECUTION)
        return reject_all({StatusCode::UNSUPPORTED, "nvme-gpu executes on the device"});

    const std::uint64_t lba = lba_;
    const bool xform = ctx.transform != IoTransform::NONE;
    if (xform && ctx.transform != IoTransform::FP8_E4M3_BLOCK128)
        return reject_all({StatusCode::INVALID_ARGUMENT, "unknown IoTransform"});
    // Soft size of a transformed command: it may grow past this (up to one
    // slot) to reach an LBA-aligned end.
    const std::uint32_t xform_budget = cmd_bytes_ > (256u << 10) ? cmd_bytes_ - (256u << 10) : cmd_bytes_ / 2;
    auto op = std::make_unique<OpRec>();
    std::vector<io::IoCommand> cmds;
    std::vector<io::IoPiece> pieces;
    cmds.reserve(count / 8 + 1);
    pieces.reserve(count + 16);
    op->cmd_first_piece.reserve(count / 8 + 1);
    op->piece_req.reserve(count + 16);
    Status first_reject;
    std::size_t accepted = 0;
    op->req_input_index.reserve(count);
    op->req_bytes.reserve(count);
    std::uint64_t last_mem_token = 0;
    auto last_mit = memories_.end();

    for (std::size_t i = 0; i < count; ++i) {
        const DataPathRequest& r = reqs[i];
        const IoRequest& in = r.intent;
        if (last_mit == memories_.end() || r.memory.token != last_mem_token) {
            last_mit = memories_.find(r.memory.token);
            last_mem_token = r.memory.token;
        }
        auto mit = last_mit;
        Status bad;
        if (mit == memories_.end() || mit->second.generation != r.memory.generation)
            bad = {StatusCode::NOT_FOUND, "unknown memory"};
        else if (r.target.token >= targets_.size() || targets_[r.target.token].generation != r.target.generation ||
                 !targets_[r.target.token].open)
            bad = {StatusCode::NOT_FOUND, "unknown target"};
        else if (in.length == 0 || in.length % 16 || in.target_offset % 16)
            bad = {StatusCode::INVALID_ARGUMENT, "offset/length must be 16-byte aligned"};
        else if (xform && (in.length % 1024 || stored_bytes(ctx.transform, in.length) > cmd_bytes_))
            bad = {StatusCode::INVALID_ARGUMENT, "fp8 transform: 1024-byte lengths, one slot at most"};
        else if (!xform && (in.length % lba || in.target_offset % lba) && in.length > cmd_bytes_)
            bad = {StatusCode::INVALID_ARGUMENT, "a request that is not LBA aligned must fit one slot"};
        else if (in.memory_offset + in.length > mit->second.size)
            bad = {StatusCode::OUT_OF_RANGE, "memory range"};
        else if (in.target_offset + stored_bytes(ctx.transform, in.length) > targets_[r.target.token].size)
            bad = {StatusCode::OUT_OF_RANGE, "target range"};
        else if ((reinterpret_cast<std::uintptr_t>(mit->second.base) + in.memory_offset) % 16)
            bad = {StatusCode::INVALID_ARGUMENT, "memory address must be 16-byte aligned"};
        if (!bad.ok()) {
            out.initial_states[i] = {IoRequestState::REJECTED, bad};
            if (first_reject.ok()) first_reject = bad;
            continue;
        }
        out.initial_states[i].state = IoRequestState::ACCEPTED;  // its status is already Ok
        const std::uint32_t req_idx = static_cast<std::uint32_t>(accepted++);
        op->req_input_index.push_back(static_cast<std::uint32_t>(i));
        op->req_bytes.push_back(in.length);
        const std::uint32_t opcode = in.direction == IoDirection::READ ? nvme::kOpRead : nvme::kOpWrite;
        if (xform || in.length % lba || in.target_offset % lba) {
            // A transformed or sub-sector request is one piece (for the transform:
            // [values][scales]) and is never split. A command closes only where the
            // stored stream is LBA-aligned: past the soft budget it keeps growing
            // until such a boundary.
            const std::uint16_t kind = xform ? io::kXformFp8Block128 : io::kXformNone;
            const std::uint64_t sb = stored_bytes(ctx.transform, in.length);
            bool extend = false;
            if (!cmds.empty()) {
                const io::IoCommand& c = cmds.back();
                const bool aligned_end = (c.logical + c.bytes) % lba == 0;
                extend = c.opcode == opcode && c.transform == kind &&
                         c.target == r.target.token && c.logical + c.bytes == in.target_offset &&
                         c.bytes + sb <= cmd_bytes_ && c.n_pieces < cfg_.max_pieces_per_cmd &&
                         (c.bytes < xform_budget || !aligned_end);
            }
            if (!extend) {
                io::IoCommand c{};
                c.logical = in.target_offset;
                c.target = static_cast<std::uint32_t>(r.target.token);
                c.first_piece = static_cast<std::uint32_t>(pieces.size());
                c.opcode = static_cast<std::uint16_t>(opcode);
                c.transform = kind;
                cmds.push_back(c);
                op->cmd_first_piece.push_back(c.first_piece);
            }
            io::IoCommand& c = cmds.back();
            pieces.push_back(io::IoPiece{reinterpret_cast<std::uint64_t>(mit->second.base + in.memory_offset), c.bytes,
                                         static_cast<std::uint32_t>(sb)});
            op->piece_req.push_back(req_idx);
            c.bytes += static_cast<std::uint32_t>(sb);
            c.n_pieces += 1;
            op->bytes += in.length;
            continue;
        }
        std::uint64_t done = 0;
        while (done < in.length) {
            const std::uint64_t lo = in.target_offset + done;
            bool extend = false;
            if (!cmds.empty()) {
                const io::IoCommand& c = cmds.back();
                extend = c.opcode == opcode && c.transform == io::kXformNone && c.target == r.target.token &&
                         c.logical + c.bytes == lo &&
                         c.bytes < cmd_bytes_ && c.n_pieces < cfg_.max_pieces_per_cmd;
            }
            if (!extend) {
                io::IoCommand c{};
                c.logical = lo;
                c.target = static_cast<std::uint32_t>(r.target.token);
                c.bytes = 0;
                c.first_piece = static_cast<std::uint32_t>(pieces.size());
                c.n_pieces = 0;
                c.opcode = static_cast<std::uint16_t>(opcode);
                cmds.push_back(c);
                op->cmd_first_piece.push_back(c.first_piece);
            }
            io::IoCommand& c = cmds.back();
            const std::uint64_t n = std::min<std::uint64_t>(in.length - done, cmd_bytes_ - c.bytes);
            pieces.push_back(io::IoPiece{reinterpret_cast<std::uint64_t>(mit->second.base + in.memory_offset + done),
                                         c.bytes, static_cast<std::uint32_t>(n)});
            op->piece_req.push_back(req_idx);
            c.bytes += static_cast<std::uint32_t>(n);
            c.n_pieces += 1;
            done += n;
        }
        op->bytes += in.length;
    }
    if (accepted == 0) {
        out.status = first_reject;
        return out;
    }
    for (const auto& c : cmds)
        if (c.logical % lba || c.bytes % lba)
            return reject_all({StatusCode::INVALID_ARGUMENT,
                               "requests that are not LBA aligned (or transformed) must tile LBA-aligned runs"});
    merge_replicas(cmds, pieces, op->cmd_first_piece, op->piece_req);
    const std::uint32_t n_cmds = static_cast<std::uint32_t>(cmds.size());
    const auto t_coalesced = std::chrono::steady_clock::now();
    std::uint32_t want = std::min<std::uint32_t>(cfg_.max_ctas_per_op, n_cmds);
    std::uint32_t take = std::min<std::uint32_t>(want, static_cast<std::uint32_t>(free_leases_.size()));
    if (take == 0) return reject_all({StatusCode::BUSY, "all queue leases are held by in-flight operations"});

    DeviceGuard guard(cfg_.accel_id);
    // Arena layout: cmds | pieces | lease ids | cursor | status | timing
    const std::size_t off_cmds = 0;
    const std::size_t off_pieces = align_up(off_cmds + cmds.size() * sizeof(io::IoCommand), 256);
    const std::size_t off_leases = align_up(off_pieces + pieces.size() * sizeof(io::IoPiece), 256);
    const std::size_t off_cursor = align_up(off_leases + take * sizeof(std::uint32_t), 256);
    const std::size_t off_status = align_up(off_cursor + 16, 256);
    const std::size_t off_timing = align_up(off_status + n_cmds * sizeof(std::uint32_t), 256);
    const bool timing = cfg_.timing;
    const std::size_t copy_end = off_timing + (timing ? n_cmds * 4 * sizeof(std::uint64_t) : 0);
    // Split completion for reads of any size: the submit launch fills every leased
    // slot and exits; the drain takes those slots over and claims the rest of the
    // op's commands itself, so the SMs are held only from the drain on.
    bool split = cfg_.async_completion;
    for (std::size_t k = 0; split && k < cmds.size(); ++k) split = cmds[k].opcode == nvme::kOpRead;
    const std::size_t off_carry = align_up(copy_end, 256);  // in the mapped host half (zero-copy)
    const std::size_t total = split ? off_carry + take * sizeof(io::LeaseCarry) : copy_end;
    auto ar = take_arena(total);
    if (!ar.ok()) return reject_all(ar.status());
    std::unique_ptr<Arena> arena = std::move(ar).value();
    char* h = arena->host;
    std::memcpy(h + off_cmds, cmds.data(), cmds.size() * sizeof(io::IoCommand));
    std::memcpy(h + off_pieces, pieces.data(), pieces.size() * sizeof(io::IoPiece));
    for (std::uint32_t k = 0; k < take; ++k) {
        op->leases.push_back(free_leases_.back());
        free_leases_.pop_back();
    }
    std::memcpy(h + off_leases, op->leases.data(), take * sizeof(std::uint32_t));
    std::memset(h + off_cursor, 0, 16);
    // Status words and timing stamps live in the mapped host half of the arena:
    // the kernel stores them over PCIe, so no copy is ever queued behind it (a
    // copy waiting on a running io kernel would also hold up any drive DMA that
    // shares its hardware queue).
    if (timing) std::memset(h + off_timing, 0, copy_end - off_timing);
    auto* hst = reinterpret_cast<std::uint32_t*>(h + off_status);
    for (std::uint32_t k = 0; k < n_cmds; ++k) hst[k] = io::kCmdNotRun;

    io::IoKernelParams kp{};
    char* d = arena->dev;
    kp.cmds = reinterpret_cast<const io::IoCommand*>(d + off_cmds);
    kp.pieces = reinterpret_cast<const io::IoPiece*>(d + off_pieces);
    kp.n_cmds = n_cmds;
    kp.n_devices = static_cast<std::uint32_t>(devs_.size());
    kp.cursor = reinterpret_cast<std::uint32_t*>(d + off_cursor);
    kp.cmd_status = reinterpret_cast<std::uint32_t*>(arena->host_dev + off_status);
    kp.targets = d_targets_;
    kp.devices = d_devices_;
    kp.lease_ids = reinterpret_cast<const std::uint32_t*>(d + off_leases);
    kp.staging_dev = staging_base();
    kp.page_bus = d_page_bus_;
    kp.list_bus = d_list_bus_;
    kp.regions = d_regions_;
    kp.n_regions = n_regions_;
    kp.direct_lists = direct_lists_.device_as<std::uint64_t>();
    kp.direct_list_bus = d_direct_list_bus_;
    kp.movers = staging_on_device_ ? io::kMoversBulk : io::kMoversSimt;
    kp.slot_bytes = cfg_.slot_bytes;
    kp.slots_per_lease = cfg_.slots_per_lease;
    kp.timeout_ns = cfg_.timeout_ns;
    kp.timing = timing ? reinterpret_cast<std::uint64_t*>(arena->host_dev + off_timing) : nullptr;
    kp.carry = split ? reinterpret_cast<io::LeaseCarry*>(arena->host_dev + off_carry) : nullptr;
    kp.phase = split ? io::kPhaseSubmit : io::kPhaseFull;

    cudaStream_t s = ctx.stream;
    const bool nvtx = nvtx_enabled();
    if (nvtx) {
        char name[128];
        std::snprintf(name, sizeof(name), "tutti.nvme_gpu.submit|op=%s|cmds=%u|ctas=%u%s",
                      cmds[0].opcode == nvme::kOpRead ? "read" : "write", n_cmds, take, xform ? "|fp8" : "");
        nvtxRangePushA(name);
    }
    Status cs = cuda_status(cudaMemcpyAsync(d, h, off_status, cudaMemcpyHostToDevice, upload_stream_), "H2D commands");
    if (cs.ok()) cs = cuda_status(cudaEventRecord(arena->uploaded, upload_stream_), "event record");
    if (cs.ok()) cs = cuda_status(cudaStreamWaitEvent(s, arena->uploaded, 0), "stream wait");
    bool launched = false;
    if (cs.ok()) {
        if (take_test_fault(TestFault::LAUNCH_FAILURE)) {
            cs = {StatusCode::DEVICE_ERROR, "io kernel launch: injected failure"};
        } else {
            cs = cuda_status(io::launch_nvme_io(kp, take, s), "io kernel launch");
            launched = cs.ok();
        }
    }
    if (nvtx) nvtxRangePop();
    auto record = [&](cudaEvent_t ev) {
        if (take_test_fault(TestFault::EVENT_RECORD_FAILURE))
            return Status{StatusCode::DEVICE_ERROR, "event record: injected failure"};
        return cuda_status(cudaEventRecord(ev, s), "event record");
    };
    if (split) {
        if (cs.ok()) cs = record(arena->submitted);
    } else {
        if (cs.ok()) cs = record(arena->event);
    }
    if (!cs.ok() && !launched) {
        // The kernel was not issued, so nothing irreversible happened:
        // report every request rejected and return the leases.
        cudaStreamSynchronize(upload_stream_);
        cudaStreamSynchronize(s);
        for (auto l : op->leases) free_leases_.push_back(l);
        return_arena(std::move(arena));
        return reject_all(cs);
    }
    op->arena = std::move(arena);
    op->n_cmds = n_cmds;
    op->status_off = off_status;
    op->timing_off = off_timing;
    op->timing = timing;
    if (split) {
        op->drain_pending = true;
        op->kp = kp;
        op->kp.phase = io::kPhaseDrain;
        op->ctas = take;
        op->copy_back_bytes = copy_end - off_status;
        op->carry_off = off_carry;
        op->stream = s;
        op->submitted_at = std::chrono::steady_clock::now();
    }
    if (!cs.ok()) {
        // The kernel is issued but its completion cannot be tracked by an
        // event: the IO happens regardless, so the requests count as accepted.
        // Wait for it here (the one synchronising path of submit), run the
        // drain phase too when the read was split, then settle the op from
        // its command statuses.
        Status ws = cuda_status(cudaStreamSynchronize(s), "stream synchronize");
        if (ws.ok() && split) {
            op->kp.phase = io::kPhaseDrain;
            ws = cuda_status(io::launch_nvme_io(op->kp, op->ctas, s), "drain launch");
            op->drain_pending = false;
            if (ws.ok()) ws = cuda_status(cudaStreamSynchronize(s), "stream synchronize");
        }
        if (ws.ok()) {
            finish_op(*op);
        } else {
            cudaGetLastError();
            op->state = IoState::FAILED;
            op->status = ws;
            op->detail.failure_kind = IoFailureKind::UNKNOWN;
            op->detail.failure_scope = IoFailureScope::WHOLE_OPERATION;  // leases stay held
        }
    }
    op->generation = next_token_++;
    last_submit_profile_.coalesce_ms = std::chrono::duration<double, std::milli>(t_coalesced - t_start).count();
    last_submit_profile_.launch_ms =
        std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t_coalesced).count();
    last_submit_profile_.commands = n_cmds;
    last_submit_profile_.requests = count;
    last_submit_profile_.h2d_bytes = off_status;
    last_submit_profile_.d2h_bytes = copy_end - off_status;
    const std::uint64_t tok = op->generation;
    ops_[tok] = std::move(op);
    out.op = DataPathOp{tok, tok};
    out.status = first_reject;  // non-OK when partially rejected
    return out;
}

Status GpuNvmeDataPath::reset_dirty_queues(const std::vector<std::uint32_t>& leases) {
    // Caller holds mu_; the op is terminal, so its kernels have written the cursors.
    // A queue the controller cannot reset (a real drive resets whole queue
    // groups only) retires its lease: it never serves another op.
    Status first;
    for (std::size_t d = 0; d < devs_.size(); ++d) {
        auto* cur = cursor_mem_[d].host_as<io::QueueCursor>();
        for (auto l : leases) {
            if (!reinterpret_cast<volatile io::QueueCursor*>(cur)[l].dirty) continue;
            Status s = devs_[d].controller->reset_queue(l);
            if (!s.ok()) {
                retire_lease_locked(l, s);
                if (first.ok()) first = s;
                continue;
            }
            cur[l] = io::QueueCursor{0, 0, 1, 0};
        }
    }
    return first;
}

void GpuNvmeDataPath::retire_lease_locked(std::uint32_t lease, const Status& why) {
    if (lease < retired_.size() && !retired_[lease]) {
        retired_[lease] = true;
        std::fprintf(stderr, "[tutti] nvme-gpu accel %d: lease %u retired (%s)\n", cfg_.accel_id, lease,
                     why.message().c_str());
    }
}

void GpuNvmeDataPath::return_leases_locked(const std::vector<std::uint32_t>& leases) {
    for (auto l : leases)
        if (l >= retired_.size() || !retired_[l]) free_leases_.push_back(l);
}

bool GpuNvmeDataPath::split_data_ready(const OpRec& op) const {
    const cudaError_t e = cudaEventQuery(op.arena->submitted);
    if (e != cudaSuccess) {
        if (e != cudaErrorNotReady) cudaGetLastError();
        return false;
    }
    const auto* carry = reinterpret_cast<const volatile io::LeaseCarry*>(op.arena->host + op.carry_off);
    for (std::size_t i = 0; i < op.leases.size(); ++i) {
        const std::uint32_t l = op.leases[i];
        for (std::size_t d = 0; d < devs_.size(); ++d) {
            const std::uint32_t n = carry[i].inflight_dev[d];
            if (n == 0) continue;
            const auto* cur = reinterpret_cast<const volatile io::QueueCursor*>(cursor_mem_[d].host) + l;
            const std::uint32_t head = cur->cq_head, phase = cur->phase;
            const nvme::QueuePairView q = devs_[d].controller->host_queue(l);
            if (!q.cq) return false;  // a CQ in GPU memory: the drain waits for the fallback timer
            for (std::uint32_t k = 0; k < n; ++k) {
                const std::uint32_t at = head + k;
                const std::uint32_t want = (at >= q.depth) ? (phase ^ 1u) : phase;
                const std::uint32_t dw3 = __atomic_load_n(&q.cq[at % q.depth].dw3, __ATOMIC_ACQUIRE);
                if (nvme::cqe_phase(dw3) != want) return false;
            }
        }
    }
    return true;
}

void GpuNvmeDataPath::finish_op(OpRec& op) {
    const auto* st = reinterpret_cast<const std::uint32_t*>(op.arena->host + op.status_off);
    std::vector<char> req_failed(op.req_bytes.size(), 0);
    IoCompletionDetail det;
    bool any_fail = false, any_timeout_or_notrun = false;
    for (std::uint32_t c = 0; c < op.n_cmds; ++c) {
        const std::uint32_t code = st[c];
        if (code == io::kCmdOk) continue;
        any_fail = true;
        const std::uint32_t kind = code & 0xFFFF0000u;
        if (det.first_failed_entry == UINT32_MAX) {
            det.first_failed_entry = c;
            det.failure_kind = kind == io::kCmdResolve || kind == io::kCmdBadDevice ? IoFailureKind::RESOLVE_LBA
                               : kind == io::kCmdTimeout                           ? IoFailureKind::CQ_TIMEOUT
                               : kind == io::kCmdNvme                              ? IoFailureKind::NVME_CQ_ERROR
                                                                                   : IoFailureKind::UNKNOWN;
            det.raw_cq_status = code & 0xFFFFu;
        }
        if (kind == io::kCmdTimeout || kind == io::kCmdNotRun) any_timeout_or_notrun = true;
        if (kind == io::kCmdTimeout) det.timeout_seen = true;
        const std::uint32_t p0 = op.cmd_first_piece[c];
        const std::uint32_t p1 = c + 1 < op.n_cmds ? op.cmd_first_piece[c + 1] : static_cast<std::uint32_t>(op.piece_req.size());
        for (std::uint32_t p = p0; p < p1; ++p) req_failed[op.piece_req[p]] = 1;
    }
    for (std::size_t r = 0; r < req_failed.size(); ++r) {
        if (req_failed[r])
            det.failed_request_indices.push_back(op.req_input_index[r]);
        else
            det.confirmed_bytes += op.req_bytes[r];
    }
    if (any_fail) det.failure_scope = IoFailureScope::REQUEST_INDICES;
    op.detail = std::move(det);
    if (any_timeout_or_notrun) {
        Status rs = reset_dirty_queues(op.leases);
        (void)rs;  // a lease whose queue could not be reset is retired
    }
    return_leases_locked(op.leases);
    op.leases.clear();
    op.state = any_fail ? IoState::FAILED : IoState::COMPLETED;
    op.status = any_fail ? Status(StatusCode::DEVICE_ERROR,
                                  std::to_string(op.detail.failed_request_indices.size()) + " request(s) failed")
                         : Status::Ok();
    if (op.timing) {
        const auto* t = reinterpret_cast<const std::uint64_t*>(op.arena->host + op.timing_off);
        std::vector<double> qw, dev, mv, tot;
        for (std::uint32_t c = 0; c < op.n_cmds; ++c) {
            const std::uint64_t* s = t + 4ull * c;
            if (!s[0] || !s[3]) continue;
            qw.push_back((s[1] - s[0]) / 1e3);
            dev.push_back((s[2] - s[1]) / 1e3);
            mv.push_back((s[3] - s[2]) / 1e3);
            tot.push_back((s[3] - s[0]) / 1e3);
        }
        IoTimingSummary ts;
        ts.commands = tot.size();
        ts.queue_wait_us_p50 = percentile(qw, 0.5);
        ts.move_us_p50 = percentile(mv, 0.5);
        std::vector<double> dev2 = dev, tot2 = tot;
        ts.device_us_p50 = percentile(dev, 0.5);
        ts.device_us_p99 = percentile(dev2, 0.99);
        ts.total_us_p50 = percentile(tot, 0.5);
        ts.total_us_p99 = percentile(tot2, 0.99);
        last_timing_ = ts;
    }
}

Status GpuNvmeDataPath::launch_drain(OpRec& op, cudaStream_t stream) {
    // Caller holds mu_. Orders the drain after the submit-phase kernel and marks
    // the op's completion event (the kernel writes the statuses to host memory).
    DeviceGuard guard(cfg_.accel_id);
    Status cs = cuda_status(cudaStreamWaitEvent(stream, op.arena->submitted, 0), "stream wait");
    if (cs.ok()) cs = cuda_status(io::launch_nvme_io(op.kp, op.ctas, stream), "drain launch");
    if (cs.ok()) cs = cuda_status(cudaEventRecord(op.arena->event, stream), "event record");
    op.drain_pending = false;
    return cs;
}

Result<ProgressResult> GpuNvmeDataPath::progress(ProgressBudget budget) {
    std::lock_guard<std::mutex> g(mu_);
    ProgressResult pr;
    DeviceGuard guard(cfg_.accel_id);
    for (auto& kv : ops_) {
        OpRec& op = *kv.second;
        if (op.state != IoState::IN_FLIGHT) continue;
        if (budget.max_work_units && pr.work_units_consumed >= budget.max_work_units) {
            pr.more_work_likely = true;
            break;
        }
        ++pr.work_units_consumed;
        if (op.drain_pending) {
            // No consumer has asked for the data yet: launch the drain here once the
            // drives have completed the submitted wave, or after async_fallback_us.
            const auto waited = std::chrono::steady_clock::now() - op.submitted_at;
            if (split_data_ready(op) || waited >= std::chrono::microseconds(cfg_.async_fallback_us)) {
                Status ds = launch_drain(op, op.stream);
                if (!ds.ok()) {
                    op.state = IoState::FAILED;
                    op.status = ds;
                    op.detail.failure_kind = IoFailureKind::UNKNOWN;
                    op.detail.failure_scope = IoFailureScope::WHOLE_OPERATION;
                    ++pr.operations_terminal;
                    continue;  // leases stay held: queues hold submitted commands
                }
            }
            pr.more_work_likely = true;
            continue;
        }
        cudaError_t e = take_test_fault(TestFault::QUERY_ERROR) ? cudaErrorUnknown : cudaEventQuery(op.arena->event);
        if (e == cudaErrorNotReady) {
            pr.more_work_likely = true;
            continue;
        }
        ++pr.operations_advanced;
        ++pr.operations_terminal;
        if (e != cudaSuccess) {
            cudaGetLastError();
            op.state = IoState::FAILED;
            op.status = {StatusCode::DEVICE_ERROR, std::string("event query: ") + cudaGetErrorString(e)};
            op.detail.failure_kind = IoFailureKind::CUDA_QUERY_ERROR;
            op.detail.failure_scope = IoFailureScope::WHOLE_OPERATION;
            continue;  // leases stay held: the device state is unknown
        }
        finish_op(op);
    }
    return pr;
}

Result<DataPathSnapshot> GpuNvmeDataPath::query(DataPathOp op) const {
    std::lock_guard<std::mutex> g(mu_);
    auto it = ops_.find(op.token);
    if (it == ops_.end() || it->second->generation != op.generation)
        return Result<DataPathSnapshot>::Failure({StatusCode::NOT_FOUND, "unknown op"});
    DataPathSnapshot s;
    s.state = it->second->state;
    s.status = it->second->status;
    s.bytes_transferred = s.state == IoState::IN_FLIGHT ? 0 : it->second->detail.confirmed_bytes;
    s.detail = it->second->detail;
    return s;
}

Status GpuNvmeDataPath::release(DataPathOp op) {
    std::lock_guard<std::mutex> g(mu_);
    auto it = ops_.find(op.token);
    if (it == ops_.end() || it->second->generation != op.generation) return {StatusCode::NOT_FOUND, "unknown op"};
    if (it->second->state == IoState::IN_FLIGHT) return {StatusCode::BUSY, "op still in flight"};
    return_arena(std::move(it->second->arena));
    ops_.erase(it);
    return Status::Ok();
}

Status GpuNvmeDataPath::enqueue_wait(const DataPathOp* ops, std::size_t count, cudaStream_t stream) {
    std::lock_guard<std::mutex> g(mu_);
    DeviceGuard guard(cfg_.accel_id);
    for (std::size_t i = 0; i < count; ++i) {
        auto it = ops_.find(ops[i].token);
        if (it == ops_.end() || it->second->generation != ops[i].generation) return {StatusCode::NOT_FOUND, "unknown op"};
        if (!it->second->arena) continue;  // already terminal and released
        if (it->second->state != IoState::IN_FLIGHT) continue;  // settled: its data is in place
        if (it->second->drain_pending) {
            // Split completion: the drain runs on the consumer's stream, right where it is needed.
            TUTTI_RETURN_IF_ERROR(launch_drain(*it->second, stream));
            continue;
        }
        TUTTI_RETURN_IF_ERROR(cuda_status(cudaStreamWaitEvent(stream, it->second->arena->event, 0), "stream wait"));
    }
    return Status::Ok();
}

IoTimingSummary GpuNvmeDataPath::last_timing() const {
    std::lock_guard<std::mutex> g(mu_);
    return last_timing_;
}

std::uint32_t GpuNvmeDataPath::free_leases() const {
    std::lock_guard<std::mutex> g(mu_);
    return static_cast<std::uint32_t>(free_leases_.size());
}

std::uint32_t GpuNvmeDataPath::noalloc_acquire_leases(std::uint32_t max, std::uint32_t* out) {
    std::lock_guard<std::mutex> g(mu_);
    if (!initialized_) return 0;
    std::uint32_t n = 0;
    while (n < max && !free_leases_.empty()) {
        out[n++] = free_leases_.back();
        free_leases_.pop_back();
    }
    return n;
}

void GpuNvmeDataPath::noalloc_release_leases(const std::uint32_t* leases, std::uint32_t n, bool reset_dirty) {
    std::lock_guard<std::mutex> g(mu_);
    DeviceGuard guard(cfg_.accel_id);
    for (std::uint32_t i = 0; i < n; ++i) {
        const std::uint32_t l = leases[i];
        if (reset_dirty) {
            for (std::size_t d = 0; d < devs_.size(); ++d) {
                auto* cur = cursor_mem_[d].host_as<io::QueueCursor>();
                if (!reinterpret_cast<volatile io::QueueCursor*>(cur)[l].dirty) continue;
                Status s = devs_[d].controller->reset_queue(l);
                if (!s.ok()) {
                    retire_lease_locked(l, s);
                    continue;
                }
                cur[l] = io::QueueCursor{0, 0, 1, 0};
            }
        }
        if (l < retired_.size() && retired_[l]) continue;
        // The vector held every lease at initialize, so its capacity covers this push: no reallocation.
        free_leases_.push_back(l);
    }
}

bool GpuNvmeDataPath::noalloc_memory_ok(std::uint64_t addr, std::uint64_t bytes) const {
    std::lock_guard<std::mutex> g(mu_);
    for (const auto& kv : memories_) {
        const auto base = reinterpret_cast<std::uint64_t>(kv.second.base);
        if (addr >= base && bytes <= kv.second.size && addr - base <= kv.second.size - bytes) return true;
    }
    return false;
}

bool GpuNvmeDataPath::noalloc_target_ok(std::uint32_t row, std::uint64_t logical, std::uint64_t bytes) const {
    std::lock_guard<std::mutex> g(mu_);
    if (row >= targets_.size() || !targets_[row].open) return false;
    return bytes <= targets_[row].size && logical <= targets_[row].size - bytes;
}

void GpuNvmeDataPath::noalloc_fill_params(io::IoKernelParams& p) const {
    std::lock_guard<std::mutex> g(mu_);
    p.n_devices = static_cast<std::uint32_t>(devs_.size());
    p.targets = d_targets_;
    p.devices = d_devices_;
    p.staging_dev = staging_base();
    p.page_bus = d_page_bus_;
    p.list_bus = d_list_bus_;
    p.regions = d_regions_;
    p.n_regions = n_regions_;
    p.direct_lists = direct_lists_.device_as<std::uint64_t>();
    p.direct_list_bus = d_direct_list_bus_;
    p.movers = staging_on_device_ ? io::kMoversBulk : io::kMoversSimt;
    p.slot_bytes = cfg_.slot_bytes;
    p.slots_per_lease = cfg_.slots_per_lease;
    p.timeout_ns = cfg_.timeout_ns;
    p.timing = nullptr;
}

}  // namespace tutti
