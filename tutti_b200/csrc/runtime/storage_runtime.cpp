// StorageRuntime implementation. One registry mutex guards the handle tables;
// resolution in open_batch and DataPath progress run with it released where the
// DataPath allows.

#include <tutti/storage_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <thread>
#include <unordered_map>

#include <cuda_runtime_api.h>

#include "device_guard.h"

namespace tutti {

namespace {
std::atomic<std::uint32_t> g_runtime_ids{1};

std::string scheme_of(std::string_view uri, const OpenOptions& o) {
    if (!o.scheme.empty()) return o.scheme;
    auto p = uri.find("://");
    if (p != std::string_view::npos) return std::string(uri.substr(0, p));
    if (!uri.empty() && uri[0] == '/') return "file";
    return "";
}

bool cuda_ok() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return n > 0;
}

std::uint64_t now_ns() {
    return static_cast<std::uint64_t>(
        std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now().time_since_epoch())
            .count());
}
}  // namespace

struct StorageRuntime::Impl {
    struct DpEntry {
        std::string key;
        DataPath* dp = nullptr;
        DataPathConfig config;
    };
    struct MemoryEntry {
        std::uint64_t generation = 0;
        MemoryView view;
        bool live = false;
        int inflight = 0;
        bool runtime_owned = false;
        std::map<std::string, DataPathMemory> regs;  // per DataPath key
    };
    struct TargetEntry {
        std::uint64_t generation = 0;
        bool live = false;
        std::string uri;
        std::string dp_key;
        struct DpEntry* dpe = nullptr;  // stable: DataPaths are fixed after create
        DataPathTarget dpt;
        std::uint64_t size = 0;
        int inflight = 0;
    };
    struct OpPart {
        std::string dp_key;
        DataPathOp op;
        std::vector<std::uint32_t> input_index;  // DataPath request i -> runtime request index
        bool terminal = false;
        DataPathSnapshot snap;
    };
    struct IoEntry {
        std::uint64_t generation = 0;
        bool live = false;
        IoState state = IoState::IN_FLIGHT;
        std::vector<OpPart> parts;
        // (slot, count) references held on memories / targets while in flight
        std::vector<std::pair<std::uint32_t, std::uint32_t>> mem_refs, tgt_refs;
        IoResult result;
        bool refs_released = false;
        // stub runtimes: accepted request indices of an IO with no DataPath part,
        // in flight until testing_force_complete
        bool stub = false;
        std::vector<std::uint32_t> stub_requests;
    };

    RuntimeConfig cfg;
    std::uint32_t id = 0;
    mutable std::mutex mu;
    RuntimeState state = RuntimeState::RUNNING;
    bool stub = false;  // create_stub: targets and IOs without components
    std::map<std::string, StorageTargetResolver*> resolvers;
    std::vector<DpEntry> dps;
    OwnedComponents owned;
    std::vector<MemoryEntry> mems;
    std::vector<TargetEntry> tgts;
    std::vector<IoEntry> ios;
    std::uint64_t next_gen = 1;
    std::size_t terminal_unreleased = 0;

    DpEntry* dp(const std::string& key) {
        for (auto& d : dps)
            if (d.key == key) return &d;
        return nullptr;
    }

    template <typename Vec>
    static std::uint32_t alloc_slot(Vec& v) {
        for (std::uint32_t i = 0; i < v.size(); ++i)
            if (!v[i].live) return i;
        v.emplace_back();
        return static_cast<std::uint32_t>(v.size() - 1);
    }

    MemoryEntry* mem(const MemoryHandle& h) {
        if (!h.valid() || h.runtime_id() != id || h.slot() >= mems.size()) return nullptr;
        auto& e = mems[h.slot()];
        return (e.live && e.generation == h.generation()) ? &e : nullptr;
    }
    TargetEntry* tgt(const TargetHandle& h) {
        if (!h.valid() || h.runtime_id() != id || h.slot() >= tgts.size()) return nullptr;
        auto& e = tgts[h.slot()];
        return (e.live && e.generation == h.generation()) ? &e : nullptr;
    }
    IoEntry* io(const IoHandle& h) {
        if (!h.valid() || h.runtime_id() != id || h.slot() >= ios.size()) return nullptr;
        auto& e = ios[h.slot()];
        return (e.live && e.generation == h.generation()) ? &e : nullptr;
    }

    Result<DataPathMemory> registration_for(MemoryEntry& m, DpEntry& d) {
        auto it = m.regs.find(d.key);
        if (it != m.regs.end()) return it->second;
        DataPathMemoryView v;
        v.base = m.view.address;
        v.size_bytes = m.view.size;
        v.expected_accel_id = m.view.expected_accel_id;
        v.kind = (m.view.expected_kind == MemoryKind::DEVICE || m.view.expected_kind == MemoryKind::MANAGED)
                     ? DataPathMemoryKind::DEVICE
                     : DataPathMemoryKind::HOST;
        v.io_granularity = m.view.io_granularity;
        const auto& caps = d.dp->capabilities();
        if (v.kind == DataPathMemoryKind::DEVICE && !caps.supports_device_memory)
            return Result<DataPathMemory>::Failure({StatusCode::UNSUPPORTED, d.key + " cannot use device memory"});
        if (v.kind == DataPathMemoryKind::HOST && !caps.supports_host_memory)
            return Result<DataPathMemory>::Failure({StatusCode::UNSUPPORTED, d.key + " cannot use host memory"});
        DeviceGuard g(caps.bound_accel_id);
        auto r = d.dp->register_memory(v, RegistrationDomainKey{d.key});
        if (r.ok()) m.regs[d.key] = r.value();
        return r;
    }

    // Refresh an IO entry from its DataPath parts.
    void refresh(IoEntry& e) {
        if (e.state != IoState::IN_FLIGHT || e.stub) return;
        bool all_terminal = true;
        for (auto& p : e.parts) {
            if (p.terminal) continue;
            DpEntry* d = dp(p.dp_key);
            if (!d) {
                p.terminal = true;
                p.snap.state = IoState::FAILED;
                p.snap.status = {StatusCode::INTERNAL, "DataPath vanished"};
                continue;
            }
            auto s = d->dp->query(p.op);
            if (!s.ok()) {
                p.terminal = true;
                p.snap.state = IoState::FAILED;
                p.snap.status = s.status();
                continue;
            }
            p.snap = s.value();
            if (p.snap.state == IoState::IN_FLIGHT)
                all_terminal = false;
            else
                p.terminal = true;
        }
        if (!all_terminal) return;
        IoResult res;
        res.state = IoState::COMPLETED;
        for (auto& p : e.parts) {
            const auto& d = p.snap.detail;
            res.detail.confirmed_bytes += d.confirmed_bytes;
            res.detail.timeout_seen |= d.timeout_seen;
            if (p.snap.state == IoState::FAILED) {
                res.state = IoState::FAILED;
                if (res.status.ok()) res.status = p.snap.status;
                if (res.detail.failure_kind == IoFailureKind::NONE) {
                    res.detail.failure_kind = d.failure_kind;
                    res.detail.raw_cq_status = d.raw_cq_status;
                }
                if (d.failure_scope == IoFailureScope::WHOLE_OPERATION || d.failure_scope == IoFailureScope::NONE) {
                    res.detail.failure_scope = IoFailureScope::WHOLE_OPERATION;
                    for (auto idx : p.input_index) res.detail.failed_request_indices.push_back(idx);
                } else {
                    if (res.detail.failure_scope != IoFailureScope::WHOLE_OPERATION)
                        res.detail.failure_scope = IoFailureScope::REQUEST_INDICES;
                    for (auto idx : d.failed_request_indices)
                        if (idx < p.input_index.size()) res.detail.failed_request_indices.push_back(p.input_index[idx]);
                }
            }
        }
        std::sort(res.detail.failed_request_indices.begin(), res.detail.failed_request_indices.end());
        if (!res.detail.failed_request_indices.empty())
            res.detail.first_failed_entry = res.detail.failed_request_indices.front();
        e.result = std::move(res);
        e.state = e.result.state;
        ++terminal_unreleased;
        release_refs(e);
    }

    void release_refs(IoEntry& e) {
        if (e.refs_released) return;
        for (auto& r : e.mem_refs)
            if (r.first < mems.size()) mems[r.first].inflight -= static_cast<int>(r.second);
        for (auto& r : e.tgt_refs)
            if (r.first < tgts.size()) tgts[r.first].inflight -= static_cast<int>(r.second);
        e.refs_released = true;
    }

    void drive_progress() {
        for (auto& d : dps) {
            DeviceGuard g(d.dp->capabilities().bound_accel_id);
            ProgressBudget b{64, 0};
            (void)d.dp->progress(b);
        }
        for (auto& e : ios)
            if (e.live) refresh(e);
    }

    std::size_t inflight_ios() const {
        std::size_t n = 0;
        for (auto& e : ios)
            if (e.live && e.state == IoState::IN_FLIGHT) ++n;
        return n;
    }
};

StorageRuntime::StorageRuntime(std::unique_ptr<Impl> impl) : impl_(std::move(impl)) {}

StorageRuntime::~StorageRuntime() {
    if (impl_ && impl_->state != RuntimeState::STOPPED) shutdown(1000);
}

static Status init_runtime(StorageRuntime::Impl& im, const RuntimeComponents& c) {
    for (auto& r : c.resolvers) {
        if (r.scheme.empty() || !r.resolver) return {StatusCode::INVALID_ARGUMENT, "bad resolver binding"};
        if (im.resolvers.count(r.scheme)) return {StatusCode::INVALID_ARGUMENT, "duplicate scheme " + r.scheme};
        im.resolvers[r.scheme] = r.resolver;
    }
    for (auto& d : c.data_paths) {
        if (d.key.empty() || !d.data_path) return {StatusCode::INVALID_ARGUMENT, "bad DataPath binding"};
        if (im.dp(d.key)) return {StatusCode::INVALID_ARGUMENT, "duplicate DataPath key " + d.key};
        const auto& caps = d.data_path->capabilities();
        if (caps.supports_device_execution && caps.bound_accel_id >= 0 && caps.bound_accel_id != im.cfg.accel_id)
            return {StatusCode::INVALID_ARGUMENT, "DataPath " + d.key + " is bound to another accelerator"};
        im.dps.push_back({d.key, d.data_path, d.config});
    }
    std::vector<DataPath*> inited;
    for (auto& d : im.dps) {
        DeviceGuard g(d.dp->capabilities().bound_accel_id);
        Status s = d.dp->initialize(d.config, c.resources);
        if (!s.ok()) {
            for (auto* x : inited) x->shutdown(0);
            return Status(s.code(), "DataPath " + d.key + ": " + s.message());
        }
        inited.push_back(d.dp);
    }
    return Status::Ok();
}

Result<std::unique_ptr<StorageRuntime>> StorageRuntime::create(const RuntimeConfig& config,
                                                               const RuntimeComponents& components) {
    auto im = std::make_unique<Impl>();
    im->cfg = config;
    im->id = g_runtime_ids.fetch_add(1);
    Status s = init_runtime(*im, components);
    if (!s.ok()) return Result<std::unique_ptr<StorageRuntime>>::Failure(s);
    return std::unique_ptr<StorageRuntime>(new StorageRuntime(std::move(im)));
}

Result<std::unique_ptr<StorageRuntime>> StorageRuntime::create_owning(const RuntimeConfig& config,
                                                                      OwnedComponents components) {
    auto im = std::make_unique<Impl>();
    im->cfg = config;
    im->id = g_runtime_ids.fetch_add(1);
    RuntimeComponents c;
    for (auto& r : components.resolvers) c.resolvers.push_back({r.scheme, r.resolver.get()});
    for (auto& d : components.data_paths) c.data_paths.push_back({d.key, d.data_path.get(), d.config});
    c.resources = components.resources.get();
    im->owned = std::move(components);
    Status s = init_runtime(*im, c);
    if (!s.ok()) return Result<std::unique_ptr<StorageRuntime>>::Failure(s);
    return std::unique_ptr<StorageRuntime>(new StorageRuntime(std::move(im)));
}

std::unique_ptr<StorageRuntime> StorageRuntime::create_stub(const RuntimeConfig& config) {
    auto im = std::make_unique<Impl>();
    im->cfg = config;
    im->id = g_runtime_ids.fetch_add(1);
    im->stub = true;
    return std::unique_ptr<StorageRuntime>(new StorageRuntime(std::move(im)));
}

namespace {
constexpr std::uint64_t kStubTargetBytes = 1ull << 30;
}

Status StorageRuntime::testing_force_complete(const IoHandle& h, IoState terminal, Status io_status) {
    auto& im = *impl_;
    std::lock_guard<std::mutex> g(im.mu);
    if (!im.stub) return {StatusCode::UNSUPPORTED, "only a stub runtime's IO can be forced terminal"};
    auto* e = im.io(h);
    if (!e) return {StatusCode::NOT_FOUND, "unknown IO handle"};
    if (terminal != IoState::COMPLETED && terminal != IoState::FAILED)
        return {StatusCode::INVALID_ARGUMENT, "terminal state must be COMPLETED or FAILED"};
    if (e->state != IoState::IN_FLIGHT) return {StatusCode::INVALID_ARGUMENT, "IO is already terminal"};
    IoResult res;
    res.state = terminal;
    if (terminal == IoState::FAILED) {
        res.status = io_status.ok() ? Status(StatusCode::INTERNAL, "forced failure") : io_status;
        res.detail.failure_kind = IoFailureKind::UNKNOWN;
        res.detail.failure_scope = IoFailureScope::WHOLE_OPERATION;
        res.detail.failed_request_indices = e->stub_requests;
        if (!e->stub_requests.empty()) res.detail.first_failed_entry = e->stub_requests.front();
    }
    e->result = std::move(res);
    e->state = terminal;
    ++im.terminal_unreleased;
    im.release_refs(*e);
    return Status::Ok();
}

RuntimeState StorageRuntime::state() const noexcept {
    std::lock_guard<std::mutex> g(impl_->mu);
    return impl_->state;
}

std::int32_t StorageRuntime::accel_id() const noexcept { return impl_->cfg.accel_id; }
std::uint32_t StorageRuntime::runtime_id() const noexcept { return impl_->id; }

Status StorageRuntime::shutdown(std::uint64_t timeout_ms) {
    auto& im = *impl_;
    std::unique_lock<std::mutex> lk(im.mu);
    if (im.state == RuntimeState::STOPPED) return Status::Ok();
    im.state = RuntimeState::DRAINING;
    const std::uint64_t deadline = now_ns() + timeout_ms * 1000000ull;
    while (im.inflight_ios() > 0 && now_ns() < deadline) {
        im.drive_progress();
        if (im.inflight_ios() == 0) break;
        lk.unlock();
        std::this_thread::sleep_for(std::chrono::microseconds(200));
        lk.lock();
    }
    if (im.inflight_ios() > 0)
        return {StatusCode::TIMEOUT, std::to_string(im.inflight_ios()) + " IO(s) still in flight"};
    for (auto& e : im.ios)
        if (e.live)
            for (auto& p : e.parts)
                if (auto* d = im.dp(p.dp_key)) d->dp->release(p.op);
    for (auto& m : im.mems)
        if (m.live)
            for (auto& r : m.regs)
                if (auto* d = im.dp(r.first)) d->dp->unregister_memory(r.second);
    for (auto& t : im.tgts)
        if (t.live)
            if (auto* d = im.dp(t.dp_key)) d->dp->close(t.dpt);
    for (auto it = im.dps.rbegin(); it != im.dps.rend(); ++it) {
        DeviceGuard g(it->dp->capabilities().bound_accel_id);
        it->dp->shutdown(timeout_ms * 1000000ull);
    }
    for (auto& m : im.mems) {
        if (m.live && m.runtime_owned && m.view.address) {
            if (m.view.expected_kind == MemoryKind::DEVICE)
                cudaFree(m.view.address);
            else if (m.view.expected_kind == MemoryKind::PINNED_HOST)
                cudaFreeHost(m.view.address);
            else
                std::free(m.view.address);
        }
    }
    im.mems.clear();
    im.tgts.clear();
    im.ios.clear();
    im.state = RuntimeState::STOPPED;
    return Status::Ok();
}

Result<std::vector<DeviceInfo>> StorageRuntime::list_devices() const {
    std::vector<DeviceInfo> out;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return out;
    }
    for (int i = 0; i < n; ++i) {
        cudaDeviceProp p{};
        if (cudaGetDeviceProperties(&p, i) != cudaSuccess) continue;
        char bdf[32];
        std::snprintf(bdf, sizeof(bdf), "%04x:%02x:%02x.0", p.pciDomainID, p.pciBusID, p.pciDeviceID);
        out.push_back({i, p.name, static_cast<std::uint64_t>(p.totalGlobalMem), bdf});
    }
    return out;
}

Result<DeviceCapabilities> StorageRuntime::query_device_capabilities(std::int32_t accel) const {
    auto devs = list_devices();
    DeviceCapabilities c;
    c.accel_id = accel;
    for (auto& d : devs.value())
        if (d.accel_id == accel) c.pci_bdf = d.pci_bdf;
    std::lock_guard<std::mutex> g(impl_->mu);
    for (auto& d : impl_->dps) {
        const auto& k = d.dp->capabilities();
        c.supports_device_execution |= k.supports_device_execution;
        c.max_io_size = std::max(c.max_io_size, k.max_single_io_bytes);
    }
    return c;
}

std::vector<DataPathCapabilities> StorageRuntime::data_path_capabilities() const {
    std::lock_guard<std::mutex> g(impl_->mu);
    std::vector<DataPathCapabilities> v;
    for (auto& d : impl_->dps) v.push_back(d.dp->capabilities());
    return v;
}

Result<MemoryAllocation> StorageRuntime::allocate_memory(const MemorySpec& spec) {
    using R = Result<MemoryAllocation>;
    if (spec.size == 0) return R::Failure({StatusCode::INVALID_ARGUMENT, "size 0"});
    void* p = nullptr;
    switch (spec.kind) {
        case MemoryKind::DEVICE: {
            if (!cuda_ok()) return R::Failure({StatusCode::UNSUPPORTED, "no CUDA device"});
            DeviceGuard g(spec.accel_id >= 0 ? spec.accel_id : impl_->cfg.accel_id);
            if (cudaMalloc(&p, spec.size) != cudaSuccess) {
                cudaGetLastError();
                return R::Failure({StatusCode::RESOURCE_EXHAUSTED, "cudaMalloc failed"});
            }
            break;
        }
        case MemoryKind::PINNED_HOST:
            if (!cuda_ok()) return R::Failure({StatusCode::UNSUPPORTED, "no CUDA device"});
            if (cudaHostAlloc(&p, spec.size, cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) {
                cudaGetLastError();
                return R::Failure({StatusCode::RESOURCE_EXHAUSTED, "cudaHostAlloc failed"});
            }
            break;
        case MemoryKind::HOST:
            if (posix_memalign(&p, 4096, spec.size) != 0) return R::Failure({StatusCode::RESOURCE_EXHAUSTED, "oom"});
            break;
        default:
            return R::Failure({StatusCode::UNSUPPORTED, "managed allocation not supported"});
    }
    MemoryView v;
    v.address = p;
    v.size = spec.size;
    v.expected_kind = spec.kind;
    v.ownership = MemoryOwnership::RUNTIME_OWNED;
    v.expected_accel_id = spec.kind == MemoryKind::DEVICE ? (spec.accel_id >= 0 ? spec.accel_id : impl_->cfg.accel_id) : -1;
    auto h = register_memory(v);
    if (!h.ok()) {
        if (spec.kind == MemoryKind::DEVICE)
            cudaFree(p);
        else if (spec.kind == MemoryKind::PINNED_HOST)
            cudaFreeHost(p);
        else
            std::free(p);
        return R::Failure(h.status());
    }
    {
        std::lock_guard<std::mutex> g(impl_->mu);
        impl_->mem(h.value())->runtime_owned = true;
    }
    return MemoryAllocation{h.value(), p, spec.size};
}

Status StorageRuntime::free_memory(const MemoryHandle& h) {
    void* addr = nullptr;
    MemoryKind kind;
    {
        std::lock_guard<std::mutex> g(impl_->mu);
        auto* m = impl_->mem(h);
        if (!m) return {StatusCode::NOT_FOUND, "unknown memory handle"};
        if (!m->runtime_owned) return {StatusCode::INVALID_ARGUMENT, "memory is caller-owned; use unregister_memory"};
        addr = m->view.address;
        kind = m->view.expected_kind;
    }
    TUTTI_RETURN_IF_ERROR(unregister_memory(h));
    if (kind == MemoryKind::DEVICE)
        cudaFree(addr);
    else if (kind == MemoryKind::PINNED_HOST)
        cudaFreeHost(addr);
    else
        std::free(addr);
    return Status::Ok();
}

Result<MemoryHandle> StorageRuntime::register_memory(const MemoryView& view) {
    using R = Result<MemoryHandle>;
    auto& im = *impl_;
    std::lock_guard<std::mutex> g(im.mu);
    if (im.state != RuntimeState::RUNNING) return R::Failure({StatusCode::NOT_READY, "runtime is not running"});
    if (!view.address || view.size == 0) return R::Failure({StatusCode::INVALID_ARGUMENT, "empty memory view"});
    if (!view.expected_profile.empty() && view.expected_profile != im.cfg.profile_name)
        return R::Failure({StatusCode::INVALID_ARGUMENT, "profile mismatch"});
    if (view.expected_kind == MemoryKind::DEVICE && cuda_ok()) {
        cudaPointerAttributes a{};
        if (cudaPointerGetAttributes(&a, view.address) != cudaSuccess) {
            cudaGetLastError();
            return R::Failure({StatusCode::INVALID_ARGUMENT, "address is not device memory"});
        }
        if (a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged)
            return R::Failure({StatusCode::INVALID_ARGUMENT, "address is not device memory"});
        // Memory imported through CUDA IPC reports the importing device, not the
        // one it lives on: a caller that names a peer device is taken at its word
        // (the data path then checks that the peer is reachable).
        if (view.expected_accel_id >= 0 && a.device != view.expected_accel_id &&
            !(view.expected_accel_id != im.cfg.accel_id && a.device == im.cfg.accel_id))
            return R::Failure({StatusCode::INVALID_ARGUMENT, "device memory belongs to another accelerator"});
    }
    // Overlapping registrations are refused: one owner per byte.
    const char* lo = static_cast<const char*>(view.address);
    for (auto& m : im.mems) {
        if (!m.live) continue;
        const char* mlo = static_cast<const char*>(m.view.address);
        if (lo < mlo + m.view.size && mlo < lo + view.size)
            return R::Failure({StatusCode::INVALID_ARGUMENT, "memory overlaps an existing registration"});
    }
    const std::uint32_t slot = Impl::alloc_slot(im.mems);
    auto& e = im.mems[slot];
    e = Impl::MemoryEntry{};
    e.generation = im.next_gen++;
    e.view = view;
    e.live = true;
    // Register eagerly with every DataPath that accepts this kind of memory.
    for (auto& d : im.dps) {
        auto r = im.registration_for(e, d);
        (void)r;
    }
    return MemoryHandle::from_raw(im.id, slot, e.generation);
}

Status StorageRuntime::unregister_memory(const MemoryHandle& h) {
    auto& im = *impl_;
    std::lock_guard<std::mutex> g(im.mu);
    auto* m = im.mem(h);
    if (!m) return {StatusCode::NOT_FOUND, "unknown memory handle"};
    if (m->inflight > 0) return {StatusCode::BUSY, "memory has IO in flight"};
    for (auto& r : m->regs)
        if (auto* d = im.dp(r.first)) d->dp->unregister_memory(r.second);
    m->regs.clear();
    m->live = false;
    return Status::Ok();
}

Result<MemoryInfo> StorageRuntime::query_memory(const MemoryHandle& h) const {
    auto& im = *impl_;
    std::lock_guard<std::mutex> g(im.mu);
    auto* m = const_cast<Impl&>(im).mem(h);
    if (!m) return Result<MemoryInfo>::Failure({StatusCode::NOT_FOUND, "unknown memory handle"});
    MemoryInfo i;
    i.kind = m->view.expected_kind;
    i.ownership = m->runtime_owned ? MemoryOwnership::RUNTIME_OWNED : MemoryOwnership::CALLER_OWNED;
    i.size = m->view.size;
    i.address = m->view.address;
    i.accel_id = m->view.expected_accel_id;
    i.inflight_count = m->inflight;
    return i;
}

Result<TargetHandle> StorageRuntime::open(std::string_view uri, const OpenOptions& o) {
    auto v = open_batch({std::string(uri)}, o);
    return std::move(v[0]);
}

std::vector<Result<TargetHandle>> StorageRuntime::open_batch(const std::vector<std::string>& uris,
                                                             const OpenOptions& o) {
    using R = Result<TargetHandle>;
    auto& im = *impl_;
    std::vector<R> out;
    out.reserve(uris.size());
    std::vector<std::optional<Result<ResolvedTarget>>> resolved(uris.size());
    std::vector<StorageTargetResolver*> rs(uris.size(), nullptr);
    {
        std::lock_guard<std::mutex> g(im.mu);
        if (im.state != RuntimeState::RUNNING) {
            for (std::size_t i = 0; i < uris.size(); ++i)
                out.push_back(R::Failure({StatusCode::NOT_READY, "runtime is not running"}));
            return out;
        }
        if (im.stub) {
            for (const auto& u : uris) {
                const std::uint32_t slot = Impl::alloc_slot(im.tgts);
                auto& t = im.tgts[slot];
                t = Impl::TargetEntry{};
                t.generation = im.next_gen++;
                t.live = true;
                t.uri = u;
                t.size = kStubTargetBytes;
                out.push_back(TargetHandle::from_raw(im.id, slot, t.generation));
            }
            return out;
        }
        for (std::size_t i = 0; i < uris.size(); ++i) {
            auto it = im.resolvers.find(scheme_of(uris[i], o));
            if (it != im.resolvers.end()) rs[i] = it->second;
        }
    }
    // Resolution (open + fsync + FIEMAP) in parallel without the registry lock.
    std::atomic<std::size_t> next{0};
    auto work = [&] {
        for (std::size_t i = next.fetch_add(1); i < uris.size(); i = next.fetch_add(1)) {
            if (!rs[i]) {
                resolved[i] = Result<ResolvedTarget>::Failure(
                    {StatusCode::NOT_FOUND, "no resolver for scheme of " + uris[i]});
                continue;
            }
            resolved[i] = rs[i]->resolve(uris[i], ResolveOptions{scheme_of(uris[i], o)});
        }
    };
    const std::size_t nthreads = std::min<std::size_t>(std::max<std::uint32_t>(1, im.cfg.open_batch_threads),
                                                       uris.size());
    if (nthreads <= 1) {
        work();
    } else {
        std::vector<std::thread> th;
        for (std::size_t t = 0; t < nthreads; ++t) th.emplace_back(work);
        for (auto& t : th) t.join();
    }
    std::lock_guard<std::mutex> g(im.mu);
    // One open_many per DataPath (it may share per-open costs across the batch),
    // then handles in input order.
    std::vector<Impl::DpEntry*> dps(uris.size(), nullptr);
    std::vector<std::optional<Result<DataPathTarget>>> opened(uris.size());
    std::vector<std::pair<Impl::DpEntry*, std::vector<std::size_t>>> by_dp;
    for (std::size_t i = 0; i < uris.size(); ++i) {
        auto& r = *resolved[i];
        if (!r.ok()) continue;
        std::string key(r.value().recommended_data_path_key());
        dps[i] = im.dp(key);
        if (!dps[i]) {
            opened[i] = Result<DataPathTarget>::Failure(
                {StatusCode::NOT_FOUND, "no DataPath registered for key '" + key + "'"});
            continue;
        }
        auto it = std::find_if(by_dp.begin(), by_dp.end(), [&](const auto& x) { return x.first == dps[i]; });
        if (it == by_dp.end()) {
            by_dp.push_back({dps[i], {}});
            it = by_dp.end() - 1;
        }
        it->second.push_back(i);
    }
    for (auto& [d, idx] : by_dp) {
        std::vector<const ResolvedTarget*> ts;
        ts.reserve(idx.size());
        for (auto i : idx) ts.push_back(&resolved[i]->value());
        DeviceGuard dg(d->dp->capabilities().bound_accel_id);
        auto res = d->dp->open_many(ts.data(), ts.size());
        for (std::size_t k = 0; k < idx.size(); ++k)
            opened[idx[k]] = k < res.size() ? std::move(res[k])
                                            : Result<DataPathTarget>::Failure({StatusCode::INTERNAL, "missing open"});
    }
    for (std::size_t i = 0; i < uris.size(); ++i) {
        auto& r = *resolved[i];
        if (!r.ok()) {
            out.push_back(R::Failure(r.status()));
            continue;
        }
        const ResolvedTarget& t = r.value();
        auto* d = dps[i];
        auto& dpt = *opened[i];
        if (!dpt.ok()) {
            out.push_back(R::Failure(dpt.status()));
            continue;
        }
        std::string key(t.recommended_data_path_key());
        const std::uint32_t slot = Impl::alloc_slot(im.tgts);
        auto& e = im.tgts[slot];
        e = Impl::TargetEntry{};
        e.generation = im.next_gen++;
        e.live = true;
        e.uri = uris[i];
        e.dp_key = key;
        e.dpe = d;
        e.dpt = dpt.value();
        e.size = t.logical_size();
        out.push_back(TargetHandle::from_raw(im.id, slot, e.generation));
    }
    return out;
}

Status StorageRuntime::close(const TargetHandle& h) {
    auto& im = *impl_;
    std::lock_guard<std::mutex> g(im.mu);
    auto* t = im.tgt(h);
    if (!t) return {StatusCode::NOT_FOUND, "unknown target handle"};
    if (t->inflight > 0) return {StatusCode::BUSY, "target has IO in flight"};
    if (auto* d = im.dp(t->dp_key)) d->dp->close(t->dpt);
    t->live = false;
    return Status::Ok();
}

Status StorageRuntime::close_batch(const std::vector<TargetHandle>& hs) {
    Status first;
    for (auto& h : hs) {
        Status s = close(h);
        if (!s.ok() && first.ok()) first = s;
    }
    return first;
}

Result<TargetInfo> StorageRuntime::query_target(const TargetHandle& h) const {
    auto& im = *impl_;
    std::lock_guard<std::mutex> g(im.mu);
    auto* t = const_cast<Impl&>(im).tgt(h);
    if (!t) return Result<TargetInfo>::Failure({StatusCode::NOT_FOUND, "unknown target handle"});
    return TargetInfo{t->uri, t->size, t->inflight, t->dp_key};
}

IoSubmitOutcome StorageRuntime::submit(const IoRequest* reqs, std::size_t count, const HostSubmitContext& ctx) {
    auto& im = *impl_;
    IoSubmitOutcome out;
    out.initial_states.resize(count);
    if (count == 0) return out;
    std::lock_guard<std::mutex> g(im.mu);
    auto reject_all = [&](Status s) {
        for (auto& st : out.initial_states) st = {IoRequestState::REJECTED, s};
        out.status = s;
        return out;
    };
    if (im.state != RuntimeState::RUNNING) return reject_all({StatusCode::NOT_READY, "runtime is not running"});
    if (!reqs) return reject_all({StatusCode::INVALID_ARGUMENT, "null requests"});
    if (ctx.accel_id >= 0 && ctx.accel_id != im.cfg.accel_id)
        return reject_all({StatusCode::INVALID_ARGUMENT, "context accel_id differs from the runtime's"});
    if (im.terminal_unreleased >= im.cfg.max_terminal_results)
        return reject_all({StatusCode::RESOURCE_EXHAUSTED, "too many unreleased terminal results; call release_io"});

    // Validate and group by DataPath (stable input order inside each group).
    struct Group {
        Impl::DpEntry* d;
        std::vector<DataPathRequest> reqs;
        std::vector<std::uint32_t> idx;
        std::uint64_t bytes = 0;
    };
    std::vector<Group> groups;
    groups.reserve(im.dps.size());
    Status first_reject;
    // Batches address few memories and targets: cache the last lookups so the
    // per-request cost is arithmetic, not registry searches.
    MemoryHandle last_mh;
    TargetHandle last_th;
    Impl::MemoryEntry* last_m = nullptr;
    Impl::TargetEntry* last_t = nullptr;
    Impl::MemoryEntry* reg_m = nullptr;
    Impl::DpEntry* reg_d = nullptr;
    DataPathMemory reg_dpm;
    Status reg_status;
    Impl::DpEntry* caps_d = nullptr;
    const DataPathCapabilities* caps = nullptr;
    Group* last_gp = nullptr;
    std::vector<std::uint32_t> mem_count(im.mems.size(), 0), tgt_count(im.tgts.size(), 0);
    const bool xform = ctx.transform != IoTransform::NONE;
    if (xform && ctx.transform != IoTransform::FP8_E4M3_BLOCK128)
        return reject_all({StatusCode::INVALID_ARGUMENT, "unknown IoTransform"});
    std::vector<std::uint32_t> stub_accepted;
    for (std::size_t i = 0; i < count; ++i) {
        const IoRequest& r = reqs[i];
        if (!last_m || r.memory != last_mh) {
            last_m = im.mem(r.memory);
            last_mh = r.memory;
        }
        if (!last_t || r.target != last_th) {
            last_t = im.tgt(r.target);
            last_th = r.target;
        }
        auto* m = last_m;
        auto* t = last_t;
        Status bad;
        if (!m)
            bad = {StatusCode::NOT_FOUND, "invalid memory handle"};
        else if (!t)
            bad = {StatusCode::NOT_FOUND, "invalid target handle"};
        else if (r.length == 0)
            bad = {StatusCode::INVALID_ARGUMENT, "zero length"};
        else if (r.memory_offset > m->view.size || r.length > m->view.size - r.memory_offset)
            bad = {StatusCode::OUT_OF_RANGE, "memory range exceeds registration"};
        else if (r.target_offset > t->size || stored_bytes(ctx.transform, r.length) > t->size - r.target_offset)
            bad = {StatusCode::OUT_OF_RANGE, "target range exceeds logical size"};
        else if (xform && (r.length % 1024 || r.target_offset % 16))
            bad = {StatusCode::INVALID_ARGUMENT, "fp8 block transform needs 1024-byte lengths, 16-byte target offsets"};
        if (im.stub) {  // no DataPath: accepted into an IO that waits for testing_force_complete
            if (!bad.ok()) {
                out.initial_states[i] = {IoRequestState::REJECTED, bad};
                if (first_reject.ok()) first_reject = bad;
            } else {
                out.initial_states[i] = {IoRequestState::ACCEPTED, Status::Ok()};
                stub_accepted.push_back(static_cast<std::uint32_t>(i));
                ++mem_count[r.memory.slot()];
                ++tgt_count[r.target.slot()];
            }
            continue;
        }
        Impl::DpEntry* d = nullptr;
        if (bad.ok()) {
            d = t->dpe;
            if (!d) bad = {StatusCode::INTERNAL, "target's DataPath missing"};
        }
        if (bad.ok()) {
            if (d != caps_d) {
                caps_d = d;
                caps = &d->dp->capabilities();
            }
            const auto& c = *caps;
            if ((r.direction == IoDirection::READ && !c.supports_read) ||
                (r.direction == IoDirection::WRITE && !c.supports_write))
                bad = {StatusCode::UNSUPPORTED, "direction not supported by " + d->key};
            else if ((ctx.execution_domain == ExecutionDomain::DEVICE_EXECUTION && !c.supports_device_execution) ||
                     (ctx.execution_domain == ExecutionDomain::HOST_EXECUTION && !c.supports_host_execution))
                bad = {StatusCode::UNSUPPORTED, "execution domain not supported by " + d->key};
            else if (xform && !c.supports_fp8_block_transform)
                bad = {StatusCode::UNSUPPORTED, d->key + " cannot apply the fp8 block transform"};
            else if ((!xform && (r.target_offset % c.target_alignment_bytes || r.length % c.length_alignment_bytes)) ||
                     (reinterpret_cast<std::uintptr_t>(m->view.address) + r.memory_offset) % c.memory_alignment_bytes)
                bad = {StatusCode::INVALID_ARGUMENT, "alignment violates " + d->key + " capabilities"};
            else if (c.max_single_io_bytes && r.length > c.max_single_io_bytes)
                bad = {StatusCode::INVALID_ARGUMENT, "request exceeds max_single_io_bytes"};
        }
        DataPathMemory dpm;
        if (bad.ok()) {
            if (m != reg_m || d != reg_d) {
                auto reg = im.registration_for(*m, *d);
                reg_m = m;
                reg_d = d;
                reg_status = reg.ok() ? Status::Ok() : reg.status();
                if (reg.ok()) reg_dpm = reg.value();
            }
            if (!reg_status.ok())
                bad = reg_status;
            else
                dpm = reg_dpm;
        }
        if (!bad.ok()) {
            out.initial_states[i] = {IoRequestState::REJECTED, bad};
            if (first_reject.ok()) first_reject = bad;
            continue;
        }
        Group* gp = (last_gp && last_gp->d == d) ? last_gp : nullptr;
        if (!gp) {
            for (auto& x : groups)
                if (x.d == d) gp = &x;
            if (!gp) {
                groups.push_back({d, {}, {}, 0});
                gp = &groups.back();
                gp->reqs.reserve(count);
                gp->idx.reserve(count);
            }
            last_gp = gp;
        }
        // The DataPath's batch width is a hard limit: requests past it are rejected
        // as exhausted (resubmit them), the rest of the batch proceeds.
        const auto& wc = *caps;
        if ((wc.max_batch_requests && gp->reqs.size() >= wc.max_batch_requests) ||
            (wc.max_batch_bytes && gp->bytes + r.length > wc.max_batch_bytes)) {
            const Status full{StatusCode::RESOURCE_EXHAUSTED, "batch width of " + d->key + " reached; resubmit"};
            out.initial_states[i] = {IoRequestState::REJECTED, full};
            if (first_reject.ok()) first_reject = full;
            continue;
        }
        gp->bytes += r.length;
        gp->reqs.push_back({r, dpm, t->dpt});
        gp->idx.push_back(static_cast<std::uint32_t>(i));
    }
    Impl::IoEntry entry;
    for (auto& gp : groups) {
        DeviceGuard dg(gp.d->dp->capabilities().bound_accel_id);
        SubmitOutcome so = gp.d->dp->submit(gp.reqs.data(), gp.reqs.size(), ctx);
        Impl::OpPart part;
        part.dp_key = gp.d->key;
        for (std::size_t k = 0; k < gp.reqs.size(); ++k) {
            auto& dst = out.initial_states[gp.idx[k]];
            if (k >= so.initial_states.size()) {
                dst = {IoRequestState::REJECTED, {StatusCode::INTERNAL, "missing state"}};
            } else if (so.initial_states[k].state == IoRequestState::ACCEPTED && so.initial_states[k].status.ok()) {
                dst.state = IoRequestState::ACCEPTED;  // the common case: no status to copy
            } else {
                dst = std::move(so.initial_states[k]);
            }
            if (dst.state == IoRequestState::REJECTED) {
                if (first_reject.ok()) first_reject = dst.status;
                continue;
            }
            const IoRequest& r = reqs[gp.idx[k]];
            ++mem_count[r.memory.slot()];
            ++tgt_count[r.target.slot()];
        }
        if (so.op) {
            part.op = *so.op;
            // DataPath request index k -> runtime request index
            part.input_index = gp.idx;
            entry.parts.push_back(std::move(part));
        }
    }
    out.status = first_reject;
    if (im.stub && !stub_accepted.empty()) {
        entry.stub = true;
        entry.stub_requests = std::move(stub_accepted);
    } else if (entry.parts.empty()) {
        return out;
    }
    for (std::uint32_t s = 0; s < mem_count.size(); ++s)
        if (mem_count[s]) {
            im.mems[s].inflight += static_cast<int>(mem_count[s]);
            entry.mem_refs.emplace_back(s, mem_count[s]);
        }
    for (std::uint32_t s = 0; s < tgt_count.size(); ++s)
        if (tgt_count[s]) {
            im.tgts[s].inflight += static_cast<int>(tgt_count[s]);
            entry.tgt_refs.emplace_back(s, tgt_count[s]);
        }
    const std::uint32_t slot = Impl::alloc_slot(im.ios);
    entry.generation = im.next_gen++;
    entry.live = true;
    im.ios[slot] = std::move(entry);
    out.io = IoHandle::from_raw(im.id, slot, im.ios[slot].generation);
    return out;
}

Result<IoSnapshot> StorageRuntime::query(const IoHandle& h) {
    auto& im = *impl_;
    std::lock_guard<std::mutex> g(im.mu);
    auto* e = im.io(h);
    if (!e) return Result<IoSnapshot>::Failure({StatusCode::NOT_FOUND, "unknown IO handle"});
    if (e->state == IoState::IN_FLIGHT) {
        im.drive_progress();
    }
    return IoSnapshot{e->state};
}

WaitOutcome StorageRuntime::wait(const IoHandle& h, std::uint64_t timeout_ms) {
    auto& im = *impl_;
    std::unique_lock<std::mutex> lk(im.mu);
    auto* e = im.io(h);
    if (!e) return {Status(StatusCode::NOT_FOUND, "unknown IO handle"), std::nullopt};
    const std::uint64_t deadline = now_ns() + timeout_ms * 1000000ull;
    std::uint32_t spins = 0;
    for (;;) {
        e = im.io(h);
        if (!e) return {Status(StatusCode::NOT_FOUND, "IO handle released while waiting"), std::nullopt};
        if (e->state == IoState::IN_FLIGHT) im.drive_progress();
        if (e->state != IoState::IN_FLIGHT) return {Status::Ok(), e->result};
        if (now_ns() >= deadline) return {Status(StatusCode::TIMEOUT, "IO still in flight"), std::nullopt};
        lk.unlock();
        if (++spins < 64)
            std::this_thread::yield();
        else
            std::this_thread::sleep_for(std::chrono::microseconds(20));
        lk.lock();
    }
}

Result<IoResult> StorageRuntime::wait_detail(const IoHandle& h, std::uint64_t timeout_ms) {
    auto w = wait(h, timeout_ms);
    if (!w.observation_status.ok()) return Result<IoResult>::Failure(w.observation_status);
    return *w.result;
}

Status StorageRuntime::enqueue_wait(const IoHandle* hs, std::size_t count, cudaStream_t stream) {
    auto& im = *impl_;
    std::lock_guard<std::mutex> g(im.mu);
    for (std::size_t i = 0; i < count; ++i) {
        auto* e = im.io(hs[i]);
        if (!e) return {StatusCode::NOT_FOUND, "unknown IO handle"};
        for (auto& p : e->parts) {
            auto* d = im.dp(p.dp_key);
            if (!d) continue;
            auto* ac = dynamic_cast<AsyncCompletion*>(d->dp);
            if (!ac) return {StatusCode::UNSUPPORTED, d->key + " has no device-side completion wait"};
            DeviceGuard dg(d->dp->capabilities().bound_accel_id);
            TUTTI_RETURN_IF_ERROR(ac->enqueue_wait(&p.op, 1, stream));
        }
    }
    return Status::Ok();
}

Status StorageRuntime::release_io(const IoHandle& h) {
    auto& im = *impl_;
    std::lock_guard<std::mutex> g(im.mu);
    auto* e = im.io(h);
    if (!e) return {StatusCode::NOT_FOUND, "unknown IO handle"};
    if (e->state == IoState::IN_FLIGHT) im.refresh(*e);
    if (e->state == IoState::IN_FLIGHT) return {StatusCode::BUSY, "IO still in flight"};
    for (auto& p : e->parts)
        if (auto* d = im.dp(p.dp_key)) d->dp->release(p.op);
    im.release_refs(*e);
    if (im.terminal_unreleased > 0) --im.terminal_unreleased;
    e->live = false;
    e->parts.clear();
    return Status::Ok();
}

Result<DataPathTarget> StorageRuntime::data_path_target(const TargetHandle& h) const {
    std::lock_guard<std::mutex> g(impl_->mu);
    auto* t = const_cast<Impl&>(*impl_).tgt(h);
    if (!t) return Result<DataPathTarget>::Failure({StatusCode::NOT_FOUND, "unknown target handle"});
    return t->dpt;
}

std::size_t StorageRuntime::unreleased_terminal_results() const {
    std::lock_guard<std::mutex> g(impl_->mu);
    return impl_->terminal_unreleased;
}

}  // namespace tutti
