#include "fake_snvme.h"

#include <algorithm>
#include <cerrno>
#include <cstdio>
#include <cstring>

namespace tutti {
namespace testing {

namespace uapi = snvme::uapi;

Result<std::unique_ptr<FakeSnvmeDriver>> FakeSnvmeDriver::create(const FakeSnvmeConfig& cfg) {
    using R = Result<std::unique_ptr<FakeSnvmeDriver>>;
    std::unique_ptr<FakeSnvmeDriver> d(new FakeSnvmeDriver(cfg));
    nvme::EmulatedControllerConfig hw = cfg.drive;
    hw.driver_created_queues = true;
    if (hw.queue_depth > 65535) return R::Failure({StatusCode::INVALID_ARGUMENT, "queue depth beyond CAP.MQES"});
    auto drive = nvme::EmulatedNvmeController::create(hw);
    if (!drive.ok()) return R::Failure(drive.status());
    d->drive_ = std::move(drive).value();
    d->qid_used_.assign(hw.num_io_queues + 1, false);
    if (cfg.owner_mode) d->node_created_ = d->bound_ = false;
    return R(std::move(d));
}

FakeSnvmeDriver::~FakeSnvmeDriver() {
    std::lock_guard<std::mutex> g(mu_);
    for (auto& kv : files_) release_file(kv.second);
    files_.clear();
    if (drive_) drive_->stop();
}

int FakeSnvmeDriver::open_node(const std::string& path) {
    std::lock_guard<std::mutex> g(mu_);
    const bool control = path == cfg_.control_node;
    if (!control && (path != cfg_.node || !node_created_)) return -ENOENT;
    const int fd = next_fd_++;
    File f;
    f.control = control;
    files_.emplace(fd, std::move(f));
    return fd;
}

int FakeSnvmeDriver::control_ioctl(unsigned long request, void* arg) {
    snvme::uapi::PciAddress a;
    std::memcpy(&a, arg, sizeof(a));
    char text[32];
    std::snprintf(text, sizeof(text), "%04x:%02x:%02x.%x", a.domain, a.bus, a.slot, a.function);
    if (cfg_.pci != text) return -ENODEV;
    switch (request) {
        case uapi::kChrdevCreate:
            if (node_created_) return -EEXIST;
            node_created_ = true;
            a.domain = cfg_.minor;  // the node's minor comes back in the domain field
            std::memcpy(arg, &a, sizeof(a));
            return 0;
        case uapi::kChrdevRemove:
            if (!node_created_) return -ENOENT;
            if (bound_) return -EBUSY;
            node_created_ = false;
            return 0;
        case uapi::kDeviceBind:
            if (!node_created_) return -ENODEV;
            if (bound_) return -EBUSY;
            bound_ = true;
            probe_polls_left_ = cfg_.probe_polls;
            return 0;
        case uapi::kDeviceUnbind:
            if (!bound_) return -EINVAL;
            bound_ = false;
            return 0;
        default:
            return -ENOTTY;
    }
}

int FakeSnvmeDriver::close_node(int fd) {
    std::lock_guard<std::mutex> g(mu_);
    auto it = files_.find(fd);
    if (it == files_.end()) return -EBADF;
    release_file(it->second);  // the close cascade
    files_.erase(it);
    return 0;
}

void FakeSnvmeDriver::fail_next(unsigned long request, int errno_value, std::uint32_t count) {
    std::lock_guard<std::mutex> g(mu_);
    fail_[request] = {errno_value, count};
}

int FakeSnvmeDriver::ioctl_node(int fd, unsigned long request, void* arg) {
    std::lock_guard<std::mutex> g(mu_);
    auto it = files_.find(fd);
    if (it == files_.end()) return -EBADF;
    auto f = fail_.find(request);
    if (f != fail_.end() && f->second.second > 0) {
        f->second.second -= 1;
        return -f->second.first;
    }
    if (!arg) return -EFAULT;
    File& file = it->second;
    if (file.control) return control_ioctl(request, arg);
    switch (request) {
        case uapi::kSetKernelIoqCap:
            if (bound_) return -EBUSY;  // a pre-bind hint
            kernel_ioq_cap_ = *static_cast<std::uint32_t*>(arg);
            return 0;
        case uapi::kGetDevInfo: return get_info(arg);
        case uapi::kCreateQueueGroup: return create_group(file, arg);
        case uapi::kDestroyQueueGroup: return destroy_group(file, *static_cast<std::uint32_t*>(arg));
        case uapi::kMapHostMemory: return map(file, arg, false);
        case uapi::kMapDeviceMemory: return map(file, arg, true);
        case uapi::kUnmapHostMemory: return unmap(file, *static_cast<std::uint64_t*>(arg), false);
        case uapi::kUnmapDeviceMemory: return unmap(file, *static_cast<std::uint64_t*>(arg), true);
        case uapi::kAddUserQueue: return add_queues(file, arg);
        default: return -ENOTTY;  // legacy and owner-side requests are not emulated
    }
}

int FakeSnvmeDriver::get_info(void* arg) {
    uapi::DevInfo di{};
    const nvme::ControllerInfo& hw = drive_->info();
    di.first_user_qid = cfg_.first_user_qid;
    di.last_user_qid = hw.num_io_queues;
    di.doorbell_stride_log = 0;
    di.max_transfer_bytes = hw.mdts_bytes;
    di.lba_bytes = hw.lba_bytes;
    // the disk is named once the driver is bound and its namespace scan ran
    if (bound_ && probe_polls_left_ == 0)
        std::snprintf(di.disk_name, sizeof(di.disk_name), "%sn1", hw.name.c_str());
    else if (bound_)
        --probe_polls_left_;
    di.queue_depth = static_cast<std::uint16_t>(hw.queue_depth);
    di.bar0_bytes = static_cast<std::uint32_t>(drive_->bar0_bytes());
    di.max_queues_per_group = cfg_.max_queues_per_group;
    di.abi_version = cfg_.abi_version;
    di.capabilities = cfg_.abi_version == 0 ? 0 : cfg_.capabilities;
    std::memcpy(arg, &di, sizeof(di));
    return 0;
}

int FakeSnvmeDriver::create_group(File& f, void* arg) {
    uapi::QueueGroup req;
    std::memcpy(&req, arg, sizeof(req));
    if (req.flags != 0) return -EINVAL;
    for (std::uint32_t v : req.mbz)
        if (v != 0) return -EINVAL;
    if (f.groups.size() >= uapi::kMaxGroupsPerFile) return -EBUSY;
    Group g;
    g.id = next_group_++;
    f.groups.push_back(g);
    req.group_id = g.id;
    req.max_queues = cfg_.max_queues_per_group;
    std::memcpy(arg, &req, sizeof(req));
    return 0;
}

int FakeSnvmeDriver::destroy_group(File& f, std::uint32_t id) {
    auto it = std::find_if(f.groups.begin(), f.groups.end(), [&](const Group& g) { return g.id == id; });
    if (it == f.groups.end()) return -ENOENT;
    for (std::uint32_t q : it->qids) {  // Delete I/O SQ + CQ
        (void)drive_->delete_io_queue_pair(q);
        qid_used_[q] = false;
    }
    for (const Mapping& m : it->rings) (void)drive_->unmap_window(m.va);
    f.groups.erase(it);
    return 0;
}

int FakeSnvmeDriver::map(File& f, void* arg, bool device) {
    uapi::MapRequest req;
    std::memcpy(&req, arg, sizeof(req));
    if (req.mbz[0] || req.mbz[1] || req.mbz[2]) return -EINVAL;
    if (req.kind > uapi::kMapData) return -EINVAL;
    const bool ring = req.kind == uapi::kMapRingSq || req.kind == uapi::kMapRingCq;
    if (ring && req.group_id == 0) return -EINVAL;
    if (req.n_pages == 0 || req.ioaddrs == 0) return -EINVAL;
    const std::uint64_t page = device ? uapi::kDeviceMapPage : uapi::kHostMapPage;
    if (req.vaddr % page != 0) return -EINVAL;
    if (ring && device) return -EOPNOTSUPP;  // the emulated drive reads rings with host threads
    Group* grp = nullptr;
    if (ring) {
        for (auto& g : f.groups)
            if (g.id == req.group_id) grp = &g;
        if (!grp) return -ENOENT;
    }
    const std::uint64_t bytes = req.n_pages * page;
    auto bus = drive_->map_window(reinterpret_cast<void*>(req.vaddr), bytes, device);
    if (!bus.ok()) return -ENOMEM;
    auto* out = reinterpret_cast<std::uint64_t*>(req.ioaddrs);
    for (std::uint64_t i = 0; i < req.n_pages; ++i) out[i] = bus.value() + i * page;
    Mapping m{req.vaddr, bytes, req.kind, device};
    if (grp)
        grp->rings.push_back(m);
    else
        f.data.push_back(m);
    return 0;
}

int FakeSnvmeDriver::unmap(File& f, std::uint64_t va, bool device) {
    auto it = std::find_if(f.data.begin(), f.data.end(),
                           [&](const Mapping& m) { return m.va == va && m.device == device; });
    if (it == f.data.end()) return -ENOENT;  // ring mappings go with their group
    (void)drive_->unmap_window(va);
    f.data.erase(it);
    return 0;
}

const FakeSnvmeDriver::Mapping* FakeSnvmeDriver::find_ring(const Group& g, std::uint64_t va, std::uint8_t kind) {
    for (const Mapping& m : g.rings)
        if (m.kind == kind && va >= m.va && va < m.va + m.bytes) return &m;
    return nullptr;
}

int FakeSnvmeDriver::add_queues(File& f, void* arg) {
    auto req = std::make_unique<uapi::AddUserQueues>();
    std::memcpy(req.get(), arg, sizeof(*req));
    if (req->flags != 0) return -EINVAL;
    for (std::uint32_t v : req->mbz)
        if (v != 0) return -EINVAL;
    Group* grp = nullptr;
    for (auto& g : f.groups)
        if (g.id == req->group_id) grp = &g;
    if (!grp) return -ENOENT;
    if (req->nr_pairs == 0 || req->nr_pairs > uapi::kMaxQueuesPerGroup) return -EINVAL;
    if (grp->qids.size() + req->nr_pairs > cfg_.max_queues_per_group) return -ENOSPC;
    const std::uint32_t depth = drive_->info().queue_depth;
    for (std::uint32_t i = 0; i < req->nr_pairs; ++i) {
        const uapi::QueueRings& r = req->rings[i];
        const Mapping* sq = find_ring(*grp, r.sq_vaddr, uapi::kMapRingSq);
        const Mapping* cq = find_ring(*grp, r.cq_vaddr, uapi::kMapRingCq);
        if (!sq || !cq) return -EINVAL;
        if (r.sq_vaddr + std::uint64_t(depth) * sizeof(nvme::Sqe) > sq->va + sq->bytes ||
            r.cq_vaddr + std::uint64_t(depth) * sizeof(nvme::Cqe) > cq->va + cq->bytes)
            return -EINVAL;  // the ring is shorter than the controller's queue depth
    }
    std::vector<std::uint32_t> got;
    for (std::uint32_t q = cfg_.first_user_qid; q < qid_used_.size() && got.size() < req->nr_pairs; ++q)
        if (!qid_used_[q]) got.push_back(q);
    if (got.size() < req->nr_pairs) return -ENOSPC;
    for (std::uint32_t i = 0; i < req->nr_pairs; ++i) {
        const uapi::QueueRings& r = req->rings[i];
        Status s = drive_->create_io_queue_pair(got[i], reinterpret_cast<void*>(r.sq_vaddr),
                                                reinterpret_cast<void*>(r.cq_vaddr), depth);
        if (!s.ok()) {
            for (std::uint32_t k = 0; k < i; ++k) {  // undo the pairs created so far
                (void)drive_->delete_io_queue_pair(got[k]);
                qid_used_[got[k]] = false;
            }
            return -EIO;
        }
        qid_used_[got[i]] = true;
        grp->qids.push_back(got[i]);
        req->out[i].qid = got[i];
        req->out[i].sq_tail_offset = nvme::sq_doorbell_offset(got[i]);
        req->out[i].cq_head_offset = nvme::cq_doorbell_offset(got[i]);
        req->out[i].mbz = 0;
    }
    std::memcpy(arg, req.get(), sizeof(*req));
    return 0;
}

void FakeSnvmeDriver::release_file(File& f) {
    while (!f.groups.empty()) (void)destroy_group(f, f.groups.back().id);
    for (const Mapping& m : f.data) (void)drive_->unmap_window(m.va);
    f.data.clear();
}

void* FakeSnvmeDriver::map_registers(int fd, std::size_t bytes) {
    std::lock_guard<std::mutex> g(mu_);
    if (!files_.count(fd) || bytes > drive_->bar0_bytes()) return nullptr;
    bar_maps_ += 1;
    return drive_->bar0_host();
}

void FakeSnvmeDriver::unmap_registers(void* p, std::size_t) {
    std::lock_guard<std::mutex> g(mu_);
    if (p == drive_->bar0_host() && bar_maps_ > 0) bar_maps_ -= 1;
}

Result<void*> FakeSnvmeDriver::register_registers(void* p, std::size_t) {
    // The emulated register file is already page-locked and mapped into the GPU.
    if (p != drive_->bar0_host()) return Result<void*>::Failure({StatusCode::INVALID_ARGUMENT, "not the BAR"});
    std::lock_guard<std::mutex> g(mu_);
    registered_ += 1;
    return Result<void*>(drive_->bar0_device() ? drive_->bar0_device() : drive_->bar0_host());
}

void FakeSnvmeDriver::unregister_registers(void* p) {
    std::lock_guard<std::mutex> g(mu_);
    if (p == drive_->bar0_host() && registered_ > 0) registered_ -= 1;
}

FakeSnvmeDriver::Counts FakeSnvmeDriver::counts() const {
    std::lock_guard<std::mutex> g(mu_);
    Counts c;
    c.files = static_cast<std::uint32_t>(files_.size());
    for (const auto& kv : files_) {
        c.groups += static_cast<std::uint32_t>(kv.second.groups.size());
        c.data_maps += static_cast<std::uint32_t>(kv.second.data.size());
        for (const auto& gr : kv.second.groups) {
            c.queues += static_cast<std::uint32_t>(gr.qids.size());
            c.ring_maps += static_cast<std::uint32_t>(gr.rings.size());
        }
    }
    c.bar_maps = bar_maps_;
    c.registered = registered_;
    c.node_created = node_created_;
    c.bound = bound_;
    c.kernel_ioq_cap = kernel_ioq_cap_;
    return c;
}

std::vector<std::uint32_t> FakeSnvmeDriver::live_qids() const {
    std::lock_guard<std::mutex> g(mu_);
    std::vector<std::uint32_t> out;
    for (std::uint32_t q = 0; q < qid_used_.size(); ++q)
        if (qid_used_[q]) out.push_back(q);
    return out;
}

}  // namespace testing
}  // namespace tutti
