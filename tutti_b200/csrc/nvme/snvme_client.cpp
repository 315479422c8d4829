#include "snvme_client.h"

#include <algorithm>
#include <cerrno>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <thread>

#include <fcntl.h>
#include <sys/mman.h>
#include <unistd.h>

#include <cuda_runtime.h>

namespace tutti {
namespace nvme {

namespace uapi = snvme::uapi;

namespace {

class LinuxSnvmeSys final : public SnvmeSys {
public:
    int open_node(const std::string& path) override {
        const int fd = ::open(path.c_str(), O_RDWR | O_CLOEXEC);
        return fd >= 0 ? fd : -errno;
    }
    int close_node(int fd) override { return ::close(fd) == 0 ? 0 : -errno; }
    int ioctl_node(int fd, unsigned long request, void* arg) override {
        return ::ioctl(fd, request, arg) == 0 ? 0 : -errno;
    }
    void* map_registers(int fd, std::size_t bytes) override {
        void* p = ::mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
        return p == MAP_FAILED ? nullptr : p;
    }
    void unmap_registers(void* p, std::size_t bytes) override { ::munmap(p, bytes); }
    Result<void*> register_registers(void* p, std::size_t bytes) override {
        using R = Result<void*>;
        if (cudaHostRegister(p, bytes, cudaHostRegisterIoMemory | cudaHostRegisterMapped) != cudaSuccess) {
            const char* why = cudaGetErrorString(cudaGetLastError());
            return R::Failure({StatusCode::UNSUPPORTED, std::string("cannot register BAR0 with CUDA: ") + why});
        }
        void* dev = nullptr;
        if (cudaHostGetDevicePointer(&dev, p, 0) != cudaSuccess) {
            cudaGetLastError();
            cudaHostUnregister(p);
            return R::Failure({StatusCode::UNSUPPORTED, "BAR0 has no device address"});
        }
        return R(dev);
    }
    void unregister_registers(void* p) override {
        if (cudaHostUnregister(p) != cudaSuccess) cudaGetLastError();
    }
    bool registers_are_mmio() const override { return true; }
};

Status errno_status(int neg_errno, const std::string& what) {
    const int e = -neg_errno;
    StatusCode code = StatusCode::INTERNAL;
    switch (e) {
        case ENOENT: case ENODEV: case ENXIO: code = StatusCode::NOT_FOUND; break;
        case EACCES: case EPERM: code = StatusCode::PERMISSION_DENIED; break;
        case EINVAL: case EFAULT: code = StatusCode::INVALID_ARGUMENT; break;
        case EBUSY: code = StatusCode::BUSY; break;
        case ENOSPC: case ENOMEM: code = StatusCode::RESOURCE_EXHAUSTED; break;
        case ENOTTY: case EOPNOTSUPP: code = StatusCode::UNSUPPORTED; break;
        case EEXIST: code = StatusCode::BUSY; break;
        default: break;
    }
    return {code, what + ": " + std::strerror(e)};
}

constexpr std::uint64_t round_up(std::uint64_t v, std::uint64_t a) { return (v + a - 1) / a * a; }

}  // namespace

SnvmeSys& linux_snvme_sys() {
    static LinuxSnvmeSys sys;
    return sys;
}

// ---- SnvmeClient -------------------------------------------------------------

Status SnvmeClient::ioctl(unsigned long request, void* arg, const char* what) {
    const int rc = sys_->ioctl_node(fd_, request, arg);
    return rc == 0 ? Status::Ok() : errno_status(rc, node_ + ": " + what);
}

Result<std::unique_ptr<SnvmeClient>> SnvmeClient::attach(const std::string& node, SnvmeSys& sys, bool for_gpu) {
    using R = Result<std::unique_ptr<SnvmeClient>>;
    std::unique_ptr<SnvmeClient> c(new SnvmeClient());
    c->sys_ = &sys;
    c->node_ = node;
    const int fd = sys.open_node(node);
    if (fd < 0) return R::Failure(errno_status(fd, "cannot open snvme node " + node));
    c->fd_ = fd;
    uapi::DevInfo di{};
    Status s = c->ioctl(uapi::kGetDevInfo, &di, "GET_DEV_INFO");
    if (!s.ok()) {
        if (s.code() == StatusCode::UNSUPPORTED)
            return R::Failure({StatusCode::UNSUPPORTED, node + " is not an snvme controller node"});
        return R::Failure(s);
    }
    // ABI handshake: the structures and ioctl numbers of this client are those of version 2.
    if (di.abi_version == 0)
        return R::Failure({StatusCode::UNSUPPORTED,
                           node + ": the snvme driver predates the ABI handshake; this client needs ABI " +
                               std::to_string(uapi::kAbiVersion)});
    if (di.abi_version != uapi::kAbiVersion)
        return R::Failure({StatusCode::UNSUPPORTED, node + ": snvme driver ABI " +
                                                                std::to_string(di.abi_version) + ", this client speaks " +
                                                                std::to_string(uapi::kAbiVersion)});
    if ((di.capabilities & uapi::kClientCaps) != uapi::kClientCaps)
        return R::Failure({StatusCode::UNSUPPORTED,
                           node + ": the snvme driver lacks queue groups, user queues or tagged mappings"});
    SnvmeDeviceInfo& in = c->info_;
    in.disk_name.assign(di.disk_name, strnlen(di.disk_name, sizeof(di.disk_name)));
    in.abi_version = di.abi_version;
    in.capabilities = di.capabilities;
    in.lba_bytes = static_cast<std::uint32_t>(di.lba_bytes);
    in.max_transfer_bytes = di.max_transfer_bytes;
    in.queue_depth = di.queue_depth;
    in.doorbell_stride = 4u << di.doorbell_stride_log;
    in.first_user_qid = di.first_user_qid;
    in.last_user_qid = di.last_user_qid;
    in.max_queues_per_group = std::min(di.max_queues_per_group, uapi::kMaxQueuesPerGroup);
    in.bar0_bytes = di.bar0_bytes;
    in.sgl = di.sgl_support != 0;
    if (in.lba_bytes < 512 || (in.lba_bytes & (in.lba_bytes - 1)) != 0)
        return R::Failure({StatusCode::INTERNAL, node + ": implausible logical block size"});
    if (in.queue_depth < 2 || in.max_queues_per_group == 0 || in.max_transfer_bytes < 4096)
        return R::Failure({StatusCode::INTERNAL, node + ": implausible queue limits"});
    if (di.doorbell_stride_log > 12 || in.bar0_bytes < 0x1000 + 2ull * in.doorbell_stride * (in.last_user_qid + 1))
        return R::Failure({StatusCode::INTERNAL, node + ": BAR0 does not hold the user queues' doorbells"});
    c->bar_ = sys.map_registers(fd, in.bar0_bytes);
    if (!c->bar_) return R::Failure({StatusCode::INTERNAL, node + ": cannot map BAR0"});
    if (for_gpu) {
        auto dev = sys.register_registers(c->bar_, in.bar0_bytes);
        if (!dev.ok()) return R::Failure(dev.status());
        c->bar_device_ = dev.value();
    }
    return R(std::move(c));
}

SnvmeClient::~SnvmeClient() {
    if (fd_ < 0) return;
    // Reverse order of creation; the driver would release the same on close.
    for (auto it = maps_.rbegin(); it != maps_.rend(); ++it) {
        if (it->group != 0) continue;  // ring mappings go with their group
        std::uint64_t va = it->va;
        (void)sys_->ioctl_node(fd_, it->where == SnvmeMemory::DEVICE ? uapi::kUnmapDeviceMemory : uapi::kUnmapHostMemory,
                               &va);
    }
    for (std::uint32_t g : groups_) (void)sys_->ioctl_node(fd_, uapi::kDestroyQueueGroup, &g);
    if (bar_device_) sys_->unregister_registers(bar_);
    if (bar_) sys_->unmap_registers(bar_, info_.bar0_bytes);
    sys_->close_node(fd_);
}

Result<std::uint32_t> SnvmeClient::create_group(std::uint32_t* max_queues) {
    using R = Result<std::uint32_t>;
    if (groups_.size() >= uapi::kMaxGroupsPerFile)
        return R::Failure({StatusCode::RESOURCE_EXHAUSTED, node_ + ": one queue group per open file"});
    uapi::QueueGroup g{};
    Status s = ioctl(uapi::kCreateQueueGroup, &g, "CREATE_QUEUE_GROUP");
    if (!s.ok()) return R::Failure(s);
    if (g.group_id == 0) return R::Failure({StatusCode::INTERNAL, node_ + ": driver returned queue group 0"});
    groups_.push_back(g.group_id);
    if (max_queues) *max_queues = std::min(g.max_queues, info_.max_queues_per_group);
    return R(g.group_id);
}

Status SnvmeClient::destroy_group(std::uint32_t group) {
    auto it = std::find(groups_.begin(), groups_.end(), group);
    if (it == groups_.end()) return {StatusCode::NOT_FOUND, node_ + ": no such queue group"};
    std::uint32_t g = group;
    Status s = ioctl(uapi::kDestroyQueueGroup, &g, "DESTROY_QUEUE_GROUP");
    if (!s.ok()) return s;
    groups_.erase(it);
    maps_.erase(std::remove_if(maps_.begin(), maps_.end(), [&](const Mapped& m) { return m.group == group; }),
                maps_.end());
    return Status::Ok();
}

Result<DmaMapping> SnvmeClient::map(void* p, std::uint64_t bytes, SnvmeMemory where, std::uint8_t kind,
                                    std::uint32_t group) {
    using R = Result<DmaMapping>;
    if (!p || bytes == 0) return R::Failure({StatusCode::INVALID_ARGUMENT, "empty DMA mapping"});
    const bool ring = kind == uapi::kMapRingSq || kind == uapi::kMapRingCq;
    if (ring && std::find(groups_.begin(), groups_.end(), group) == groups_.end())
        return R::Failure({StatusCode::INVALID_ARGUMENT, "ring mappings need a queue group of this file"});
    const std::uint64_t page = where == SnvmeMemory::DEVICE ? uapi::kDeviceMapPage : uapi::kHostMapPage;
    const auto a = reinterpret_cast<std::uint64_t>(p);
    const std::uint64_t va = a / page * page;
    const std::uint64_t n = (round_up(a + bytes, page) - va) / page;
    DmaMapping m;
    m.va = va;
    m.bytes = n * page;
    m.page_bytes = page;
    m.bus.assign(n, 0);
    m.kind = static_cast<int>(where);
    uapi::MapRequest req{};
    req.vaddr = va;
    req.n_pages = n;
    req.ioaddrs = reinterpret_cast<std::uint64_t>(m.bus.data());
    req.legacy_queue = -1;
    req.legacy_is_cq = -1;
    req.group_id = ring ? group : 0;
    req.kind = kind;
    Status s = ioctl(where == SnvmeMemory::DEVICE ? uapi::kMapDeviceMemory : uapi::kMapHostMemory, &req, "MAP_MEMORY");
    if (!s.ok()) return R::Failure(s);
    for (std::uint64_t b : m.bus)
        if (b == 0 || (b & (uapi::kHostMapPage - 1)) != 0) {
            std::uint64_t v = va;
            (void)sys_->ioctl_node(fd_, where == SnvmeMemory::DEVICE ? uapi::kUnmapDeviceMemory : uapi::kUnmapHostMemory,
                                   &v);
            return R::Failure({StatusCode::INTERNAL, node_ + ": driver returned an unaligned bus address"});
        }
    maps_.push_back({va, where, req.group_id});
    return R(std::move(m));
}

Status SnvmeClient::unmap(const DmaMapping& m) {
    auto it = std::find_if(maps_.begin(), maps_.end(), [&](const Mapped& x) { return x.va == m.va; });
    if (it == maps_.end()) return {StatusCode::NOT_FOUND, node_ + ": no mapping at that address"};
    std::uint64_t va = m.va;
    Status s = ioctl(it->where == SnvmeMemory::DEVICE ? uapi::kUnmapDeviceMemory : uapi::kUnmapHostMemory, &va,
                     "UNMAP_MEMORY");
    if (!s.ok()) return s;
    maps_.erase(it);
    return Status::Ok();
}

Result<std::vector<SnvmeQueue>> SnvmeClient::add_queues(std::uint32_t group,
                                                        const std::vector<uapi::QueueRings>& rings) {
    using R = Result<std::vector<SnvmeQueue>>;
    if (std::find(groups_.begin(), groups_.end(), group) == groups_.end())
        return R::Failure({StatusCode::INVALID_ARGUMENT, node_ + ": no such queue group"});
    if (rings.empty() || rings.size() > info_.max_queues_per_group)
        return R::Failure({StatusCode::INVALID_ARGUMENT, "1.." + std::to_string(info_.max_queues_per_group) +
                                                             " queue pairs per group"});
    auto req = std::make_unique<uapi::AddUserQueues>();
    std::memset(req.get(), 0, sizeof(*req));
    req->group_id = group;
    req->nr_pairs = static_cast<std::uint32_t>(rings.size());
    for (std::size_t i = 0; i < rings.size(); ++i) req->rings[i] = rings[i];
    Status s = ioctl(uapi::kAddUserQueue, req.get(), "ADD_USER_QUEUE");
    if (!s.ok()) return R::Failure(s);
    std::vector<SnvmeQueue> out(rings.size());
    for (std::size_t i = 0; i < rings.size(); ++i) {
        const uapi::QueueDoorbells& d = req->out[i];
        const auto in_bar = [&](std::uint32_t off) { return off >= 0x1000 && off % 4 == 0 && off + 4 <= info_.bar0_bytes; };
        if (!in_bar(d.sq_tail_offset) || !in_bar(d.cq_head_offset) || d.qid < info_.first_user_qid ||
            d.qid > info_.last_user_qid)
            return R::Failure({StatusCode::INTERNAL, node_ + ": driver returned doorbells outside BAR0"});
        out[i] = {d.qid, d.sq_tail_offset, d.cq_head_offset};
    }
    return R(std::move(out));
}

std::uint32_t* SnvmeClient::doorbell_host(std::uint32_t offset) const {
    return reinterpret_cast<std::uint32_t*>(static_cast<char*>(bar_) + offset);
}

std::uint32_t* SnvmeClient::doorbell_device(std::uint32_t offset) const {
    return bar_device_ ? reinterpret_cast<std::uint32_t*>(static_cast<char*>(bar_device_) + offset) : nullptr;
}

// ---- SnvmeOwner ----------------------------------------------------------------

Result<uapi::PciAddress> parse_pci_address(const std::string& text) {
    using R = Result<uapi::PciAddress>;
    unsigned dom = 0, bus = 0, slot = 0, fn = 0;
    char tail = 0;
    if (std::sscanf(text.c_str(), "%x:%x:%x.%x%c", &dom, &bus, &slot, &fn, &tail) != 4 || bus > 0xFF || slot > 0x1F ||
        fn > 7 || dom > 0xFFFF)
        return R::Failure({StatusCode::INVALID_ARGUMENT, "bad PCI address '" + text + "' (want dddd:bb:ss.f)"});
    uapi::PciAddress a{};
    a.domain = static_cast<std::int32_t>(dom);
    a.bus = static_cast<std::int32_t>(bus);
    a.slot = static_cast<std::int32_t>(slot);
    a.function = static_cast<std::int32_t>(fn);
    return R(a);
}

Result<std::unique_ptr<SnvmeOwner>> SnvmeOwner::bring_up(const std::string& control_node, const std::string& pci,
                                                         std::uint32_t kernel_ioq_cap, SnvmeSys& sys,
                                                         std::uint32_t probe_wait_ms) {
    using R = Result<std::unique_ptr<SnvmeOwner>>;
    auto addr = parse_pci_address(pci);
    if (!addr.ok()) return R::Failure(addr.status());
    std::unique_ptr<SnvmeOwner> o(new SnvmeOwner());
    o->sys_ = &sys;
    o->pci_ = addr.value();
    const int cfd = sys.open_node(control_node);
    if (cfd < 0) return R::Failure(errno_status(cfd, "cannot open the snvme control node " + control_node));
    o->control_fd_ = cfd;
    uapi::PciAddress a = o->pci_;
    if (int rc = sys.ioctl_node(cfd, uapi::kChrdevCreate, &a); rc != 0)
        return R::Failure(errno_status(rc, pci + ": CHRDEV_CREATE"));
    o->created_ = true;
    o->minor_ = a.domain;  // the driver returns the node's minor in the domain field
    o->node_ = "/dev/ssnvme" + std::to_string(o->minor_);
    const int dfd = sys.open_node(o->node_);
    if (dfd < 0) return R::Failure(errno_status(dfd, "cannot open " + o->node_));
    o->dev_fd_ = dfd;
    if (kernel_ioq_cap != 0) {
        std::uint32_t cap = kernel_ioq_cap;
        if (int rc = sys.ioctl_node(dfd, uapi::kSetKernelIoqCap, &cap); rc != 0)
            return R::Failure(errno_status(rc, o->node_ + ": SET_KERNEL_IOQ_CAP"));
    }
    a = o->pci_;
    if (int rc = sys.ioctl_node(cfd, uapi::kDeviceBind, &a); rc != 0)
        return R::Failure(errno_status(rc, pci + ": DEVICE_BIND"));
    o->bound_ = true;
    // The bind returns before the namespace scan: poll until the disk is named.
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(probe_wait_ms);
    for (;;) {
        uapi::DevInfo di{};
        const int rc = sys.ioctl_node(dfd, uapi::kGetDevInfo, &di);
        if (rc == 0 && di.disk_name[0] != 0) {
            if (di.abi_version != uapi::kAbiVersion)
                return R::Failure({StatusCode::UNSUPPORTED, o->node_ + ": snvme driver ABI " + std::to_string(di.abi_version) +
                                                                ", this build speaks " + std::to_string(uapi::kAbiVersion)});
            SnvmeDeviceInfo& in = o->info_;
            in.disk_name.assign(di.disk_name, strnlen(di.disk_name, sizeof(di.disk_name)));
            in.abi_version = di.abi_version;
            in.capabilities = di.capabilities;
            in.lba_bytes = static_cast<std::uint32_t>(di.lba_bytes);
            in.max_transfer_bytes = di.max_transfer_bytes;
            in.queue_depth = di.queue_depth;
            in.doorbell_stride = 4u << di.doorbell_stride_log;
            in.first_user_qid = di.first_user_qid;
            in.last_user_qid = di.last_user_qid;
            in.max_queues_per_group = std::min(di.max_queues_per_group, uapi::kMaxQueuesPerGroup);
            in.bar0_bytes = di.bar0_bytes;
            in.sgl = di.sgl_support != 0;
            break;
        }
        if (rc != 0 && rc != -EAGAIN && rc != -ENODEV) return R::Failure(errno_status(rc, o->node_ + ": GET_DEV_INFO"));
        if (std::chrono::steady_clock::now() >= deadline)
            return R::Failure({StatusCode::TIMEOUT, o->node_ + ": the namespace scan did not finish in " +
                                                        std::to_string(probe_wait_ms) + " ms"});
        std::this_thread::sleep_for(std::chrono::milliseconds(10));
    }
    return R(std::move(o));
}

SnvmeOwner::~SnvmeOwner() {
    if (dev_fd_ >= 0) sys_->close_node(dev_fd_);
    if (control_fd_ >= 0) {
        uapi::PciAddress a = pci_;
        if (bound_) (void)sys_->ioctl_node(control_fd_, uapi::kDeviceUnbind, &a);
        a = pci_;
        if (created_) (void)sys_->ioctl_node(control_fd_, uapi::kChrdevRemove, &a);
        sys_->close_node(control_fd_);
    }
}

// ---- SnvmeController -----------------------------------------------------------

Result<std::unique_ptr<SnvmeController>> SnvmeController::create(const SnvmeControllerConfig& cfg, SnvmeSys& sys) {
    using R = Result<std::unique_ptr<SnvmeController>>;
    if (cfg.num_io_queues == 0) return R::Failure({StatusCode::INVALID_ARGUMENT, "num_io_queues must be > 0"});
    std::unique_ptr<SnvmeController> c(new SnvmeController());
    c->sys_ = &sys;
    Status s = c->bring_up(cfg);
    if (!s.ok()) return R::Failure(s);
    return R(std::move(c));
}

Result<std::unique_ptr<SnvmeController>> SnvmeController::create(const SnvmeControllerConfig& cfg,
                                                                  std::shared_ptr<SnvmeSys> sys) {
    using R = Result<std::unique_ptr<SnvmeController>>;
    if (!sys) return R::Failure({StatusCode::INVALID_ARGUMENT, "no snvme system interface"});
    if (cfg.num_io_queues == 0) return R::Failure({StatusCode::INVALID_ARGUMENT, "num_io_queues must be > 0"});
    std::unique_ptr<SnvmeController> c(new SnvmeController());
    c->sys_owner_ = std::move(sys);
    c->sys_ = c->sys_owner_.get();
    Status s = c->bring_up(cfg);
    if (!s.ok()) return R::Failure(s);
    return R(std::move(c));
}

Status SnvmeController::bring_up(const SnvmeControllerConfig& cfg) {
    const bool gpu = cuda_device_present();
    if (gpu) {
        cuda_device_ = cfg.cuda_device;
        if (cuda_device_ < 0 && cudaGetDevice(&cuda_device_) != cudaSuccess) {
            cudaGetLastError();
            cuda_device_ = 0;
        }
        if (cudaSetDevice(cuda_device_) != cudaSuccess) {
            cudaGetLastError();
            return {StatusCode::UNSUPPORTED, "cannot select CUDA device " + std::to_string(cuda_device_)};
        }
    }
    if (cfg.rings_in_gpu_memory && !gpu) return {StatusCode::UNSUPPORTED, "rings in GPU memory need a CUDA device"};
    auto first = SnvmeClient::attach(cfg.node, *sys_, gpu);
    if (!first.ok()) return first.status();
    clients_.push_back(std::move(first).value());
    const SnvmeDeviceInfo di = clients_[0]->info();
    // The driver creates every user queue with the controller's depth (CAP.MQES
    // + 1, clamped), so the rings have exactly that many entries.
    const std::uint32_t depth = di.queue_depth;
    const std::uint32_t room = di.last_user_qid >= di.first_user_qid ? di.last_user_qid - di.first_user_qid + 1 : 0;
    if (cfg.num_io_queues > room)
        return {StatusCode::RESOURCE_EXHAUSTED, cfg.node + ": " + std::to_string(cfg.num_io_queues) +
                                                     " queue pairs asked, the driver hands out " + std::to_string(room)};
    // Ring memory: one region, each ring on its own mapping page.
    const std::uint64_t page = cfg.rings_in_gpu_memory ? uapi::kDeviceMapPage : uapi::kHostMapPage;
    const std::uint64_t sq_bytes = round_up(std::uint64_t(depth) * sizeof(Sqe), page);
    const std::uint64_t cq_bytes = round_up(std::uint64_t(depth) * sizeof(Cqe), page);
    const std::uint64_t per_queue = sq_bytes + cq_bytes;
    const std::uint64_t total = per_queue * cfg.num_io_queues;
    char* ring_host = nullptr;   // host address (host rings only)
    char* ring_dev = nullptr;    // device address
    if (cfg.rings_in_gpu_memory) {
        if (cudaMalloc(&device_rings_raw_, total + page) != cudaSuccess) {
            cudaGetLastError();
            return {StatusCode::RESOURCE_EXHAUSTED, "cannot allocate queue rings in GPU memory"};
        }
        ring_dev = reinterpret_cast<char*>(round_up(reinterpret_cast<std::uint64_t>(device_rings_raw_), page));
        if (cudaMemset(ring_dev, 0, total) != cudaSuccess) {
            cudaGetLastError();
            return {StatusCode::INTERNAL, "cannot clear the queue rings"};
        }
    } else {
        auto hb = host_mapped_alloc(total);
        if (!hb.ok()) return hb.status();
        host_rings_ = hb.value();
        ring_host = static_cast<char*>(host_rings_.host);
        ring_dev = static_cast<char*>(host_rings_.device);
    }
    char* const ring_va = cfg.rings_in_gpu_memory ? ring_dev : ring_host;  // what the driver pins
    const SnvmeMemory where = cfg.rings_in_gpu_memory ? SnvmeMemory::DEVICE : SnvmeMemory::HOST;
    device_views_.resize(cfg.num_io_queues);
    host_views_.resize(cfg.num_io_queues);
    std::uint32_t next = 0;
    while (next < cfg.num_io_queues) {
        if (next > 0) {  // another open file for the next group
            auto more = SnvmeClient::attach(cfg.node, *sys_, gpu);
            if (!more.ok()) return more.status();
            clients_.push_back(std::move(more).value());
        }
        SnvmeClient& cl = *clients_.back();
        std::uint32_t cap = 0;
        auto g = cl.create_group(&cap);
        if (!g.ok()) return g.status();
        group_of_client_.push_back(g.value());
        if (cap == 0) return {StatusCode::RESOURCE_EXHAUSTED, cfg.node + ": queue group without room for queues"};
        const std::uint32_t n = std::min(cap, cfg.num_io_queues - next);
        std::vector<uapi::QueueRings> rings(n);
        for (std::uint32_t k = 0; k < n; ++k) {
            char* sq = ring_va + std::uint64_t(next + k) * per_queue;
            char* cq = sq + sq_bytes;
            auto ms = cl.map(sq, sq_bytes, where, uapi::kMapRingSq, g.value());
            if (!ms.ok()) return ms.status();
            auto mc = cl.map(cq, cq_bytes, where, uapi::kMapRingCq, g.value());
            if (!mc.ok()) return mc.status();
            // Queues are created physically contiguous from the first bus address.
            for (const DmaMapping* m : {&ms.value(), &mc.value()})
                for (std::size_t pg = 1; pg < m->bus.size(); ++pg)
                    if (m->bus[pg] != m->bus[0] + pg * m->page_bytes)
                        return {StatusCode::UNSUPPORTED,
                                cfg.node + ": a queue ring spans pages that are not adjacent on the bus (put the "
                                           "rings in GPU memory, whose 64 KiB pages hold a whole ring)"};
            rings[k] = {reinterpret_cast<std::uint64_t>(sq), reinterpret_cast<std::uint64_t>(cq)};
        }
        auto qs = cl.add_queues(g.value(), rings);
        if (!qs.ok()) return qs.status();
        for (std::uint32_t k = 0; k < n; ++k) {
            const SnvmeQueue& q = qs.value()[k];
            const std::uint64_t off = std::uint64_t(next + k) * per_queue;
            QueuePairView dv{};
            if (ring_dev) {  // no device address without a GPU
                dv.sq = reinterpret_cast<Sqe*>(ring_dev + off);
                dv.cq = reinterpret_cast<const Cqe*>(ring_dev + off + sq_bytes);
            }
            dv.sq_doorbell = cl.doorbell_device(q.sq_tail_offset);
            dv.cq_doorbell = cl.doorbell_device(q.cq_head_offset);
            dv.depth = depth;
            dv.qid = q.qid;
            dv.nsid = cfg.nsid;
            dv.flags = cl.mmio_doorbells() ? kQueueMmioDoorbells : 0u;
            QueuePairView hv = dv;
            hv.sq = ring_host ? reinterpret_cast<Sqe*>(ring_host + off) : nullptr;
            hv.cq = ring_host ? reinterpret_cast<const Cqe*>(ring_host + off + sq_bytes) : nullptr;
            hv.sq_doorbell = cl.doorbell_host(q.sq_tail_offset);
            hv.cq_doorbell = cl.doorbell_host(q.cq_head_offset);
            device_views_[next + k] = dv;
            host_views_[next + k] = hv;
        }
        next += n;
    }
    info_.name = di.disk_name.empty() ? cfg.node : di.disk_name;
    info_.kind = "snvme";
    info_.lba_bytes = di.lba_bytes;
    const std::uint64_t mdts = std::min<std::uint64_t>(di.max_transfer_bytes, cfg.max_command_bytes);
    info_.mdts_bytes = static_cast<std::uint32_t>(mdts / 4096 * 4096);
    info_.queue_depth = depth;
    info_.num_io_queues = cfg.num_io_queues;
    info_.nsid = cfg.nsid;
    info_.namespace_bytes = cfg.namespace_bytes;
    info_.device_dma = gpu;
    return Status::Ok();
}

SnvmeController::~SnvmeController() {
    // Groups (and their queue pairs and ring mappings) first, then the files.
    for (std::size_t i = 0; i < clients_.size() && i < group_of_client_.size(); ++i)
        (void)clients_[i]->destroy_group(group_of_client_[i]);
    clients_.clear();
    host_mapped_free(host_rings_);
    if (device_rings_raw_) cudaFree(device_rings_raw_);
}

QueuePairView SnvmeController::device_queue(std::uint32_t i) const {
    return i < device_views_.size() ? device_views_[i] : QueuePairView{};
}

QueuePairView SnvmeController::host_queue(std::uint32_t i) const {
    return i < host_views_.size() ? host_views_[i] : QueuePairView{};
}

Result<DmaMapping> SnvmeController::map_dma(void* ptr, std::uint64_t bytes) {
    SnvmeMemory where = SnvmeMemory::HOST;
    if (cuda_device_ >= 0) {
        cudaPointerAttributes a{};
        if (cudaPointerGetAttributes(&a, ptr) == cudaSuccess) {
            if (a.type == cudaMemoryTypeDevice) where = SnvmeMemory::DEVICE;
        } else {
            cudaGetLastError();
        }
    }
    std::lock_guard<std::mutex> g(map_mu_);
    // Data mappings belong to an open file; every file of this controller sees
    // the same bus addresses, so the first one holds them.
    return clients_[0]->map(ptr, bytes, where, uapi::kMapData, 0);
}

Status SnvmeController::unmap_dma(const DmaMapping& m) {
    std::lock_guard<std::mutex> g(map_mu_);
    return clients_[0]->unmap(m);
}

Status SnvmeController::reset_queue(std::uint32_t i) {
    if (i >= device_views_.size()) return {StatusCode::OUT_OF_RANGE, "queue index"};
    return {StatusCode::UNSUPPORTED, "snvme queue pairs are deleted and created per group; queue " +
                                         std::to_string(device_views_[i].qid) + " stays out of service"};
}

}  // namespace nvme
}  // namespace tutti
