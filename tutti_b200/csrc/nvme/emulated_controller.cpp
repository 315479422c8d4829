// Host-emulated NVMe controller: the "drive" side of the queue protocol.
//
// Each worker thread owns queues q with q % workers == worker, so a queue's
// head/tail/phase state has exactly one writer and needs no lock. A worker
// observes the SQ tail doorbell (acquire), copies each new SQE, executes it
// against the namespace's file-backed ranges into/out of the PRP-described
// host buffers, and posts a CQE whose dword 3 (CID, phase, status) is stored
// last with release semantics, which is the order a PCIe device's posted writes
// give a CQ poller.

#include "controller.h"

#include <fcntl.h>
#include <immintrin.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <sys/uio.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cstring>

namespace tutti {
namespace nvme {

namespace {
inline std::uint32_t load_acquire(const std::uint32_t* p) { return __atomic_load_n(p, __ATOMIC_ACQUIRE); }
inline void store_release(std::uint32_t* p, std::uint32_t v) { __atomic_store_n(p, v, __ATOMIC_RELEASE); }
}  // namespace

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
    std::unique_ptr<EmulatedNvmeController> c(new EmulatedNvmeController(cfg));
    Status st = c->start();
    if (!st.ok()) return R::Failure(st);
    return R(std::move(c));
}

Status EmulatedNvmeController::start() {
    const std::uint64_t nq = cfg_.num_io_queues, d = cfg_.queue_depth;
    auto sq = host_mapped_alloc(nq * d * sizeof(Sqe));
    if (!sq.ok()) return sq.status();
    sq_mem_ = sq.value();
    auto cq = host_mapped_alloc(nq * d * sizeof(Cqe));
    if (!cq.ok()) return cq.status();
    cq_mem_ = cq.value();
    auto bar = host_mapped_alloc(kDoorbellBase + 8 * nq);
    if (!bar.ok()) return bar.status();
    bar_mem_ = bar.value();
    for (std::uint32_t i = 0; i < nq; ++i) qstate_.emplace_back(new QueueState());
    std::uint32_t nw = std::max<std::uint32_t>(1, std::min(cfg_.worker_threads, cfg_.num_io_queues));
    for (std::uint32_t w = 0; w < nw; ++w) workers_.emplace_back([this, w] { worker_main(w); });
    return Status::Ok();
}

EmulatedNvmeController::~EmulatedNvmeController() {
    stop();
    for (auto& b : backings_) {
        if (b.map) ::munmap(const_cast<char*>(b.map), b.map_len);
        if (b.fd >= 0) ::close(b.fd);
    }
    host_mapped_free(sq_mem_);
    host_mapped_free(cq_mem_);
    host_mapped_free(bar_mem_);
}

void EmulatedNvmeController::stop() {
    stop_.store(true);
    for (auto& t : workers_)
        if (t.joinable()) t.join();
    workers_.clear();
}

static QueuePairView make_view(char* sq, char* cq, char* bar, std::uint32_t i, std::uint32_t depth,
                               std::uint32_t nsid) {
    QueuePairView v{};
    v.sq = reinterpret_cast<Sqe*>(sq) + std::uint64_t(i) * depth;
    v.cq = reinterpret_cast<const Cqe*>(cq) + std::uint64_t(i) * depth;
    v.sq_doorbell = reinterpret_cast<std::uint32_t*>(bar + sq_doorbell_offset(i));
    v.cq_doorbell = reinterpret_cast<std::uint32_t*>(bar + cq_doorbell_offset(i));
    v.depth = depth;
    v.qid = i + 1;  // queue 0 is the admin queue on a real controller
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

Result<std::uint64_t> EmulatedNvmeController::map_dma(void* host_ptr, std::uint64_t bytes) {
    if (!host_ptr || bytes == 0)
        return Result<std::uint64_t>::Failure({StatusCode::INVALID_ARGUMENT, "empty DMA window"});
    std::lock_guard<std::mutex> g(map_mu_);
    auto next = std::make_shared<std::vector<Window>>(*std::atomic_load(&windows_));
    next->push_back({reinterpret_cast<std::uint64_t>(host_ptr), bytes});
    std::atomic_store(&windows_, std::shared_ptr<const std::vector<Window>>(next));
    // The emulator's IOMMU is the identity: bus address == host virtual address.
    return reinterpret_cast<std::uint64_t>(host_ptr);
}

Status EmulatedNvmeController::unmap_dma(std::uint64_t iova) {
    std::lock_guard<std::mutex> g(map_mu_);
    auto next = std::make_shared<std::vector<Window>>(*std::atomic_load(&windows_));
    auto it = std::find_if(next->begin(), next->end(), [&](const Window& w) { return w.base == iova; });
    if (it == next->end()) return {StatusCode::NOT_FOUND, "no DMA window at that address"};
    next->erase(it);
    std::atomic_store(&windows_, std::shared_ptr<const std::vector<Window>>(next));
    return Status::Ok();
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
    return s;
}

Status EmulatedNvmeController::attach_file(const std::string& path, const std::vector<BackingRange>& ranges) {
    std::lock_guard<std::mutex> g(map_mu_);
    for (auto& b : backings_) {
        if (b.path == path) {
            // Same file: accept ranges already present, add new ones.
            for (const auto& r : ranges) {
                bool have = std::any_of(b.ranges.begin(), b.ranges.end(), [&](const BackingRange& x) {
                    return x.ns_offset == r.ns_offset && x.length == r.length && x.file_offset == r.file_offset;
                });
                if (!have) b.ranges.push_back(r);
            }
            goto rebuild;
        }
    }
    {
        int flags = O_RDWR | O_CLOEXEC;
        int fd = ::open(path.c_str(), flags | (cfg_.direct_io ? O_DIRECT : 0));
        if (fd < 0 && cfg_.direct_io) fd = ::open(path.c_str(), flags);  // e.g. tmpfs rejects O_DIRECT
        if (fd < 0) return {StatusCode::NOT_FOUND, "emulated namespace cannot open " + path};
        Backing nb{path, fd, ranges};
        if (!cfg_.direct_io && cfg_.map_reads) {
            // Page-cached mode: READs copy from a shared read-only mapping (the page
            // cache itself) instead of pread; WRITEs keep pwrite, which the mapping sees.
            struct stat st {};
            if (::fstat(fd, &st) == 0 && st.st_size > 0) {
                void* m = ::mmap(nullptr, static_cast<std::size_t>(st.st_size), PROT_READ, MAP_SHARED, fd, 0);
                if (m != MAP_FAILED) {
                    nb.map = static_cast<const char*>(m);
                    nb.map_len = static_cast<std::uint64_t>(st.st_size);
                }
            }
        }
        backings_.push_back(std::move(nb));
    }
rebuild: {
    auto spans = std::make_shared<std::vector<Span>>();
    for (auto& b : backings_)
        for (auto& r : b.ranges) spans->push_back({r.ns_offset, r.length, r.file_offset, b.fd, b.map, b.map_len});
    std::sort(spans->begin(), spans->end(), [](const Span& a, const Span& b) { return a.ns < b.ns; });
    for (std::size_t i = 1; i < spans->size(); ++i) {
        const Span& p = (*spans)[i - 1];
        const Span& c = (*spans)[i];
        if (p.ns + p.len > c.ns && !(p.ns == c.ns && p.fd == c.fd && p.foff == c.foff))
            return {StatusCode::INVALID_ARGUMENT, "namespace ranges overlap"};
    }
    // drop exact duplicates
    spans->erase(std::unique(spans->begin(), spans->end(),
                             [](const Span& a, const Span& b) { return a.ns == b.ns && a.fd == b.fd; }),
                 spans->end());
    std::atomic_store(&spans_, std::shared_ptr<const std::vector<Span>>(spans));
}
    return Status::Ok();
}

Status EmulatedNvmeController::detach_file(const std::string& path) {
    std::lock_guard<std::mutex> g(map_mu_);
    auto it = std::find_if(backings_.begin(), backings_.end(), [&](const Backing& b) { return b.path == path; });
    if (it == backings_.end()) return {StatusCode::NOT_FOUND, "not attached: " + path};
    // Keep the fd open (a worker may hold a span snapshot); clear its ranges.
    it->ranges.clear();
    auto spans = std::make_shared<std::vector<Span>>();
    for (auto& b : backings_)
        for (auto& r : b.ranges) spans->push_back({r.ns_offset, r.length, r.file_offset, b.fd, b.map, b.map_len});
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

bool EmulatedNvmeController::dma_ok(std::uint64_t addr, std::uint64_t bytes) const {
    auto w = std::atomic_load(&windows_);
    for (const auto& x : *w)
        if (addr >= x.base && addr + bytes <= x.base + x.bytes) return true;
    return false;
}

bool EmulatedNvmeController::collect_iov(std::uint64_t prp1, std::uint64_t prp2, std::uint64_t bytes,
                                         std::vector<std::pair<char*, std::uint64_t>>& iov) const {
    iov.clear();
    auto push = [&](std::uint64_t addr, std::uint64_t len) -> bool {
        if (!dma_ok(addr, len)) return false;
        char* p = reinterpret_cast<char*>(addr);
        if (!iov.empty() && iov.back().first + iov.back().second == p)
            iov.back().second += len;
        else
            iov.emplace_back(p, len);
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
    // PRP list: 8-byte entries; the last slot of a list page chains to the next page.
    if (prp2 & 7) return false;
    std::uint64_t list = prp2;
    std::uint64_t slots = (P - (list & (P - 1))) / 8;
    while (remaining > 0) {
        if (!dma_ok(list, 8)) return false;
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

std::uint32_t EmulatedNvmeController::execute(const Sqe& sqe, bool* drop_cqe) {
    *drop_cqe = false;
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
        std::lock_guard<std::mutex> g(map_mu_);
        for (auto& b : backings_)
            if (b.fd >= 0) ::fdatasync(b.fd);
        return 0;
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
    thread_local std::vector<std::pair<char*, std::uint64_t>> iov;
    if (!collect_iov(sqe.prp1, sqe.prp2, bytes, iov)) {
        st_errors_.fetch_add(1);
        return make_status(0, kScDataTransferError);
    }
    if (cfg_.skip_data) {
        (op == kOpRead ? st_read_ : st_write_).fetch_add(bytes, std::memory_order_relaxed);
        return 0;
    }
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
        std::uint64_t span_left = it->ns + it->len - pos;
        std::uint64_t chunk = std::min(span_left, end - pos);
        std::uint64_t foff = it->foff + (pos - it->ns);
        // issue chunk against the iov cursor (may cross iov segments)
        while (chunk > 0) {
            std::uint64_t seg_left = iov[seg].second - seg_off;
            std::uint64_t n = std::min(chunk, seg_left);
            char* buf = iov[seg].first + seg_off;
            std::uint64_t done = 0;
            if (op == kOpRead && it->map && foff + n <= it->map_len) {
                std::memcpy(buf, it->map + foff, n);
                done = n;
            }
            while (done < n) {
                ssize_t r = (op == kOpRead) ? ::pread(it->fd, buf + done, n - done, foff + done)
                                            : ::pwrite(it->fd, buf + done, n - done, foff + done);
                if (r < 0 && errno == EINTR) continue;
                if (r <= 0) {
                    if (op == kOpRead && r == 0) {  // past EOF of a backing file: zero fill
                        std::memset(buf + done, 0, n - done);
                        done = n;
                        break;
                    }
                    st_errors_.fetch_add(1);
                    return make_status(kSctMedia, kScUnrecoveredRead);
                }
                done += static_cast<std::uint64_t>(r);
            }
            chunk -= n;
            pos += n;
            foff += n;
            seg_off += n;
            if (seg_off == iov[seg].second) {
                ++seg;
                seg_off = 0;
            }
        }
        ++it;
    }
    if (op == kOpRead)
        st_read_.fetch_add(bytes, std::memory_order_relaxed);
    else
        st_write_.fetch_add(bytes, std::memory_order_relaxed);
    return 0;
}

bool EmulatedNvmeController::service_queue(std::uint32_t q) {
    QueueState& qs = *qstate_[q];
    QueuePairView v = host_queue(q);
    if (qs.reset_request.load(std::memory_order_acquire)) {
        qs.sq_head = 0;
        qs.cq_tail = 0;
        qs.phase = 1;
        std::memset(const_cast<Cqe*>(v.cq), 0, sizeof(Cqe) * v.depth);
        store_release(v.sq_doorbell, 0);
        store_release(v.cq_doorbell, 0);
        qs.fatal.store(0);
        qs.reset_request.store(0, std::memory_order_release);
        return true;
    }
    if (qs.fatal.load(std::memory_order_relaxed)) return false;
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
        bool drop = false;
        std::uint32_t status = execute(sqe, &drop);
        any = true;
        if (drop) continue;
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
        store_release(&slot->dw3, make_cqe_dw3(sqe_cid(sqe), qs.phase, status));
        qs.cq_tail = next;
        if (qs.cq_tail == 0) qs.phase ^= 1u;
        if (qs.sq_head == tail) tail = load_acquire(v.sq_doorbell);
    }
    return any;
}

void EmulatedNvmeController::worker_main(std::uint32_t worker) {
    const std::uint32_t nw = static_cast<std::uint32_t>(
        std::max<std::size_t>(1, std::min<std::size_t>(cfg_.worker_threads, cfg_.num_io_queues)));
    std::uint32_t idle = 0;
    while (!stop_.load(std::memory_order_relaxed)) {
        bool any = false;
        for (std::uint32_t q = worker; q < cfg_.num_io_queues; q += nw) any |= service_queue(q);
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
}

}  // namespace nvme
}  // namespace tutti
