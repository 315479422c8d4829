#include "posix_data_path.h"

#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstring>

#include <cuda_runtime_api.h>

#include "../runtime/device_guard.h"

namespace tutti {

PosixDataPath::PosixDataPath(PosixConfig cfg) : cfg_(cfg) {
    caps_.name = "posix";
    caps_.source_api_version = 1;
    caps_.supports_host_execution = true;
    caps_.supports_device_execution = false;
    caps_.supports_host_memory = true;
    caps_.supports_device_memory = true;
    caps_.supports_direct = true;
    caps_.supports_staged = true;
    caps_.supports_read = true;
    caps_.supports_write = true;
    caps_.target_alignment_bytes = 1;
    caps_.memory_alignment_bytes = 1;
    caps_.length_alignment_bytes = 1;
    caps_.registration_scope = RegistrationScope::GLOBAL;
    caps_.progress_model = ProgressModel::HOST_POLL;
    caps_.supports_multi_stream = true;
    caps_.bound_accel_id = -1;
}

PosixDataPath::~PosixDataPath() { shutdown(0); }

Status PosixDataPath::initialize(const DataPathConfig&, ResourceProvider*) {
    std::lock_guard<std::mutex> g(mu_);
    if (initialized_) return {StatusCode::INVALID_ARGUMENT, "already initialized"};
    stop_ = false;
    for (std::uint32_t i = 0; i < std::max<std::uint32_t>(1, cfg_.threads); ++i)
        workers_.emplace_back([this] { worker(); });
    initialized_ = true;
    return Status::Ok();
}

Status PosixDataPath::shutdown(std::uint64_t) {
    {
        std::lock_guard<std::mutex> g(qmu_);
        stop_ = true;
    }
    qcv_.notify_all();
    for (auto& t : workers_)
        if (t.joinable()) t.join();
    workers_.clear();
    std::lock_guard<std::mutex> g(mu_);
    for (auto& kv : targets_) {
        if (kv.second.fd_direct >= 0) ::close(kv.second.fd_direct);
        if (kv.second.fd_buffered >= 0) ::close(kv.second.fd_buffered);
    }
    targets_.clear();
    initialized_ = false;
    return Status::Ok();
}

Result<DataPathTarget> PosixDataPath::open(const ResolvedTarget& t) {
    using R = Result<DataPathTarget>;
    auto pv = t.view<FileExtentPayload>(kFileExtentPayloadType, kFileExtentPayloadVersion);
    if (!pv.ok()) return R::Failure(pv.status());
    const auto& p = *pv.value();
    Target tg;
    tg.fd_buffered = ::open(p.path.c_str(), O_RDWR | O_CLOEXEC);
    if (tg.fd_buffered < 0) tg.fd_buffered = ::open(p.path.c_str(), O_RDONLY | O_CLOEXEC);
    if (tg.fd_buffered < 0) return R::Failure({StatusCode::NOT_FOUND, "open " + p.path + ": " + std::strerror(errno)});
    if (cfg_.direct_io) {
        tg.fd_direct = ::open(p.path.c_str(), O_RDWR | O_CLOEXEC | O_DIRECT);
        if (tg.fd_direct < 0) tg.fd_direct = ::open(p.path.c_str(), O_RDONLY | O_CLOEXEC | O_DIRECT);
    }
    tg.size = p.file_size;
    std::lock_guard<std::mutex> g(mu_);
    tg.gen = next_++;
    targets_[tg.gen] = tg;
    return DataPathTarget{tg.gen, tg.gen};
}

Status PosixDataPath::close(DataPathTarget t) {
    std::lock_guard<std::mutex> g(mu_);
    auto it = targets_.find(t.token);
    if (it == targets_.end()) return {StatusCode::NOT_FOUND, "unknown target"};
    if (it->second.fd_direct >= 0) ::close(it->second.fd_direct);
    if (it->second.fd_buffered >= 0) ::close(it->second.fd_buffered);
    targets_.erase(it);
    return Status::Ok();
}

Result<RegistrationDomainKey> PosixDataPath::registration_domain(DataPathTarget) const {
    return RegistrationDomainKey{"posix"};
}

Result<DataPathMemory> PosixDataPath::register_memory(const DataPathMemoryView& v, const RegistrationDomainKey&) {
    std::lock_guard<std::mutex> g(mu_);
    Mem m{next_++, static_cast<char*>(v.base), v.size_bytes, v.kind};
    mems_[m.gen] = m;
    return DataPathMemory{m.gen, m.gen};
}

Status PosixDataPath::unregister_memory(DataPathMemory m) {
    std::lock_guard<std::mutex> g(mu_);
    return mems_.erase(m.token) ? Status::Ok() : Status(StatusCode::NOT_FOUND, "unknown memory");
}

SubmitOutcome PosixDataPath::submit(const DataPathRequest* reqs, std::size_t count, const HostSubmitContext&) {
    SubmitOutcome out;
    out.initial_states.resize(count);
    if (count == 0) return out;
    auto op = std::make_shared<Op>();
    std::vector<Task> tasks;
    {
        std::lock_guard<std::mutex> g(mu_);
        op->gen = next_++;
        for (std::size_t i = 0; i < count; ++i) {
            const auto& r = reqs[i];
            auto t = targets_.find(r.target.token);
            auto m = mems_.find(r.memory.token);
            if (t == targets_.end() || m == mems_.end()) {
                out.initial_states[i] = {IoRequestState::REJECTED, {StatusCode::NOT_FOUND, "unknown handle"}};
                continue;
            }
            out.initial_states[i] = {IoRequestState::ACCEPTED, Status::Ok()};
            tasks.push_back({op->gen, static_cast<std::uint32_t>(i), r.intent.direction, t->second.fd_direct,
                             t->second.fd_buffered, r.intent.target_offset, r.intent.length,
                             m->second.base + r.intent.memory_offset, m->second.kind == DataPathMemoryKind::DEVICE});
        }
        if (tasks.empty()) {
            out.status = {StatusCode::NOT_FOUND, "no request accepted"};
            return out;
        }
        op->n = static_cast<std::uint32_t>(tasks.size());
        op->remaining.store(op->n);
        ops_[op->gen] = op;
    }
    {
        std::lock_guard<std::mutex> g(qmu_);
        for (auto& t : tasks) queue_.push_back(t);
    }
    qcv_.notify_all();
    out.op = DataPathOp{op->gen, op->gen};
    return out;
}

bool PosixDataPath::run(const Task& t, char* bounce) {
    const std::uint64_t n = executed_.fetch_add(1) + 1;
    if (cfg_.inject_fail_every && n % cfg_.inject_fail_every == 0) return false;
    auto io = [&](char* buf, std::uint64_t off, std::uint64_t len) -> bool {
        const bool aligned = ((reinterpret_cast<std::uintptr_t>(buf) | off | len) & 4095) == 0;
        int fd = (aligned && t.fd_direct >= 0) ? t.fd_direct : t.fd_buffered;
        std::uint64_t done = 0;
        while (done < len) {
            ssize_t r = t.dir == IoDirection::READ ? ::pread(fd, buf + done, len - done, off + done)
                                                   : ::pwrite(fd, buf + done, len - done, off + done);
            if (r < 0 && errno == EINTR) continue;
            if (r < 0 && fd == t.fd_direct) {
                fd = t.fd_buffered;  // O_DIRECT refused (filesystem): fall back
                continue;
            }
            if (r <= 0) return false;
            done += static_cast<std::uint64_t>(r);
        }
        return true;
    };
    if (!t.device) return io(t.mem, t.foff, t.len);
    // Device memory: bounce through page-locked memory.
    for (std::uint64_t o = 0; o < t.len; o += cfg_.bounce_bytes) {
        const std::uint64_t len = std::min<std::uint64_t>(cfg_.bounce_bytes, t.len - o);
        if (t.dir == IoDirection::READ) {
            if (!io(bounce, t.foff + o, len)) return false;
            if (cudaMemcpy(t.mem + o, bounce, len, cudaMemcpyHostToDevice) != cudaSuccess) {
                cudaGetLastError();
                return false;
            }
        } else {
            if (cudaMemcpy(bounce, t.mem + o, len, cudaMemcpyDeviceToHost) != cudaSuccess) {
                cudaGetLastError();
                return false;
            }
            if (!io(bounce, t.foff + o, len)) return false;
        }
    }
    return true;
}

void PosixDataPath::worker() {
    char* bounce = nullptr;
    bool pinned = false;
    for (;;) {
        Task t;
        {
            std::unique_lock<std::mutex> lk(qmu_);
            qcv_.wait(lk, [&] { return stop_ || !queue_.empty(); });
            if (stop_ && queue_.empty()) break;
            t = queue_.front();
            queue_.pop_front();
        }
        if (t.device && !bounce) {
            DeviceGuard g(cfg_.accel_id);
            if (cudaHostAlloc(reinterpret_cast<void**>(&bounce), cfg_.bounce_bytes, cudaHostAllocDefault) == cudaSuccess) {
                pinned = true;
            } else {
                cudaGetLastError();
                if (posix_memalign(reinterpret_cast<void**>(&bounce), 4096, cfg_.bounce_bytes) != 0) bounce = nullptr;
            }
        }
        bool ok;
        {
            DeviceGuard g(t.device ? cfg_.accel_id : -1);
            ok = (t.device && !bounce) ? false : run(t, bounce);
        }
        std::shared_ptr<Op> op;
        {
            std::lock_guard<std::mutex> g(mu_);
            auto it = ops_.find(t.op);
            if (it != ops_.end()) op = it->second;
        }
        if (!op) continue;
        {
            std::lock_guard<std::mutex> g(op->mu);
            if (ok)
                op->ok_bytes += t.len;
            else
                op->failed.push_back(t.index);
        }
        op->remaining.fetch_sub(1);
    }
    if (bounce) {
        if (pinned)
            cudaFreeHost(bounce);
        else
            std::free(bounce);
    }
}

Result<ProgressResult> PosixDataPath::progress(ProgressBudget) {
    ProgressResult r;
    std::lock_guard<std::mutex> g(mu_);
    for (auto& kv : ops_)
        if (kv.second->remaining.load() > 0) r.more_work_likely = true;
    return r;
}

Result<DataPathSnapshot> PosixDataPath::query(DataPathOp op) const {
    std::lock_guard<std::mutex> g(mu_);
    auto it = ops_.find(op.token);
    if (it == ops_.end()) return Result<DataPathSnapshot>::Failure({StatusCode::NOT_FOUND, "unknown op"});
    DataPathSnapshot s;
    Op& o = *it->second;
    if (o.remaining.load() > 0) return s;
    std::lock_guard<std::mutex> g2(o.mu);
    s.state = o.failed.empty() ? IoState::COMPLETED : IoState::FAILED;
    s.bytes_transferred = o.ok_bytes;
    s.detail.confirmed_bytes = o.ok_bytes;
    if (!o.failed.empty()) {
        s.status = {StatusCode::DEVICE_ERROR, std::to_string(o.failed.size()) + " request(s) failed"};
        s.detail.failure_kind = IoFailureKind::NVME_CQ_ERROR;
        s.detail.failure_scope = IoFailureScope::REQUEST_INDICES;
        s.detail.failed_request_indices = o.failed;
        std::sort(s.detail.failed_request_indices.begin(), s.detail.failed_request_indices.end());
        s.detail.first_failed_entry = s.detail.failed_request_indices.front();
    }
    return s;
}

Status PosixDataPath::release(DataPathOp op) {
    std::lock_guard<std::mutex> g(mu_);
    auto it = ops_.find(op.token);
    if (it == ops_.end()) return {StatusCode::NOT_FOUND, "unknown op"};
    if (it->second->remaining.load() > 0) return {StatusCode::BUSY, "op in flight"};
    ops_.erase(it);
    return Status::Ok();
}

}  // namespace tutti
