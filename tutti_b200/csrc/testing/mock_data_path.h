#pragma once
// Mock DataPath kit: a complete, hardware-free DataPath + resolver pair with
// injection points, for contract tests of StorageRuntime and its callers.
//   resolver "mem://<name>" -> a target whose bytes live in a std::string
//   set_reject_at_index(i)   -> request i of the next submit is REJECTED
//   set_fail_request(i)      -> request i of the next op completes FAILED
//   set_manual_mode(true)    -> ops stay IN_FLIGHT until complete_all()
//   set_fail_progress(true)  -> progress() returns an error
// Parity: reference csrc/testing/mock_data_path.h (same injection seams).

#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include <tutti/spi/data_path.h>
#include <tutti/spi/resolver.h>

namespace tutti {
namespace testing {

struct MemTargetPayload {
    std::string name;
    std::shared_ptr<std::string> bytes;
};
constexpr char kMemPayloadType[] = "tutti.mock-mem";

class MemResolver : public StorageTargetResolver {
public:
    std::map<std::string, std::shared_ptr<std::string>> objects;
    Result<ResolvedTarget> resolve(std::string_view uri, const ResolveOptions&) override {
        std::string u(uri);
        const std::string pre = "mem://";
        if (u.rfind(pre, 0) != 0) return Result<ResolvedTarget>::Failure({StatusCode::INVALID_ARGUMENT, "not mem://"});
        auto it = objects.find(u.substr(pre.size()));
        if (it == objects.end()) return Result<ResolvedTarget>::Failure({StatusCode::NOT_FOUND, "no object " + u});
        auto p = std::make_shared<MemTargetPayload>(MemTargetPayload{it->first, it->second});
        return ResolvedTarget::make<MemTargetPayload>("mock-mem", kMemPayloadType, 1, it->second->size(), "mock",
                                                      u, p);
    }
};

class MockDataPath : public DataPath {
public:
    MockDataPath() {
        caps_.name = "mock";
        caps_.supports_host_execution = true;
        caps_.supports_host_memory = true;
        caps_.supports_read = caps_.supports_write = true;
    }
    const DataPathCapabilities& capabilities() const override { return caps_; }
    DataPathCapabilities& mutable_caps() { return caps_; }
    Status initialize(const DataPathConfig&, ResourceProvider*) override {
        initialized = true;
        return Status::Ok();
    }
    Status shutdown(std::uint64_t) override {
        shut_down = true;
        return Status::Ok();
    }
    Result<DataPathTarget> open(const ResolvedTarget& t) override {
        auto v = t.view<MemTargetPayload>(kMemPayloadType, 1);
        if (!v.ok()) return Result<DataPathTarget>::Failure(v.status());
        std::lock_guard<std::mutex> g(mu_);
        const std::uint64_t id = next_++;
        targets_[id] = v.value()->bytes;
        return DataPathTarget{id, id};
    }
    Status close(DataPathTarget t) override {
        std::lock_guard<std::mutex> g(mu_);
        return targets_.erase(t.token) ? Status::Ok() : Status(StatusCode::NOT_FOUND, "unknown target");
    }
    Result<RegistrationDomainKey> registration_domain(DataPathTarget) const override {
        return RegistrationDomainKey{"mock"};
    }
    Result<DataPathMemory> register_memory(const DataPathMemoryView& v, const RegistrationDomainKey&) override {
        std::lock_guard<std::mutex> g(mu_);
        const std::uint64_t id = next_++;
        mems_[id] = static_cast<char*>(v.base);
        return DataPathMemory{id, id};
    }
    Status unregister_memory(DataPathMemory m) override {
        std::lock_guard<std::mutex> g(mu_);
        return mems_.erase(m.token) ? Status::Ok() : Status(StatusCode::NOT_FOUND, "unknown memory");
    }
    SubmitOutcome submit(const DataPathRequest* reqs, std::size_t n, const HostSubmitContext&) override {
        std::lock_guard<std::mutex> g(mu_);
        SubmitOutcome out;
        out.initial_states.resize(n);
        Op op;
        bool any = false;
        for (std::size_t i = 0; i < n; ++i) {
            if (static_cast<long>(i) == reject_at_) {
                out.initial_states[i] = {IoRequestState::REJECTED, {StatusCode::BUSY, "injected rejection"}};
                if (out.status.ok()) out.status = out.initial_states[i].status;
                continue;
            }
            out.initial_states[i] = {IoRequestState::ACCEPTED, Status::Ok()};
            any = true;
            op.reqs.push_back(reqs[i]);
            op.index.push_back(static_cast<std::uint32_t>(i));
        }
        reject_at_ = -1;
        if (!any) return out;
        op.fail_index = fail_request_;
        fail_request_ = -1;
        const std::uint64_t id = next_++;
        ops_[id] = std::move(op);
        if (!manual_) execute_locked(id);
        out.op = DataPathOp{id, id};
        return out;
    }
    Result<ProgressResult> progress(ProgressBudget) override {
        if (fail_progress_) return Result<ProgressResult>::Failure({StatusCode::DEVICE_ERROR, "injected progress failure"});
        return ProgressResult{};
    }
    Result<DataPathSnapshot> query(DataPathOp op) const override {
        std::lock_guard<std::mutex> g(mu_);
        auto it = ops_.find(op.token);
        if (it == ops_.end()) return Result<DataPathSnapshot>::Failure({StatusCode::NOT_FOUND, "unknown op"});
        return it->second.snap;
    }
    Status release(DataPathOp op) override {
        std::lock_guard<std::mutex> g(mu_);
        auto it = ops_.find(op.token);
        if (it == ops_.end()) return {StatusCode::NOT_FOUND, "unknown op"};
        if (it->second.snap.state == IoState::IN_FLIGHT) return {StatusCode::BUSY, "in flight"};
        ops_.erase(it);
        ++released;
        return Status::Ok();
    }

    void set_reject_at_index(long i) { reject_at_ = i; }
    void set_fail_request(long i) { fail_request_ = i; }
    void set_manual_mode(bool m) { manual_ = m; }
    void set_fail_progress(bool f) { fail_progress_ = f; }
    void complete_all() {
        std::lock_guard<std::mutex> g(mu_);
        for (auto& kv : ops_)
            if (kv.second.snap.state == IoState::IN_FLIGHT) execute_locked(kv.first);
    }
    bool initialized = false, shut_down = false;
    int released = 0;

private:
    struct Op {
        std::vector<DataPathRequest> reqs;
        std::vector<std::uint32_t> index;
        long fail_index = -1;
        DataPathSnapshot snap;
    };
    void execute_locked(std::uint64_t id) {
        Op& op = ops_[id];
        op.snap.state = IoState::COMPLETED;
        for (std::size_t k = 0; k < op.reqs.size(); ++k) {
            const auto& r = op.reqs[k];
            if (op.fail_index == static_cast<long>(op.index[k])) {
                op.snap.state = IoState::FAILED;
                op.snap.status = {StatusCode::DEVICE_ERROR, "injected request failure"};
                op.snap.detail.failure_kind = IoFailureKind::NVME_CQ_ERROR;
                op.snap.detail.failure_scope = IoFailureScope::REQUEST_INDICES;
                // indices name entries of the DataPath submit's request array
                op.snap.detail.failed_request_indices.push_back(op.index[k]);
                continue;
            }
            auto& blob = *targets_[r.target.token];
            char* mem = mems_[r.memory.token] + r.intent.memory_offset;
            if (r.intent.direction == IoDirection::READ)
                std::memcpy(mem, blob.data() + r.intent.target_offset, r.intent.length);
            else
                std::memcpy(&blob[r.intent.target_offset], mem, r.intent.length);
            op.snap.detail.confirmed_bytes += r.intent.length;
        }
        op.snap.bytes_transferred = op.snap.detail.confirmed_bytes;
    }
    DataPathCapabilities caps_;
    mutable std::mutex mu_;
    std::map<std::uint64_t, std::shared_ptr<std::string>> targets_;
    std::map<std::uint64_t, char*> mems_;
    std::map<std::uint64_t, Op> ops_;
    std::uint64_t next_ = 1;
    long reject_at_ = -1, fail_request_ = -1;
    bool manual_ = false, fail_progress_ = false;
};

}  // namespace testing
}  // namespace tutti
