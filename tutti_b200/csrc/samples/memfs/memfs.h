#pragma once
// memfs: an in-memory storage backend built only on the public SPI headers
// (resolver, payload, DataPath, resource provider). It shows that a new
// backend plugs into StorageRuntime without touching the runtime or the SPI:
// nothing outside this header names a memfs type except the preset that
// assembles it.
//
//   memfs://<name>?size=<n>[K|M|G]   creates the object on its first resolve
//   memfs://<name>                   an existing object
//
// Objects are host byte arrays charged against one MemoryResource budget.
// Every request runs synchronously inside submit(): host memory by memcpy,
// device memory by cudaMemcpy (the sample's stand-in for a device with no
// latency), so each op is terminal when submit returns.
// Parity: reference csrc/payloads/memfs/{payload.h,memfs_data_path.h} (the
// sample DataPath and its private payload) and csrc/resource/memory/
// memory_resource.h (the byte budget behind it).

#include <cuda_runtime_api.h>

#include <cstdint>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <string_view>
#include <unordered_map>
#include <vector>

#include <tutti/spi/data_path.h>
#include <tutti/spi/resolver.h>
#include <tutti/status.h>

namespace tutti::samples::memfs {

inline constexpr const char* kResolverType = "tutti.memfs";
inline constexpr const char* kPayloadType = "tutti.memfs.object";
inline constexpr std::uint32_t kPayloadVersion = 1;
inline constexpr const char* kDataPathKey = "memfs";

// The byte budget every memfs object is charged against.
class MemoryResource final : public ResourceProvider {
public:
    explicit MemoryResource(std::uint64_t capacity_bytes) : capacity_(capacity_bytes) {}
    Status charge(std::uint64_t bytes) {
        std::lock_guard<std::mutex> g(mu_);
        if (bytes > capacity_ - used_)
            return {StatusCode::RESOURCE_EXHAUSTED, "memfs budget: " + std::to_string(capacity_ - used_) +
                                                        " bytes free, " + std::to_string(bytes) + " asked"};
        used_ += bytes;
        return Status::Ok();
    }
    void refund(std::uint64_t bytes) {
        std::lock_guard<std::mutex> g(mu_);
        used_ -= bytes < used_ ? bytes : used_;
    }
    std::uint64_t capacity() const { return capacity_; }
    std::uint64_t used() const {
        std::lock_guard<std::mutex> g(mu_);
        return used_;
    }

private:
    const std::uint64_t capacity_;
    mutable std::mutex mu_;
    std::uint64_t used_ = 0;
};

// One object's bytes; shared by the resolver's namespace and every open target,
// refunded to the budget when the last of them lets go.
class Object {
public:
    Object(std::string name, std::uint64_t size, std::shared_ptr<MemoryResource> budget)
        : name_(std::move(name)), bytes_(size, 0), budget_(std::move(budget)) {}
    ~Object() {
        if (budget_) budget_->refund(bytes_.size());
    }
    const std::string& name() const { return name_; }
    std::uint64_t size() const { return bytes_.size(); }
    std::uint8_t* data() { return bytes_.data(); }

private:
    std::string name_;
    std::vector<std::uint8_t> bytes_;
    std::shared_ptr<MemoryResource> budget_;
};

// The payload private between the memfs resolver and the memfs DataPath.
struct Payload {
    std::shared_ptr<Object> object;
};

inline Result<std::uint64_t> parse_size(std::string_view s) {
    using R = Result<std::uint64_t>;
    if (s.empty()) return R::Failure({StatusCode::INVALID_ARGUMENT, "empty size"});
    std::uint64_t mult = 1;
    const char last = s.back();
    if (last == 'K' || last == 'k') mult = 1ull << 10;
    if (last == 'M' || last == 'm') mult = 1ull << 20;
    if (last == 'G' || last == 'g') mult = 1ull << 30;
    if (mult != 1) s.remove_suffix(1);
    std::uint64_t v = 0;
    for (char c : s) {
        if (c < '0' || c > '9') return R::Failure({StatusCode::INVALID_ARGUMENT, "bad size"});
        v = v * 10 + static_cast<std::uint64_t>(c - '0');
    }
    return v * mult;
}

class Resolver final : public StorageTargetResolver {
public:
    explicit Resolver(std::shared_ptr<MemoryResource> budget) : budget_(std::move(budget)) {}

    Result<ResolvedTarget> resolve(std::string_view uri, const ResolveOptions&) override {
        using R = Result<ResolvedTarget>;
        constexpr std::string_view kPrefix = "memfs://";
        if (uri.substr(0, kPrefix.size()) != kPrefix)
            return R::Failure({StatusCode::INVALID_ARGUMENT, "not a memfs URI: " + std::string(uri)});
        std::string_view rest = uri.substr(kPrefix.size());
        std::string_view name = rest, query;
        if (auto q = rest.find('?'); q != std::string_view::npos) {
            name = rest.substr(0, q);
            query = rest.substr(q + 1);
        }
        if (name.empty()) return R::Failure({StatusCode::INVALID_ARGUMENT, "memfs URI without a name"});
        std::uint64_t size = 0;
        bool sized = false;
        if (!query.empty()) {
            if (query.substr(0, 5) != "size=") return R::Failure({StatusCode::INVALID_ARGUMENT, "unknown memfs option"});
            auto sz = parse_size(query.substr(5));
            if (!sz.ok()) return R::Failure(sz.status());
            size = sz.value();
            sized = true;
        }
        std::shared_ptr<Object> obj;
        {
            std::lock_guard<std::mutex> g(mu_);
            auto it = objects_.find(std::string(name));
            if (it != objects_.end()) {
                if (sized && size != it->second->size())
                    return R::Failure({StatusCode::INVALID_ARGUMENT, "memfs object exists with another size"});
                obj = it->second;
            } else {
                if (!sized) return R::Failure({StatusCode::NOT_FOUND, "no memfs object " + std::string(name)});
                if (size == 0) return R::Failure({StatusCode::INVALID_ARGUMENT, "memfs object of size 0"});
                TUTTI_RETURN_IF_ERROR_R(R, budget_->charge(size));
                obj = std::make_shared<Object>(std::string(name), size, budget_);
                objects_.emplace(obj->name(), obj);
            }
        }
        auto payload = std::make_shared<const Payload>(Payload{obj});
        return ResolvedTarget::make<Payload>(kResolverType, kPayloadType, kPayloadVersion, obj->size(), kDataPathKey,
                                             std::string(uri), payload);
    }

    // Drops `name` from the namespace; targets already open keep its bytes until closed.
    Status remove(std::string_view name) {
        std::lock_guard<std::mutex> g(mu_);
        return objects_.erase(std::string(name)) ? Status::Ok() : Status(StatusCode::NOT_FOUND, "no such object");
    }

private:
    std::shared_ptr<MemoryResource> budget_;
    std::mutex mu_;
    std::unordered_map<std::string, std::shared_ptr<Object>> objects_;
};

class MemfsDataPath final : public DataPath {
public:
    MemfsDataPath() {
        caps_.name = kDataPathKey;
        caps_.source_api_version = kPayloadVersion;
        caps_.supports_host_execution = true;
        caps_.supports_host_memory = true;
        caps_.supports_device_memory = true;
        caps_.supports_direct = true;
        caps_.supports_read = true;
        caps_.supports_write = true;
        caps_.registration_scope = RegistrationScope::GLOBAL;
        caps_.progress_model = ProgressModel::HOST_POLL;
        caps_.supports_multi_stream = true;
    }
    const DataPathCapabilities& capabilities() const override { return caps_; }
    Status initialize(const DataPathConfig&, ResourceProvider*) override { return Status::Ok(); }
    Status shutdown(std::uint64_t) override {
        std::lock_guard<std::mutex> g(mu_);
        targets_.clear();
        mems_.clear();
        ops_.clear();
        return Status::Ok();
    }

    Result<DataPathTarget> open(const ResolvedTarget& t) override {
        auto pv = t.view<Payload>(kPayloadType, kPayloadVersion);
        if (!pv.ok()) return Result<DataPathTarget>::Failure(pv.status());
        std::lock_guard<std::mutex> g(mu_);
        const std::uint64_t id = next_++;
        targets_[id] = pv.value()->object;
        return DataPathTarget{id, id};
    }
    Status close(DataPathTarget t) override {
        std::lock_guard<std::mutex> g(mu_);
        return targets_.erase(t.token) ? Status::Ok() : Status(StatusCode::NOT_FOUND, "unknown target");
    }
    Result<RegistrationDomainKey> registration_domain(DataPathTarget) const override {
        return RegistrationDomainKey{kDataPathKey};
    }
    Result<DataPathMemory> register_memory(const DataPathMemoryView& v, const RegistrationDomainKey&) override {
        if (!v.base || !v.size_bytes)
            return Result<DataPathMemory>::Failure({StatusCode::INVALID_ARGUMENT, "empty memory"});
        std::lock_guard<std::mutex> g(mu_);
        const std::uint64_t id = next_++;
        mems_[id] = Mem{static_cast<std::uint8_t*>(v.base), v.size_bytes, v.kind == DataPathMemoryKind::DEVICE};
        return DataPathMemory{id, id};
    }
    Status unregister_memory(DataPathMemory m) override {
        std::lock_guard<std::mutex> g(mu_);
        return mems_.erase(m.token) ? Status::Ok() : Status(StatusCode::NOT_FOUND, "unknown memory");
    }

    SubmitOutcome submit(const DataPathRequest* reqs, std::size_t count, const HostSubmitContext&) override {
        SubmitOutcome out;
        out.initial_states.resize(count);
        if (count == 0) return out;
        std::lock_guard<std::mutex> g(mu_);
        Op op;
        std::size_t accepted = 0;
        for (std::size_t i = 0; i < count; ++i) {
            auto& st = out.initial_states[i];
            const DataPathRequest& r = reqs[i];
            auto t = targets_.find(r.target.token);
            auto m = mems_.find(r.memory.token);
            if (t == targets_.end() || m == mems_.end()) {
                st = {IoRequestState::REJECTED, {StatusCode::NOT_FOUND, "unknown target or memory"}};
                continue;
            }
            const std::uint64_t len = r.intent.length;
            Object& obj = *t->second;
            if (r.intent.target_offset > obj.size() || len > obj.size() - r.intent.target_offset ||
                r.intent.memory_offset > m->second.size || len > m->second.size - r.intent.memory_offset) {
                st = {IoRequestState::REJECTED, {StatusCode::OUT_OF_RANGE, "request outside target or memory"}};
                continue;
            }
            std::uint8_t* dev = obj.data() + r.intent.target_offset;
            std::uint8_t* mem = m->second.base + r.intent.memory_offset;
            const bool read = r.intent.direction == IoDirection::READ;
            bool ok = true;
            if (m->second.device) {
                ok = cudaMemcpy(read ? static_cast<void*>(mem) : dev, read ? static_cast<const void*>(dev) : mem, len,
                                read ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToHost) == cudaSuccess;
                if (!ok) cudaGetLastError();
            } else {
                std::memcpy(read ? mem : dev, read ? dev : mem, len);
            }
            st = {IoRequestState::ACCEPTED, Status::Ok()};
            ++accepted;
            if (ok) {
                op.detail.confirmed_bytes += len;
            } else {
                op.detail.failed_request_indices.push_back(static_cast<std::uint32_t>(i));
            }
        }
        if (!accepted) {
            out.status = out.initial_states[0].status;
            return out;
        }
        if (!op.detail.failed_request_indices.empty()) {
            op.state = IoState::FAILED;
            op.status = {StatusCode::DEVICE_ERROR, "device copy failed"};
            op.detail.failure_kind = IoFailureKind::UNKNOWN;
            op.detail.failure_scope = IoFailureScope::REQUEST_INDICES;
            op.detail.first_failed_entry = op.detail.failed_request_indices.front();
        }
        const std::uint64_t id = next_++;
        ops_[id] = std::move(op);
        out.op = DataPathOp{id, id};
        out.status = accepted == count ? Status::Ok() : Status(StatusCode::INVALID_ARGUMENT, "some requests rejected");
        return out;
    }

    Result<ProgressResult> progress(ProgressBudget) override { return ProgressResult{}; }  // nothing is ever in flight
    Result<DataPathSnapshot> query(DataPathOp o) const override {
        std::lock_guard<std::mutex> g(mu_);
        auto it = ops_.find(o.token);
        if (it == ops_.end()) return Result<DataPathSnapshot>::Failure({StatusCode::NOT_FOUND, "unknown op"});
        DataPathSnapshot s;
        s.state = it->second.state;
        s.status = it->second.status;
        s.bytes_transferred = it->second.detail.confirmed_bytes;
        s.detail = it->second.detail;
        return s;
    }
    Status release(DataPathOp o) override {
        std::lock_guard<std::mutex> g(mu_);
        return ops_.erase(o.token) ? Status::Ok() : Status(StatusCode::NOT_FOUND, "unknown op");
    }

private:
    struct Mem {
        std::uint8_t* base = nullptr;
        std::uint64_t size = 0;
        bool device = false;
    };
    struct Op {
        IoState state = IoState::COMPLETED;
        Status status;
        IoCompletionDetail detail;
    };
    DataPathCapabilities caps_;
    mutable std::mutex mu_;
    std::uint64_t next_ = 1;
    std::unordered_map<std::uint64_t, std::shared_ptr<Object>> targets_;
    std::unordered_map<std::uint64_t, Mem> mems_;
    std::unordered_map<std::uint64_t, Op> ops_;
};

}  // namespace tutti::samples::memfs
