#pragma once
// DataPath SPI: the host-side data-plane contract every transport implements.
//
// Contract (parity with reference csrc/include/tutti/spi/data_path.h:171-397):
//  * capabilities are hard constraints: the runtime rejects what violates them
//    before any irreversible submit;
//  * submit() is partial-commit: per-request ACCEPTED/REJECTED in input order,
//    an op exists iff at least one request was issued;
//  * progress() is bounded by its budget; query() never destroys an op;
//  * release() is legal only on a terminal op (BUSY otherwise); a terminal op
//    never touches caller memory again.

#include <cstddef>
#include <cstdint>
#include <optional>
#include <string>
#include <vector>

#include <tutti/io_types.h>
#include <tutti/status.h>

namespace tutti {

class ResolvedTarget;

// Opaque environment handed to DataPath::initialize (leases, device grants).
class ResourceProvider {
public:
    virtual ~ResourceProvider() = default;
};

// (token, generation) identity minted by a DataPath for its own objects.
template <typename Tag>
struct SpiIdentity {
    std::uint64_t token = 0;
    std::uint64_t generation = 0;
    bool valid() const noexcept { return generation != 0; }
    bool operator==(const SpiIdentity& o) const noexcept {
        return token == o.token && generation == o.generation;
    }
    bool operator!=(const SpiIdentity& o) const noexcept { return !(*this == o); }
};
struct DataPathTargetTag {};
struct DataPathMemoryTag {};
struct DataPathOpTag {};
using DataPathTarget = SpiIdentity<DataPathTargetTag>;
using DataPathMemory = SpiIdentity<DataPathMemoryTag>;
using DataPathOp = SpiIdentity<DataPathOpTag>;

struct RegistrationDomainKey {
    std::string value;
    bool operator==(const RegistrationDomainKey& o) const noexcept { return value == o.value; }
    bool operator!=(const RegistrationDomainKey& o) const noexcept { return value != o.value; }
};

enum class DataPathMemoryKind { HOST, DEVICE };

struct DataPathMemoryView {
    void* base = nullptr;
    std::uint64_t size_bytes = 0;
    std::int32_t expected_accel_id = -1;
    DataPathMemoryKind kind = DataPathMemoryKind::HOST;
    std::uint64_t io_granularity = 0;
};

struct DataPathConfig {
    std::string name;
};

enum class RegistrationScope { PER_TARGET, PER_DEVICE, GLOBAL };
enum class ProgressModel { HOST_POLL, DEVICE_AUTONOMOUS };

struct DataPathCapabilities {
    std::string name;
    std::uint32_t source_api_version = 0;
    bool supports_host_execution = false;
    bool supports_device_execution = false;
    bool supports_host_memory = false;
    bool supports_device_memory = false;
    bool supports_direct = false;
    bool supports_staged = false;
    bool supports_read = false;
    bool supports_write = false;
    std::uint64_t target_alignment_bytes = 1;
    std::uint64_t memory_alignment_bytes = 1;
    std::uint64_t length_alignment_bytes = 1;
    std::uint64_t max_single_io_bytes = 0;  // 0: unlimited
    std::uint64_t max_batch_requests = 0;   // 0: unlimited
    std::uint64_t max_batch_bytes = 0;
    std::uint64_t max_in_flight_operations = 0;
    bool supports_scatter_gather = false;
    std::uint64_t max_scatter_gather_entries = 0;
    RegistrationScope registration_scope = RegistrationScope::PER_TARGET;
    ProgressModel progress_model = ProgressModel::HOST_POLL;
    bool device_completion_fence_on_caller_stream = false;
    bool device_execution_autonomous = false;
    bool supports_multi_stream = false;
    std::uint64_t max_concurrent_streams = 0;
    std::uint64_t max_concurrent_operations = 0;
    std::int32_t bound_accel_id = -1;  // -1: host-only / unbound
    bool supports_multi_gpu = false;
    bool supports_cross_device = false;
    bool supports_fp8_block_transform = false;  // IoTransform::FP8_E4M3_BLOCK128
    std::vector<std::string> optional_target_features;
};

struct DataPathRequest {
    IoRequest intent;
    DataPathMemory memory;
    DataPathTarget target;
};

enum class IoRequestState { ACCEPTED, REJECTED };

struct IoRequestInitialState {
    IoRequestState state = IoRequestState::REJECTED;
    Status status;
};

struct SubmitOutcome {
    Status status;
    std::optional<DataPathOp> op;
    std::vector<IoRequestInitialState> initial_states;
};

enum class IoState { IN_FLIGHT, COMPLETED, FAILED };

enum class IoFailureKind : std::uint8_t {
    NONE,
    RESOLVE_LBA,
    CQ_TIMEOUT,
    NVME_CQ_ERROR,
    CUDA_QUERY_ERROR,
    STATUS_D2H_ERROR,
    UNKNOWN,
};

enum class IoFailureScope : std::uint8_t { NONE, REQUEST_INDICES, WHOLE_OPERATION };

struct IoCompletionDetail {
    std::uint64_t confirmed_bytes = 0;  // bytes whose completion was observed
    bool timeout_seen = false;
    std::uint32_t first_failed_entry = UINT32_MAX;
    IoFailureKind failure_kind = IoFailureKind::NONE;
    std::uint32_t raw_cq_status = 0;
    IoFailureScope failure_scope = IoFailureScope::NONE;
    std::vector<std::uint32_t> failed_request_indices;
};

struct DataPathSnapshot {
    IoState state = IoState::IN_FLIGHT;
    Status status;
    std::uint64_t bytes_transferred = 0;
    IoCompletionDetail detail;
};

struct ProgressBudget {
    std::uint64_t max_work_units = 0;
    std::uint64_t timeout_ns = 0;
};

struct ProgressResult {
    std::uint64_t work_units_consumed = 0;
    std::uint64_t operations_advanced = 0;
    std::uint64_t operations_terminal = 0;
    bool more_work_likely = false;
    std::optional<std::uint64_t> next_poll_deadline_ns;
};

class DataPath {
public:
    virtual ~DataPath() = default;

    virtual const DataPathCapabilities& capabilities() const = 0;

    virtual Status initialize(const DataPathConfig& config, ResourceProvider* resources) = 0;
    virtual Status shutdown(std::uint64_t timeout_ns) = 0;

    virtual Result<DataPathTarget> open(const ResolvedTarget& target) = 0;
    // Several opens at once (StorageRuntime::open_batch): a DataPath may share
    // per-open costs, e.g. device uploads, across the batch. Same results as
    // calling open() on each target in order.
    virtual std::vector<Result<DataPathTarget>> open_many(const ResolvedTarget* const* targets, std::size_t count) {
        std::vector<Result<DataPathTarget>> out;
        out.reserve(count);
        for (std::size_t i = 0; i < count; ++i) out.push_back(open(*targets[i]));
        return out;
    }
    virtual Status close(DataPathTarget target) = 0;
    virtual Result<RegistrationDomainKey> registration_domain(DataPathTarget target) const = 0;

    virtual Result<DataPathMemory> register_memory(const DataPathMemoryView& view,
                                                   const RegistrationDomainKey& domain) = 0;
    virtual Status unregister_memory(DataPathMemory memory) = 0;

    // requests may mix targets of this DataPath; the runtime groups by DataPath only.
    virtual SubmitOutcome submit(const DataPathRequest* requests, std::size_t count,
                                 const HostSubmitContext& ctx) = 0;
    virtual Result<ProgressResult> progress(ProgressBudget budget) = 0;
    virtual Result<DataPathSnapshot> query(DataPathOp op) const = 0;
    virtual Status release(DataPathOp op) = 0;
};

// Optional: device-side completion waits on a consumer stream
// (reference spi/async_completion.h:18).
class AsyncCompletion {
public:
    virtual ~AsyncCompletion() = default;
    virtual Status enqueue_wait(const DataPathOp* ops, std::size_t count, cudaStream_t stream) = 0;
};

}  // namespace tutti
