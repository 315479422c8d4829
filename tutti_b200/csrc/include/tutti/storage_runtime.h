#pragma once
// StorageRuntime: the stable public API.
//
//   create / create_owning / create_stub
//   register_memory / unregister_memory / allocate_memory / free_memory
//   open / open_batch / close / close_batch / query_target
//   submit (partial commit) / query / wait / wait_result / wait_detail
//   enqueue_wait / release_io / shutdown
//
// Parity: reference csrc/include/tutti/storage_runtime.h:236-1196 (same verbs,
// same partial-commit and terminal-result-budget semantics, resolver routing
// by URI scheme, DataPath routing by the resolver's recommended key, one
// DataPath submit per DataPath per runtime submit, parallel open_batch with
// per-item results). This implementation is a compiled library rather than a
// header-only class.

#include <cstdint>
#include <memory>
#include <optional>
#include <string>
#include <string_view>
#include <vector>

#include <tutti/io_types.h>
#include <tutti/memory_types.h>
#include <tutti/spi/data_path.h>
#include <tutti/spi/resolver.h>
#include <tutti/status.h>

namespace tutti {

enum class RuntimeState { RUNNING, DRAINING, STOPPED };

struct RuntimeConfig {
    std::int32_t accel_id = 0;
    std::uint64_t max_terminal_results = 64;  // unreleased terminal IOs before submit refuses
    std::uint32_t open_batch_threads = 8;
    std::string profile_name = "CUDA";
};

struct ResolverBinding {
    std::string scheme;
    StorageTargetResolver* resolver = nullptr;
};
struct DataPathBinding {
    std::string key;
    DataPath* data_path = nullptr;
    DataPathConfig config;
};
struct RuntimeComponents {
    std::vector<ResolverBinding> resolvers;
    std::vector<DataPathBinding> data_paths;
    ResourceProvider* resources = nullptr;
};
struct OwnedResolver {
    std::string scheme;
    std::unique_ptr<StorageTargetResolver> resolver;
};
struct OwnedDataPath {
    std::string key;
    std::shared_ptr<DataPath> data_path;
    DataPathConfig config;
};
struct OwnedComponents {
    std::vector<OwnedResolver> resolvers;
    std::vector<OwnedDataPath> data_paths;
    std::unique_ptr<ResourceProvider> resources;
    std::vector<std::shared_ptr<void>> keep_alive;  // e.g. controllers
};

struct DeviceInfo {
    std::int32_t accel_id = -1;
    std::string name;
    std::uint64_t total_memory = 0;
    std::string pci_bdf;
};
struct DeviceCapabilities {
    std::int32_t accel_id = -1;
    bool supports_host_execution = true;
    bool supports_device_execution = false;
    std::uint64_t max_io_size = 0;
    std::string pci_bdf;
};
struct MemorySpec {
    std::uint64_t size = 0;
    MemoryKind kind = MemoryKind::HOST;
    std::int32_t accel_id = -1;
};
struct MemoryAllocation {
    MemoryHandle handle;
    void* address = nullptr;
    std::uint64_t size = 0;
};
struct MemoryInfo {
    MemoryKind kind = MemoryKind::HOST;
    MemoryOwnership ownership = MemoryOwnership::CALLER_OWNED;
    std::uint64_t size = 0;
    void* address = nullptr;
    std::int32_t accel_id = -1;
    int inflight_count = 0;
};
struct OpenOptions {
    std::string scheme;
};
struct TargetInfo {
    std::string uri;
    std::uint64_t logical_size = 0;
    int inflight_count = 0;
    std::string data_path_key;
};
struct IoSnapshot {
    IoState state = IoState::IN_FLIGHT;
};
struct IoResult {
    IoState state = IoState::COMPLETED;
    Status status;
    IoCompletionDetail detail;
};
// observation_status OK -> terminal, result set; TIMEOUT -> still in flight;
// other -> handle error.
struct WaitOutcome {
    Status observation_status;
    std::optional<IoResult> result;
};
// io set <=> at least one request was irreversibly accepted.
struct IoSubmitOutcome {
    Status status;
    std::optional<IoHandle> io;
    std::vector<IoRequestInitialState> initial_states;
};

class StorageRuntime {
public:
    static Result<std::unique_ptr<StorageRuntime>> create(const RuntimeConfig& config,
                                                          const RuntimeComponents& components);
    static Result<std::unique_ptr<StorageRuntime>> create_owning(const RuntimeConfig& config,
                                                                 OwnedComponents components);
    // A runtime with no components, for hardware-free API tests: memory verbs
    // work; open gives any URI a 1 GiB stub target; submit validates requests
    // as usual and accepts them into an IO that stays IN_FLIGHT (no DataPath
    // moves data) until testing_force_complete makes it terminal.
    static std::unique_ptr<StorageRuntime> create_stub(const RuntimeConfig& config);

    ~StorageRuntime();
    StorageRuntime(const StorageRuntime&) = delete;
    StorageRuntime& operator=(const StorageRuntime&) = delete;

    Status shutdown(std::uint64_t timeout_ms);
    RuntimeState state() const noexcept;
    std::int32_t accel_id() const noexcept;
    std::uint32_t runtime_id() const noexcept;

    Result<std::vector<DeviceInfo>> list_devices() const;
    Result<DeviceCapabilities> query_device_capabilities(std::int32_t accel_id) const;
    std::vector<DataPathCapabilities> data_path_capabilities() const;

    Result<MemoryAllocation> allocate_memory(const MemorySpec& spec);
    Status free_memory(const MemoryHandle& handle);
    Result<MemoryHandle> register_memory(const MemoryView& view);
    Status unregister_memory(const MemoryHandle& handle);
    Result<MemoryInfo> query_memory(const MemoryHandle& handle) const;

    Result<TargetHandle> open(std::string_view uri, const OpenOptions& options = {});
    std::vector<Result<TargetHandle>> open_batch(const std::vector<std::string>& uris,
                                                 const OpenOptions& options = {});
    Status close(const TargetHandle& handle);
    Status close_batch(const std::vector<TargetHandle>& handles);
    Result<TargetInfo> query_target(const TargetHandle& handle) const;

    IoSubmitOutcome submit(const IoRequest* requests, std::size_t count, const HostSubmitContext& context);
    Result<IoSnapshot> query(const IoHandle& handle);
    WaitOutcome wait(const IoHandle& handle, std::uint64_t timeout_ms);
    WaitOutcome wait_result(const IoHandle& handle, std::uint64_t timeout_ms) { return wait(handle, timeout_ms); }
    Result<IoResult> wait_detail(const IoHandle& handle, std::uint64_t timeout_ms);
    Status enqueue_wait(const IoHandle* handles, std::size_t count, cudaStream_t stream);
    Status release_io(const IoHandle& handle);

    // Test seam: number of terminal results not yet released.
    std::size_t unreleased_terminal_results() const;

    // Test seam, stub runtimes only: make an IO of a stub runtime terminal.
    // `terminal` is COMPLETED or FAILED; a FAILED IO reports `io_status` (an
    // error; INTERNAL when Ok is given) and every accepted request as failed.
    // UNSUPPORTED on a component-backed runtime (its DataPaths complete IO),
    // NOT_FOUND for an unknown handle, INVALID_ARGUMENT for a terminal IO.
    Status testing_force_complete(const IoHandle& handle, IoState terminal, Status io_status = Status::Ok());

    // The DataPath-level identity an open target maps to (for callers that
    // drive a DataPath directly, e.g. the allocation-free C entry point).
    Result<DataPathTarget> data_path_target(const TargetHandle& handle) const;

    struct Impl;

private:
    explicit StorageRuntime(std::unique_ptr<Impl> impl);
    std::unique_ptr<Impl> impl_;
};

}  // namespace tutti
