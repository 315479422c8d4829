#pragma once
// PosixDataPath ("posix"): HOST_EXECUTION pread/pwrite against resolved files,
// O_DIRECT when the request and buffer are block aligned, buffered otherwise.
// Device memory is reached through page-locked bounce buffers and
// cudaMemcpyAsync (the CPU-centric path the GPU io kernel is compared with).
// The reference reserves HOST_EXECUTION but ships no such DataPath
// (doc/architecture/system-architecture.md:37-38).

#include <atomic>
#include <condition_variable>
#include <deque>
#include <memory>
#include <mutex>
#include <thread>
#include <unordered_map>
#include <vector>

#include <tutti/payloads.h>
#include <tutti/spi/data_path.h>
#include <tutti/spi/resolver.h>

namespace tutti {

struct PosixConfig {
    std::uint32_t threads = 8;
    std::uint32_t bounce_bytes = 4u << 20;  // per worker, for device memory
    bool direct_io = true;
    std::int32_t accel_id = -1;             // device used for bounce copies
    // Test seam: fail the n-th executed request with an IO error (0 = off).
    std::uint64_t inject_fail_every = 0;
};

class PosixDataPath final : public DataPath {
public:
    explicit PosixDataPath(PosixConfig cfg);
    ~PosixDataPath() override;
    const DataPathCapabilities& capabilities() const override { return caps_; }
    Status initialize(const DataPathConfig& config, ResourceProvider* resources) override;
    Status shutdown(std::uint64_t timeout_ns) override;
    Result<DataPathTarget> open(const ResolvedTarget& target) override;
    Status close(DataPathTarget target) override;
    Result<RegistrationDomainKey> registration_domain(DataPathTarget target) const override;
    Result<DataPathMemory> register_memory(const DataPathMemoryView& view,
                                           const RegistrationDomainKey& domain) override;
    Status unregister_memory(DataPathMemory memory) override;
    SubmitOutcome submit(const DataPathRequest* requests, std::size_t count,
                         const HostSubmitContext& ctx) override;
    Result<ProgressResult> progress(ProgressBudget budget) override;
    Result<DataPathSnapshot> query(DataPathOp op) const override;
    Status release(DataPathOp op) override;

private:
    struct Target {
        std::uint64_t gen = 0;
        int fd_direct = -1, fd_buffered = -1;
        std::uint64_t size = 0;
    };
    struct Mem {
        std::uint64_t gen = 0;
        char* base = nullptr;
        std::uint64_t size = 0;
        DataPathMemoryKind kind = DataPathMemoryKind::HOST;
    };
    struct Task {
        std::uint64_t op;
        std::uint32_t index;
        IoDirection dir;
        int fd_direct, fd_buffered;
        std::uint64_t foff, len;
        char* mem;
        bool device;
    };
    struct Op {
        std::uint64_t gen = 0;
        std::atomic<std::uint32_t> remaining{0};
        std::mutex mu;
        std::vector<std::uint32_t> failed;
        std::uint64_t ok_bytes = 0;
        std::uint32_t n = 0;
    };
    void worker();
    bool run(const Task& t, char* bounce);

    PosixConfig cfg_;
    DataPathCapabilities caps_;
    mutable std::mutex mu_;
    std::unordered_map<std::uint64_t, Target> targets_;
    std::unordered_map<std::uint64_t, Mem> mems_;
    std::unordered_map<std::uint64_t, std::shared_ptr<Op>> ops_;
    std::uint64_t next_ = 1;
    std::mutex qmu_;
    std::condition_variable qcv_;
    std::deque<Task> queue_;
    std::vector<std::thread> workers_;
    bool stop_ = false;
    bool initialized_ = false;
    std::atomic<std::uint64_t> executed_{0};
};

}  // namespace tutti
