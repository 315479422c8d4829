#pragma once
// TuttiRuntime: assembles a StorageRuntime from a TuttiRuntimeSpec.
//
// create(): validate -> resource (emulated controllers, or a queue lease from
// tutti_daemon for provider nvme-service) -> resolver (single / multi-mount /
// md RAID0) -> DataPath (GPU NVMe or POSIX) -> StorageRuntime::create_owning.
// A failure at any step undoes the earlier steps (lease released, controllers
// stopped). shutdown() runs in reverse order.
// Parity: reference csrc/tutti_runtime/tutti_runtime_create.cpp:92-330 and
// tutti_runtime.cpp (transactional create, reverse-order shutdown).

#include <memory>
#include <string>
#include <vector>

#include <tutti/storage_runtime.h>

#include "../config/runtime_spec.h"
#include "../daemon/daemon_client.h"
#include "../datapaths/gpu_nvme_data_path.h"
#include "../datapaths/posix_data_path.h"
#include "../nvme/controller.h"

namespace tutti {

class TuttiRuntime {
public:
    static Result<std::unique_ptr<TuttiRuntime>> create(const TuttiRuntimeSpec& spec);
    static Result<std::unique_ptr<TuttiRuntime>> create_from_file(const std::string& path);
    ~TuttiRuntime();

    StorageRuntime& storage() { return *runtime_; }
    std::unique_ptr<StorageRuntime> take_storage() { return std::move(runtime_); }
    const TuttiRuntimeSpec& spec() const { return spec_; }
    Status shutdown(std::uint64_t timeout_ms);

    std::vector<std::shared_ptr<nvme::NvmeController>> controllers;
    std::shared_ptr<GpuNvmeDataPath> gpu_path;
    std::shared_ptr<PosixDataPath> posix_path;
    std::shared_ptr<daemon::DaemonClient> lease;  // provider nvme-service only

private:
    TuttiRuntime() = default;
    TuttiRuntimeSpec spec_;
    std::unique_ptr<StorageRuntime> runtime_;
};

}  // namespace tutti
