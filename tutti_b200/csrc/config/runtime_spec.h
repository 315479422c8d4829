#pragma once
// TuttiRuntimeSpec: the native runtime configuration (YAML), its parser and
// validation.
//
// Schema (parity with the reference's config/storage_runtime/*.yaml and
// csrc/config/spec/tutti_runtime_spec.cpp): top-level `accelerator`,
// `runtime`, `storage` with lists `resources`, `resolvers`, `datapaths`,
// `backends`. Unknown fields are errors that name their YAML path; ids must
// be unique; a backend's references must exist; the backend's contract fixes
// which resolver/datapath/resource types may be combined; exactly one backend.
//
// Contracts:
//   nvme-device-group  local-file resolver (single | multi-mount | raid0)
//                      + nvme-device-group or local-nvme datapath + nvme resource
//   ext4-local-nvme    local-file resolver (single) + local-nvme datapath
//                      + nvme resource with exactly one device
//   posix              local-file resolver + posix datapath (+ optional resource)

#include <cstdint>
#include <string>
#include <vector>

#include <tutti/status.h>

#include "yaml_lite.h"

namespace tutti {

struct ResourceSpec {
    std::string id;
    std::string type;         // nvme | memory
    std::string provider;     // emulated | nvme-service
    std::string endpoint;     // nvme-service: UNIX socket path of the daemon
    std::string selection = "device-group";  // device-group | single
    std::vector<std::int64_t> device_ids;
    std::uint32_t queues_per_controller = 0;  // 0: provider default
    std::vector<std::string> mounts;          // emulated: one backing mount per device
    std::uint32_t queue_depth = 256;
    std::uint32_t mdts_bytes = 1u << 20;
    std::uint32_t lba_bytes = 512;
    std::uint32_t controller_threads = 4;
    bool direct_io = false;
    std::string client = "tutti";             // nvme-service lease holder name
};

struct ResolverSpec {
    std::string id;
    std::string type;                 // local-file
    std::string scheme = "file";
    std::string topology = "single";  // single | multi-mount | raid0
    std::string mapping = "auto";     // auto | fiemap | synthetic
    std::string md;                   // raid0: md device name (e.g. md0)
    std::string sysfs_root = "/sys";
};

struct DataPathSpec {
    std::string id;
    std::string type;  // nvme-device-group | local-nvme | posix
    std::uint32_t leases = 64;
    std::uint32_t max_ctas_per_op = 64;
    std::uint32_t slots_per_lease = 8;
    bool async_completion = false;  // nvme-gpu: split submit / drain launches for reads
    std::uint32_t slot_bytes = 1u << 20;
    std::uint64_t timeout_ms = 5000;
    std::uint32_t threads = 8;  // posix
    bool direct_io = true;      // posix
};

struct BackendSpec {
    std::string id;
    std::string contract;
    std::string resolver;
    std::string datapath;
    std::string resource;  // may be empty for posix
};

struct TuttiRuntimeSpec {
    std::string profile = "CUDA";
    std::int32_t accel_id = 0;
    std::uint64_t max_terminal_results = 64;
    std::vector<ResourceSpec> resources;
    std::vector<ResolverSpec> resolvers;
    std::vector<DataPathSpec> datapaths;
    std::vector<BackendSpec> backends;

    const ResourceSpec* resource(const std::string& id) const;
    const ResolverSpec* resolver(const std::string& id) const;
    const DataPathSpec* datapath(const std::string& id) const;
};

Result<TuttiRuntimeSpec> parse_runtime_spec(const yaml::Node& root);
Result<TuttiRuntimeSpec> parse_runtime_config_file(const std::string& path);
Result<TuttiRuntimeSpec> parse_runtime_config_text(const std::string& text);
Status validate_runtime_spec(const TuttiRuntimeSpec& spec);

}  // namespace tutti
