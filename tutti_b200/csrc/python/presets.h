#pragma once
// Daemon-less preset assembly used by the Python package (reference
// csrc/presets/local_nvme_preset.cpp:71,141 and include/tutti/presets/local_nvme.h):
// one emulated controller per backing mount (or per RAID0 member), a
// multi-mount FIEMAP resolver, and the GPU NVMe DataPath; or the POSIX
// host-execution DataPath over the same resolvers.

#include <memory>
#include <string>
#include <vector>

#include <tutti/storage_runtime.h>

#include "../datapaths/gpu_nvme_data_path.h"
#include "../datapaths/posix_data_path.h"
#include "../samples/memfs/memfs.h"
#include "../nvme/controller.h"

namespace tutti {

struct EmulatedPresetOptions {
    int accel_id = 0;
    std::vector<std::string> mounts;   // one drive per mount
    // Which controller answers each mount's queues:
    //   "emulated":   an EmulatedNvmeController (its own rings and doorbells);
    //   "snvme":      a real controller through the snvme driver, node snvme_nodes[i];
    //   "snvme_fake": the snvme client over a fake driver whose hardware is an
    //                 emulated drive (the real-drive code path without the drive).
    std::string provider = "emulated";
    std::vector<std::string> snvme_nodes;
    bool snvme_rings_in_gpu_memory = false;
    std::uint32_t queues = 0;          // 0: = leases
    std::uint32_t queue_depth = 256;
    std::uint32_t mdts_bytes = 1u << 20;
    std::uint32_t lba_bytes = 512;
    std::uint32_t controller_threads = 4;
    bool direct_io = false;
    bool skip_data = false;  // diagnostic: controllers move no data
    bool map_reads = false;  // page-cached reads copy from a file mapping (default: pread)
    std::uint32_t idle_spin_iters = 2000;  // queue scans before an idle worker starts sleeping
    // Emulated drives' media: "files" (pread/pwrite) or "memory" (a page-locked
    // image of the backing files, loaded on first touch, written through).
    std::string media = "files";
    std::uint64_t image_budget_bytes = 0;  // 0: no limit
    bool write_back = false;  // memory media: a volatile write cache (durable on flush)
    double drive_gbps = 0.0;               // per-drive transfer cap (0: none)
    std::string mapping = "auto";      // fiemap | synthetic | auto
    std::string raid0_md;              // non-empty: mounts[0] is an md RAID0 array
    std::string sysfs_root = "/sys";
    std::uint64_t max_terminal_results = 64;
    GpuNvmeConfig gpu;
};

struct PosixPresetOptions {
    int accel_id = -1;
    std::vector<std::string> mounts;
    std::uint64_t max_terminal_results = 64;
    PosixConfig posix;
};

struct MemfsPresetOptions {
    int accel_id = -1;
    std::uint64_t capacity_bytes = 1ull << 30;
    std::uint64_t max_terminal_results = 64;
};

struct PresetExtras {
    std::vector<std::shared_ptr<nvme::NvmeController>> controllers;
    std::shared_ptr<GpuNvmeDataPath> gpu_path;
    std::shared_ptr<PosixDataPath> posix_path;
    std::shared_ptr<samples::memfs::MemoryResource> memfs_budget;
    samples::memfs::Resolver* memfs_resolver = nullptr;  // owned by the runtime's components
};

struct PresetResult {
    std::unique_ptr<StorageRuntime> runtime;
    PresetExtras extras;
    std::uint32_t runtime_id = 0;
};

Result<PresetResult> make_emulated_nvme_runtime(const EmulatedPresetOptions& o);
Result<PresetResult> make_posix_runtime(const PosixPresetOptions& o);
// The memfs sample backend (scheme memfs://, DataPath key memfs) and nothing else.
Result<PresetResult> make_memfs_runtime(const MemfsPresetOptions& o);
std::uint32_t probe_runtime_id(const StorageRuntime& rt);

}  // namespace tutti
