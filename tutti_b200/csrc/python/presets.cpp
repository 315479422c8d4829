#include "presets.h"

#include "../nvme/snvme_client.h"
#include "../resolvers/file_resolvers.h"
#include "../testing/fake_snvme.h"

namespace tutti {

std::uint32_t probe_runtime_id(const StorageRuntime& rt) { return rt.runtime_id(); }

Result<PresetResult> make_emulated_nvme_runtime(const EmulatedPresetOptions& o) {
    using R = Result<PresetResult>;
    if (o.mounts.empty()) return R::Failure({StatusCode::INVALID_ARGUMENT, "at least one mount is required"});
    PresetResult pr;
    std::vector<GpuNvmeDevice> devs;
    std::size_t ndev = o.mounts.size();
    Raid0Geometry geo;
    if (!o.raid0_md.empty()) {
        auto g = probe_md_raid0(o.sysfs_root, o.raid0_md);
        if (!g.ok()) return R::Failure(g.status());
        geo = g.value();
        ndev = geo.members.size();
    }
    if (o.media != "files" && o.media != "memory")
        return R::Failure({StatusCode::INVALID_ARGUMENT, "emulated media must be 'files' or 'memory'"});
    if (o.provider != "emulated" && o.provider != "snvme" && o.provider != "snvme_fake")
        return R::Failure({StatusCode::INVALID_ARGUMENT, "provider must be 'emulated', 'snvme' or 'snvme_fake'"});
    if (o.provider == "snvme" && o.snvme_nodes.size() != ndev)
        return R::Failure({StatusCode::INVALID_ARGUMENT, "provider 'snvme' needs one snvme node per drive"});
    for (std::size_t i = 0; i < ndev; ++i) {
        nvme::EmulatedControllerConfig c;
        c.media = o.media == "memory" ? nvme::EmulatedControllerConfig::Media::MEMORY
                                      : nvme::EmulatedControllerConfig::Media::FILES;
        c.image_budget_bytes = o.image_budget_bytes;
        c.write_back = o.write_back && c.media == nvme::EmulatedControllerConfig::Media::MEMORY;
        c.max_gbps = o.drive_gbps;
        c.cuda_device = o.accel_id;
        c.name = "emu" + std::to_string(i);
        c.num_io_queues = o.queues ? o.queues : o.gpu.leases;
        c.queue_depth = o.queue_depth;
        c.lba_bytes = o.lba_bytes;
        c.mdts_bytes = o.mdts_bytes;
        c.worker_threads = o.controller_threads;
        c.direct_io = o.direct_io;
        c.skip_data = o.skip_data;
        c.map_reads = o.map_reads;
        c.idle_spin_iters = o.idle_spin_iters;
        std::shared_ptr<nvme::NvmeController> sp;
        if (o.provider == "emulated") {
            auto ctl = nvme::EmulatedNvmeController::create(c);
            if (!ctl.ok()) return R::Failure(ctl.status());
            sp = std::move(ctl).value();
        } else {
            nvme::SnvmeControllerConfig sc;
            sc.num_io_queues = c.num_io_queues;
            sc.rings_in_gpu_memory = o.snvme_rings_in_gpu_memory;
            sc.max_command_bytes = o.mdts_bytes;
            sc.namespace_bytes = c.namespace_bytes;
            sc.cuda_device = o.accel_id;
            std::shared_ptr<nvme::SnvmeSys> sys;
            if (o.provider == "snvme") {
                sc.node = o.snvme_nodes[i];
                sys = std::shared_ptr<nvme::SnvmeSys>(&nvme::linux_snvme_sys(), [](nvme::SnvmeSys*) {});
            } else {
                testing::FakeSnvmeConfig fc;
                fc.node = sc.node = "/dev/ssnvme" + std::to_string(i);
                fc.drive = c;
                auto fake = testing::FakeSnvmeDriver::create(fc);
                if (!fake.ok()) return R::Failure(fake.status());
                sys = std::shared_ptr<nvme::SnvmeSys>(std::move(fake).value());
            }
            auto ctl = nvme::SnvmeController::create(sc, std::move(sys));
            if (!ctl.ok()) return R::Failure(ctl.status());
            sp = std::move(ctl).value();
        }
        pr.extras.controllers.push_back(sp);
        devs.push_back({sp, c.name});
    }
    OwnedComponents comps;
    if (!o.raid0_md.empty()) {
        MountBinding b;
        b.mount_path = o.mounts[0];
        b.controller = "raid0";
        b.block_bytes = o.lba_bytes;
        b.datapath_key = "nvme-gpu";
        std::vector<std::string> ctrls;
        for (auto& d : devs) ctrls.push_back(d.identity);
        comps.resolvers.push_back({"file", std::make_unique<Raid0Resolver>(b, geo, ctrls)});
    } else {
        auto mm = std::make_unique<MultiMountResolver>();
        for (std::size_t i = 0; i < o.mounts.size(); ++i) {
            MountBinding b;
            b.mount_path = o.mounts[i];
            b.device_index = static_cast<std::uint32_t>(i);
            b.controller = devs[i].identity;
            b.block_bytes = o.lba_bytes;
            b.mapping = o.mapping;
            b.datapath_key = "nvme-gpu";
            Status s = mm->add(std::make_unique<LocalFileResolver>(b), o.mounts[i]);
            if (!s.ok()) return R::Failure(s);
        }
        comps.resolvers.push_back({"file", std::move(mm)});
    }
    GpuNvmeConfig g = o.gpu;
    g.accel_id = o.accel_id;
    // Memory media DMA each command straight into HBM staging; file media keep
    // page-locked host staging (their device DMA would go through a bounce).
    if (g.staging == GpuNvmeConfig::Staging::AUTO)
        g.staging = o.media == "memory" ? GpuNvmeConfig::Staging::DEVICE : GpuNvmeConfig::Staging::HOST;
    if (g.staging == GpuNvmeConfig::Staging::DEVICE && !cuda_device_present())
        g.staging = GpuNvmeConfig::Staging::HOST;
    auto path = std::make_shared<GpuNvmeDataPath>(g, devs);
    pr.extras.gpu_path = path;
    comps.data_paths.push_back({"nvme-gpu", path, DataPathConfig{"nvme-gpu"}});
    for (auto& c : pr.extras.controllers) comps.keep_alive.push_back(c);
    RuntimeConfig rc;
    rc.accel_id = o.accel_id;
    rc.max_terminal_results = o.max_terminal_results;
    auto rt = StorageRuntime::create_owning(rc, std::move(comps));
    if (!rt.ok()) return R::Failure(rt.status());
    pr.runtime = std::move(rt).value();
    pr.runtime_id = pr.runtime->runtime_id();
    return pr;
}

Result<PresetResult> make_posix_runtime(const PosixPresetOptions& o) {
    using R = Result<PresetResult>;
    if (o.mounts.empty()) return R::Failure({StatusCode::INVALID_ARGUMENT, "at least one mount is required"});
    PresetResult pr;
    OwnedComponents comps;
    auto mm = std::make_unique<MultiMountResolver>();
    for (std::size_t i = 0; i < o.mounts.size(); ++i) {
        MountBinding b;
        b.mount_path = o.mounts[i];
        b.device_index = static_cast<std::uint32_t>(i);
        b.controller = "posix" + std::to_string(i);
        b.mapping = "synthetic";
        b.datapath_key = "posix";
        Status s = mm->add(std::make_unique<LocalFileResolver>(b), o.mounts[i]);
        if (!s.ok()) return R::Failure(s);
    }
    comps.resolvers.push_back({"file", std::move(mm)});
    PosixConfig pc = o.posix;
    pc.accel_id = o.accel_id;
    auto path = std::make_shared<PosixDataPath>(pc);
    pr.extras.posix_path = path;
    comps.data_paths.push_back({"posix", path, DataPathConfig{"posix"}});
    RuntimeConfig rc;
    rc.accel_id = o.accel_id < 0 ? 0 : o.accel_id;
    rc.max_terminal_results = o.max_terminal_results;
    auto rt = StorageRuntime::create_owning(rc, std::move(comps));
    if (!rt.ok()) return R::Failure(rt.status());
    pr.runtime = std::move(rt).value();
    pr.runtime_id = pr.runtime->runtime_id();
    return pr;
}

Result<PresetResult> make_memfs_runtime(const MemfsPresetOptions& o) {
    using R = Result<PresetResult>;
    if (!o.capacity_bytes) return R::Failure({StatusCode::INVALID_ARGUMENT, "memfs needs a capacity"});
    PresetResult pr;
    OwnedComponents comps;
    auto budget = std::make_shared<samples::memfs::MemoryResource>(o.capacity_bytes);
    auto resolver = std::make_unique<samples::memfs::Resolver>(budget);
    pr.extras.memfs_resolver = resolver.get();
    pr.extras.memfs_budget = budget;
    comps.resolvers.push_back({"memfs", std::move(resolver)});
    comps.data_paths.push_back({samples::memfs::kDataPathKey, std::make_shared<samples::memfs::MemfsDataPath>(),
                                DataPathConfig{samples::memfs::kDataPathKey}});
    RuntimeConfig rc;
    rc.accel_id = o.accel_id < 0 ? 0 : o.accel_id;
    rc.max_terminal_results = o.max_terminal_results;
    auto rt = StorageRuntime::create_owning(rc, std::move(comps));
    if (!rt.ok()) return R::Failure(rt.status());
    pr.runtime = std::move(rt).value();
    pr.runtime_id = pr.runtime->runtime_id();
    return pr;
}

}  // namespace tutti
