#include "tutti_runtime.h"

#include "../resolvers/file_resolvers.h"

namespace tutti {

namespace {

struct DeviceRow {
    std::string mount;
    std::uint32_t queues = 0;
    std::uint32_t lba_bytes = 512;
};

}  // namespace

Result<std::unique_ptr<TuttiRuntime>> TuttiRuntime::create_from_file(const std::string& path) {
    auto spec = parse_runtime_config_file(path);
    if (!spec.ok()) return Result<std::unique_ptr<TuttiRuntime>>::Failure(spec.status());
    return create(spec.value());
}

Result<std::unique_ptr<TuttiRuntime>> TuttiRuntime::create(const TuttiRuntimeSpec& spec) {
    using R = Result<std::unique_ptr<TuttiRuntime>>;
    TUTTI_RETURN_IF_ERROR_R(R, validate_runtime_spec(spec));
    std::unique_ptr<TuttiRuntime> rt(new TuttiRuntime());
    rt->spec_ = spec;
    const BackendSpec& b = spec.backends[0];
    const ResolverSpec& rs = *spec.resolver(b.resolver);
    const DataPathSpec& ds = *spec.datapath(b.datapath);
    const ResourceSpec* res = b.resource.empty() ? nullptr : spec.resource(b.resource);

    // 1) resource: which devices, where they are mounted, how many queues
    std::vector<DeviceRow> rows;
    if (res && res->type == "nvme") {
        if (res->provider == "emulated") {
            for (auto& m : res->mounts)
                rows.push_back({m, res->queues_per_controller ? res->queues_per_controller : ds.leases, res->lba_bytes});
        } else {  // nvme-service
            auto client = std::make_shared<daemon::DaemonClient>();
            TUTTI_RETURN_IF_ERROR_R(R, client->connect(res->endpoint, res->client, spec.accel_id));
            const std::uint32_t want = res->queues_per_controller ? res->queues_per_controller : ds.leases;
            auto grant = client->acquire(res->device_ids, want);
            if (!grant.ok()) return R::Failure(grant.status());
            client->start_heartbeat(5000);
            rt->lease = client;  // released by ~TuttiRuntime on any later failure
            for (std::size_t i = 0; i < grant.value().devices.size(); ++i)
                rows.push_back({grant.value().mounts[i], grant.value().queues,
                                i < grant.value().lba_bytes.size() ? grant.value().lba_bytes[i] : 512});
        }
    } else if (res && res->type == "memory") {
        rows.push_back({res->mounts.empty() ? std::string("/") : res->mounts[0], 0, 512});
    }

    OwnedComponents comps;
    const bool gpu = ds.type == "nvme-device-group" || ds.type == "local-nvme";
    std::vector<GpuNvmeDevice> devs;
    if (gpu) {
        if (rows.empty()) return R::Failure({StatusCode::INVALID_ARGUMENT, "nvme datapath without devices"});
        for (std::size_t i = 0; i < rows.size(); ++i) {
            nvme::EmulatedControllerConfig c;
            c.name = "emu" + std::to_string(i);
            c.num_io_queues = std::max<std::uint32_t>(rows[i].queues, 1);
            c.queue_depth = res->queue_depth;
            c.lba_bytes = rows[i].lba_bytes;
            c.mdts_bytes = res->mdts_bytes;
            c.worker_threads = res->controller_threads;
            c.direct_io = res->direct_io;
            auto ctl = nvme::EmulatedNvmeController::create(c);
            if (!ctl.ok()) return R::Failure(ctl.status());
            std::shared_ptr<nvme::NvmeController> sp(std::move(ctl).value());
            rt->controllers.push_back(sp);
            devs.push_back({sp, c.name});
        }
    }
    // 2) resolver
    const std::string key = gpu ? "nvme-gpu" : "posix";
    if (rs.topology == "raid0") {
        std::string md = rs.md;
        if (md.empty()) {  // the array behind the resource's mount
            if (rows.empty()) return R::Failure({StatusCode::INVALID_ARGUMENT, "raid0 resolver has no mount"});
            auto found = find_md_array(rs.sysfs_root, rows[0].mount);
            if (!found.ok()) return R::Failure(found.status());
            md = found.value();
        }
        auto geo = probe_md_raid0(rs.sysfs_root, md);
        if (!geo.ok()) return R::Failure(geo.status());
        MountBinding mb;
        mb.mount_path = rows.empty() ? "/" : rows[0].mount;
        mb.controller = "raid0";
        mb.datapath_key = key;
        std::vector<std::string> ids;
        for (auto& d : devs) ids.push_back(d.identity);
        comps.resolvers.push_back({rs.scheme, std::make_unique<Raid0Resolver>(mb, geo.value(), ids)});
    } else {
        auto mm = std::make_unique<MultiMountResolver>();
        const std::size_t n = rs.topology == "single" ? std::min<std::size_t>(1, rows.size()) : rows.size();
        if (n == 0) return R::Failure({StatusCode::INVALID_ARGUMENT, "resolver has no mount"});
        for (std::size_t i = 0; i < n; ++i) {
            MountBinding mb;
            mb.mount_path = rows[i].mount;
            mb.device_index = static_cast<std::uint32_t>(i);
            mb.controller = gpu ? devs[i].identity : "posix" + std::to_string(i);
            mb.block_bytes = rows[i].lba_bytes;
            mb.mapping = gpu ? rs.mapping : "synthetic";
            mb.datapath_key = key;
            TUTTI_RETURN_IF_ERROR_R(R, mm->add(std::make_unique<LocalFileResolver>(mb), rows[i].mount));
        }
        comps.resolvers.push_back({rs.scheme, std::move(mm)});
    }
    // 3) datapath
    if (gpu) {
        GpuNvmeConfig g;
        g.accel_id = spec.accel_id;
        g.leases = ds.leases;
        for (auto& r : rows) g.leases = std::min(g.leases, std::max<std::uint32_t>(r.queues, 1));
        g.max_ctas_per_op = std::min(ds.max_ctas_per_op, g.leases);
        g.slots_per_lease = ds.slots_per_lease;
        g.async_completion = ds.async_completion;
        g.slot_bytes = ds.slot_bytes;
        g.timeout_ns = ds.timeout_ms * 1000000ull;
        rt->gpu_path = std::make_shared<GpuNvmeDataPath>(g, devs);
        comps.data_paths.push_back({key, rt->gpu_path, DataPathConfig{ds.id}});
    } else {
        PosixConfig pc;
        pc.threads = ds.threads;
        pc.direct_io = ds.direct_io;
        pc.accel_id = spec.accel_id;
        rt->posix_path = std::make_shared<PosixDataPath>(pc);
        comps.data_paths.push_back({key, rt->posix_path, DataPathConfig{ds.id}});
    }
    for (auto& c : rt->controllers) comps.keep_alive.push_back(c);
    // 4) runtime
    RuntimeConfig rc;
    rc.accel_id = spec.accel_id;
    rc.max_terminal_results = spec.max_terminal_results;
    rc.profile_name = spec.profile;
    auto sr = StorageRuntime::create_owning(rc, std::move(comps));
    if (!sr.ok()) return R::Failure(sr.status());
    rt->runtime_ = std::move(sr).value();
    return R(std::move(rt));
}

Status TuttiRuntime::shutdown(std::uint64_t timeout_ms) {
    Status first;
    if (runtime_) {
        first = runtime_->shutdown(timeout_ms);
        runtime_.reset();
    }
    gpu_path.reset();
    posix_path.reset();
    for (auto& c : controllers)
        if (auto* e = c->emulated_drive()) e->stop();
    controllers.clear();
    if (lease) {
        Status s = lease->release();
        lease->close();
        lease.reset();
        if (first.ok() && !s.ok()) first = s;
    }
    return first;
}

TuttiRuntime::~TuttiRuntime() { shutdown(1000); }

}  // namespace tutti
