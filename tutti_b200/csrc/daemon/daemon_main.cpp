// tutti_daemon: host-level owner of the NVMe devices; GPU processes lease
// I/O queues from it over a UNIX socket.
//
//   tutti_daemon --config daemon.yaml
//
// Config:
//   service: {socket: /run/tutti/daemon.sock}
//   lease:   {heartbeat_timeout_s: 30, reap_interval_ms: 1000}
//   queue_pool: {default_per_client: 16, max_per_client: 32}   # optional
//   devices:   # or Tutti's nvmes: [{device_id, backing_mount_path, pci_addr, namespace_id,
//              #   allowed_accel_ids (empty: every accelerator of Tutti's accelerators: list),
//              #   kernel_ioq_cap, auto_mount, block_device}]
//     - {id: 0, kind: emulated, mount: /mnt/nvme0, queues: 128, pci: "0000:1b:00.0", nsid: 1, lba_bytes: 512,
//        accelerators: [0, 1]}   # optional: only these GPUs may lease its queues
//   accelerators: [{accel_id: 0, view_root: /run/tutti/gpu0}]   # per-accelerator links to the mounts
//   raid0_arrays: [{name: kv, device_ids: [0, 1], mount_path: /mnt/kv, auto_mount: true}]
//   unmount_retry: {interval_ms: 1000, max: 30}
//   snvme: {control: /dev/snvm_control, own_controllers: false}
//
// Bring-up, in order: with snvme.own_controllers, each nvme with a pci_addr
// is bound to the snvme driver and its node created (its block device comes
// from the namespace scan); RAID0 arrays are assembled from their members'
// block devices and mounted; drives with auto_mount and a known block device
// are mounted (or an existing mount of the same device adopted); each
// accelerator's view root gets one link per drive it may use. A step that
// fails marks the drive unavailable with a diagnostic (LIST_RESOURCES) and
// the daemon serves the rest. Shutdown undoes it in reverse: the daemon's own
// mounts (busy ones retried, their holders reported; a second signal stops
// the retries), the arrays it assembled, the controllers it bound.
//
// Protocol: one request per line (see lease_ledger.h); a connection that
// closes ends nothing by itself - leases end by RELEASE, BYE, heartbeat
// expiry, or when the reaper finds the client's process gone.
// Parity: reference examples/tutti_daemon.cpp + nvmeservice (gRPC service,
// mount manager, leases with heartbeat and PID/starttime reaper). gRPC and
// protobuf are not used: the control plane is this line protocol.

#include <signal.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <map>
#include <memory>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "../config/yaml_lite.h"
#include "../nvme/snvme_client.h"
#include "host_admin.h"
#include "lease_ledger.h"

using namespace tutti;
using namespace tutti::daemon;

namespace {
std::atomic<bool> g_stop{false};
std::atomic<MountManager*> g_mounts{nullptr};
void on_signal(int) {
    // a second signal during shutdown stops the unmount retries
    if (g_stop.exchange(true))
        if (MountManager* m = g_mounts.load()) m->request_force_exit();
}

void serve_connection(int fd, LeaseLedger* ledger) {
    std::string buf;
    char tmp[4096];
    while (!g_stop.load()) {
        const ssize_t n = ::read(fd, tmp, sizeof(tmp));
        if (n <= 0) break;
        buf.append(tmp, static_cast<std::size_t>(n));
        std::size_t nl;
        while ((nl = buf.find('\n')) != std::string::npos) {
            const std::string line = buf.substr(0, nl);
            buf.erase(0, nl + 1);
            const std::string rsp = handle_request(*ledger, line);
            std::size_t off = 0;
            while (off < rsp.size()) {
                const ssize_t w = ::write(fd, rsp.data() + off, rsp.size() - off);
                if (w <= 0) break;
                off += static_cast<std::size_t>(w);
            }
        }
    }
    ::close(fd);
}

int fail(const std::string& m) {
    std::fprintf(stderr, "tutti_daemon: %s\n", m.c_str());
    return 2;
}
}  // namespace

int main(int argc, char** argv) {
    std::string config;
    for (int i = 1; i + 1 < argc; ++i)
        if (std::string(argv[i]) == "--config") config = argv[i + 1];
    if (config.empty()) return fail("usage: tutti_daemon --config <daemon.yaml>");
    auto root = yaml::parse_file(config);
    if (!root.ok()) return fail(root.status().to_string());
    const yaml::Node& r = *root.value();
    std::string socket_path = "/tmp/tutti_daemon.sock";
    std::int64_t hb_timeout = 30, reap_ms = 1000;
    std::uint32_t pool_default = 0, pool_max = 0;
    auto int_of = [](const yaml::Node* n, const std::string& path, std::int64_t& out) -> Status {
        if (!n) return Status::Ok();
        auto v = yaml::as_int(*n, path);
        if (!v.ok()) return v.status();
        out = v.value();
        return Status::Ok();
    };
    Status st;
    if (const auto* s = r.get("service"))
        if (const auto* p = s->get("socket")) socket_path = p->scalar;
    if (const auto* l = r.get("lease")) {
        if (st.ok()) st = int_of(l->get("heartbeat_timeout_s"), "lease.heartbeat_timeout_s", hb_timeout);
        if (st.ok()) st = int_of(l->get("timeout_sec"), "lease.timeout_sec", hb_timeout);  // Tutti's key
        if (st.ok()) st = int_of(l->get("reap_interval_ms"), "lease.reap_interval_ms", reap_ms);
    }
    if (const auto* q = r.get("queue_pool")) {  // Tutti's per-client queue policy
        std::int64_t d = 0, m = 0;
        if (st.ok()) st = int_of(q->get("default_per_client"), "queue_pool.default_per_client", d);
        if (st.ok()) st = int_of(q->get("max_per_client"), "queue_pool.max_per_client", m);
        pool_default = static_cast<std::uint32_t>(d);
        pool_max = static_cast<std::uint32_t>(m);
    }
    if (!st.ok()) return fail(st.to_string());
    if (r.get("nvmes") && !r.get("queue_pool")) {  // Tutti's parser defaults
        pool_default = 4;
        pool_max = 32;
    }
    if (r.get("grpc") && !r.get("service"))
        std::fprintf(stderr, "tutti_daemon: grpc.endpoint is not served (line protocol on %s)\n", socket_path.c_str());

    // Devices: this daemon's schema (devices: [{id, kind, mount, pci, queues, nsid, lba_bytes,
    // accelerators}]) or Tutti's (nvmes: [{device_id, backing_mount_path, pci_addr, namespace_id,
    // kernel_ioq_cap, allowed_accel_ids}]).
    std::vector<std::int64_t> configured_accels;  // Tutti's accelerators: [{accel_id, view_root}]
    std::vector<AcceleratorView> views;
    if (const auto* acc = r.get("accelerators")) {
        if (!acc->is_seq()) return fail("config: accelerators: expected a list");
        for (std::size_t i = 0; i < acc->seq.size(); ++i) {
            std::int64_t a = -1;
            st = int_of(acc->seq[i]->get("accel_id"), "accelerators[" + std::to_string(i) + "].accel_id", a);
            if (!st.ok()) return fail(st.to_string());
            if (a >= 0) configured_accels.push_back(a);
            AcceleratorView v;
            v.id = a;
            if (const auto* vr = acc->seq[i]->get("view_root")) v.view_root = vr->scalar;
            if (a >= 0) views.push_back(v);
        }
    }
    struct DriveExtras {
        bool auto_mount = false;
        std::uint32_t kernel_ioq_cap = 0;
    };
    std::map<std::int64_t, DriveExtras> extras;
    auto bool_of = [](const yaml::Node* n, const std::string& path, bool& out) -> Status {
        if (!n) return Status::Ok();
        auto v = yaml::as_bool(*n, path);
        if (!v.ok()) return v.status();
        out = v.value();
        return Status::Ok();
    };
    std::vector<DeviceInfo> devices;
    auto parse_list = [&](const yaml::Node& list, const std::string& name, bool tutti) -> Status {
        if (!list.is_seq()) return {StatusCode::INVALID_ARGUMENT, "config: " + name + ": expected a list"};
        for (std::size_t i = 0; i < list.seq.size(); ++i) {
            const yaml::Node& d = *list.seq[i];
            const std::string p = name + "[" + std::to_string(i) + "]";
            DeviceInfo info;
            info.kind = tutti ? "nvme" : "emulated";
            const yaml::Node* id = d.get(tutti ? "device_id" : "id");
            if (!id) return {StatusCode::INVALID_ARGUMENT, p + ": id required"};
            std::int64_t v = 0;
            TUTTI_RETURN_IF_ERROR(int_of(id, p + ".id", v));
            info.id = v;
            if (auto k = d.get("kind")) info.kind = k->scalar;
            if (auto b = d.get("block_device")) info.block_device = b->scalar;
            DriveExtras ex;
            ex.auto_mount = tutti;  // Tutti mounts its drives unless told not to
            TUTTI_RETURN_IF_ERROR(bool_of(d.get("auto_mount"), p + ".auto_mount", ex.auto_mount));
            std::int64_t cap = 0;
            TUTTI_RETURN_IF_ERROR(int_of(d.get("kernel_ioq_cap"), p + ".kernel_ioq_cap", cap));
            ex.kernel_ioq_cap = static_cast<std::uint32_t>(cap);
            if (auto m = d.get(tutti ? "backing_mount_path" : "mount")) info.mount = m->scalar;
            if (auto c = d.get(tutti ? "pci_addr" : "pci")) info.pci = c->scalar;
            // Tutti's kernel_ioq_cap is a kernel block-IO hint, not the queues offered to clients
            v = info.queues;
            if (!tutti) TUTTI_RETURN_IF_ERROR(int_of(d.get("queues"), p + ".queues", v));
            info.queues = static_cast<std::uint32_t>(v);
            v = info.namespace_id;
            TUTTI_RETURN_IF_ERROR(int_of(d.get(tutti ? "namespace_id" : "nsid"), p + ".nsid", v));
            info.namespace_id = static_cast<std::uint32_t>(v);
            v = info.lba_bytes;
            TUTTI_RETURN_IF_ERROR(int_of(d.get("lba_bytes"), p + ".lba_bytes", v));
            info.lba_bytes = static_cast<std::uint32_t>(v);
            if (auto a = d.get(tutti ? "allowed_accel_ids" : "accelerators")) {
                if (!a->is_seq()) return {StatusCode::INVALID_ARGUMENT, p + ".accelerators: expected a list of ids"};
                for (std::size_t k = 0; k < a->seq.size(); ++k) {
                    TUTTI_RETURN_IF_ERROR(int_of(a->seq[k].get(), p + ".accelerators[" + std::to_string(k) + "]", v));
                    info.accelerators.push_back(v);
                }
            }
            // Tutti: an empty allowed_accel_ids means every accelerator the file configures
            if (tutti && info.accelerators.empty()) info.accelerators = configured_accels;
            if (info.kind != "emulated" && info.kind != "nvme")
                return {StatusCode::INVALID_ARGUMENT, p + ".kind must be emulated or nvme"};
            extras[info.id] = ex;
            devices.push_back(info);
        }
        return Status::Ok();
    };
    const auto* devs = r.get("devices");
    const auto* nvmes = r.get("nvmes");
    if (!devs && !nvmes) return fail("config: devices (or nvmes): expected a list");
    if (devs) st = parse_list(*devs, "devices", false);
    if (st.ok() && nvmes) st = parse_list(*nvmes, "nvmes", true);
    if (!st.ok()) return fail(st.to_string());

    // Host administration: controllers, arrays, mounts, accelerator views.
    std::string control_node = "/dev/snvm_control";
    bool own_controllers = false;
    if (const auto* sv = r.get("snvme")) {
        if (const auto* c = sv->get("control")) control_node = c->scalar;
        st = bool_of(sv->get("own_controllers"), "snvme.own_controllers", own_controllers);
        if (!st.ok()) return fail(st.to_string());
    }
    std::int64_t retry_ms = 1000, retry_max = 30;
    if (const auto* u = r.get("unmount_retry")) {
        if (st.ok()) st = int_of(u->get("interval_ms"), "unmount_retry.interval_ms", retry_ms);
        if (st.ok()) st = int_of(u->get("max"), "unmount_retry.max", retry_max);
        if (!st.ok()) return fail(st.to_string());
    }
    std::int64_t hb_interval = 10;
    if (const auto* l = r.get("lease")) {
        st = int_of(l->get("heartbeat_interval_sec"), "lease.heartbeat_interval_sec", hb_interval);
        if (!st.ok()) return fail(st.to_string());
    }
    auto find_device = [&](std::int64_t id) -> DeviceInfo* {
        for (auto& d : devices)
            if (d.id == id) return &d;
        return nullptr;
    };
    auto mark = [](DeviceInfo& d, const std::string& why) {
        d.available = false;
        d.diagnostic = d.diagnostic.empty() ? why : d.diagnostic + "; " + why;
        std::fprintf(stderr, "tutti_daemon: device %lld unavailable: %s\n", static_cast<long long>(d.id), why.c_str());
    };
    std::vector<std::unique_ptr<nvme::SnvmeOwner>> owners;
    if (own_controllers) {
        for (auto& d : devices) {
            if (d.kind != "nvme" || d.pci.empty()) continue;
            auto o = nvme::SnvmeOwner::bring_up(control_node, d.pci, extras[d.id].kernel_ioq_cap, nvme::linux_snvme_sys());
            if (!o.ok()) {
                mark(d, "controller bring-up: " + o.status().to_string());
                continue;
            }
            d.chrdev = o.value()->node();
            d.block_device = o.value()->block_device();
            d.queue_depth = o.value()->info().queue_depth;
            d.max_data_size = o.value()->info().max_transfer_bytes;
            d.max_queues_per_group = o.value()->info().max_queues_per_group;
            d.lba_bytes = o.value()->info().lba_bytes;
            d.max_user_qid = o.value()->info().last_user_qid;
            d.chrdev_minor = o.value()->minor();
            std::uint32_t stride_log = 0;
            while ((4u << stride_log) < o.value()->info().doorbell_stride && stride_log < 15) ++stride_log;
            d.doorbell_stride = stride_log;
            owners.push_back(std::move(o).value());
        }
    }
    MountManager mounts(linux_host_sys(), static_cast<std::uint32_t>(retry_ms), static_cast<std::uint32_t>(retry_max));
    g_mounts.store(&mounts);
    std::map<std::int64_t, bool> in_array;
    if (const auto* arrays = r.get("raid0_arrays")) {
        if (!arrays->is_seq()) return fail("config: raid0_arrays: expected a list");
        for (std::size_t i = 0; i < arrays->seq.size(); ++i) {
            const yaml::Node& a = *arrays->seq[i];
            const std::string p = "raid0_arrays[" + std::to_string(i) + "]";
            const std::string name = a.get("name") ? a.get("name")->scalar : "";
            const std::string mp = a.get("mount_path") ? a.get("mount_path")->scalar : "";
            bool auto_mount = true;
            st = bool_of(a.get("auto_mount"), p + ".auto_mount", auto_mount);
            if (!st.ok()) return fail(st.to_string());
            const yaml::Node* ids = a.get("device_ids");
            if (name.empty() || mp.empty() || !ids || !ids->is_seq() || ids->seq.size() < 2)
                return fail(p + ": name, mount_path and two or more device_ids are required");
            std::vector<DeviceInfo*> members;
            std::vector<std::string> blocks;
            for (std::size_t k = 0; k < ids->seq.size(); ++k) {
                std::int64_t id = -1;
                st = int_of(ids->seq[k].get(), p + ".device_ids[" + std::to_string(k) + "]", id);
                if (!st.ok()) return fail(st.to_string());
                DeviceInfo* d = find_device(id);
                if (!d) return fail(p + ": unknown device " + std::to_string(id));
                members.push_back(d);
                blocks.push_back(d->block_device);
                in_array[id] = true;
            }
            const bool known = std::all_of(blocks.begin(), blocks.end(), [](const std::string& b) { return !b.empty(); });
            for (DeviceInfo* d : members) d->mount = mp;  // members are reached through the array's mount
            if (!auto_mount || !known) continue;  // no block devices here: the array is managed outside
            auto md = mounts.assemble_raid0(name, blocks);
            if (!md.ok()) {
                for (DeviceInfo* d : members) mark(*d, "raid0 " + name + ": " + md.status().message());
                continue;
            }
            const MountOutcome mo = mounts.mount(md.value(), mp);
            if (!mo.error.empty())
                for (DeviceInfo* d : members) mark(*d, "raid0 " + name + ": " + mo.error);
        }
    }
    for (auto& d : devices) {
        if (in_array[d.id] || !extras[d.id].auto_mount || !d.available) continue;
        if (d.block_device.empty() || d.mount.empty()) continue;  // mounted outside the daemon
        const MountOutcome mo = mounts.mount(d.block_device, d.mount);
        if (!mo.error.empty()) mark(d, "mount: " + mo.error);
    }
    for (const auto& v : views) {
        if (v.view_root.empty()) continue;
        std::vector<std::pair<std::string, std::string>> links;
        for (const auto& d : devices) {
            bool allowed = d.accelerators.empty();
            for (auto a : d.accelerators) allowed = allowed || a == v.id;
            if (allowed && !d.mount.empty()) links.emplace_back("nvme" + std::to_string(d.id), d.mount);
        }
        Status vs = build_view_root(linux_host_sys(), v.view_root, links);
        if (!vs.ok()) std::fprintf(stderr, "tutti_daemon: view root of accelerator %lld: %s\n",
                                   static_cast<long long>(v.id), vs.to_string().c_str());
    }

    LeaseLedger ledger(devices);
    ledger.set_queue_pool(pool_default, pool_max);
    ledger.set_accelerators(views);
    ledger.set_lease_timing(static_cast<std::uint32_t>(hb_interval), static_cast<std::uint32_t>(hb_timeout));

    const int srv = ::socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (srv < 0) return fail("socket failed");
    sockaddr_un addr{};
    addr.sun_family = AF_UNIX;
    if (socket_path.size() >= sizeof(addr.sun_path)) return fail("socket path too long");
    std::strncpy(addr.sun_path, socket_path.c_str(), sizeof(addr.sun_path) - 1);
    ::unlink(socket_path.c_str());
    if (::bind(srv, reinterpret_cast<sockaddr*>(&addr), sizeof(addr)) != 0) return fail("bind " + socket_path);
    if (::listen(srv, 64) != 0) return fail("listen failed");
    signal(SIGTERM, on_signal);
    signal(SIGINT, on_signal);
    signal(SIGPIPE, SIG_IGN);
    std::fprintf(stderr, "tutti_daemon: serving %zu device(s) on %s\n", devices.size(), socket_path.c_str());

    std::thread reaper([&] {
        while (!g_stop.load()) {
            std::this_thread::sleep_for(std::chrono::milliseconds(reap_ms));
            auto reaped = ledger.reap(std::chrono::seconds(hb_timeout), [](std::int64_t pid, std::uint64_t start) {
                const std::uint64_t now = process_start_time(pid);
                return now != 0 && (start == 0 || now == start);
            });
            for (auto l : reaped) std::fprintf(stderr, "tutti_daemon: reaped lease %llu\n", (unsigned long long)l);
        }
    });
    while (!g_stop.load()) {
        fd_set rd;
        FD_ZERO(&rd);
        FD_SET(srv, &rd);
        timeval tv{0, 200000};
        if (::select(srv + 1, &rd, nullptr, nullptr, &tv) <= 0) continue;
        const int c = ::accept4(srv, nullptr, nullptr, SOCK_CLOEXEC);
        if (c < 0) continue;
        std::thread(serve_connection, c, &ledger).detach();
    }
    reaper.join();
    ::close(srv);
    ::unlink(socket_path.c_str());
    // Reverse order of bring-up: mounts, arrays, controllers.
    std::vector<std::string> report;
    const int busy = mounts.unmount_all(&report);
    for (const auto& l : report) std::fprintf(stderr, "tutti_daemon: %s\n", l.c_str());
    if (busy) std::fprintf(stderr, "tutti_daemon: %d mount(s) left in place (busy)\n", busy);
    if (!busy && mounts.stop_arrays()) std::fprintf(stderr, "tutti_daemon: an md array did not stop\n");
    g_mounts.store(nullptr);
    owners.clear();  // unbinds the controllers and removes their nodes
    return busy ? 1 : 0;
}
