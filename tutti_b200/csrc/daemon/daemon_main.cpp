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
//              #   allowed_accel_ids (empty: every accelerator of Tutti's accelerators: list)}]
//     - {id: 0, kind: emulated, mount: /mnt/nvme0, queues: 128, pci: "0000:1b:00.0", nsid: 1, lba_bytes: 512,
//        accelerators: [0, 1]}   # optional: only these GPUs may lease its queues
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

#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "../config/yaml_lite.h"
#include "lease_ledger.h"

using namespace tutti;
using namespace tutti::daemon;

namespace {
std::atomic<bool> g_stop{false};
void on_signal(int) { g_stop.store(true); }

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
    if (const auto* acc = r.get("accelerators")) {
        if (!acc->is_seq()) return fail("config: accelerators: expected a list");
        for (std::size_t i = 0; i < acc->seq.size(); ++i) {
            std::int64_t a = -1;
            st = int_of(acc->seq[i]->get("accel_id"), "accelerators[" + std::to_string(i) + "].accel_id", a);
            if (!st.ok()) return fail(st.to_string());
            if (a >= 0) configured_accels.push_back(a);
        }
    }
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
    LeaseLedger ledger(devices);
    ledger.set_queue_pool(pool_default, pool_max);

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
    return 0;
}
