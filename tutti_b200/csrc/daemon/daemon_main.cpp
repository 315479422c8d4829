// tutti_daemon: host-level owner of the NVMe devices; GPU processes lease
// I/O queues from it over a UNIX socket.
//
//   tutti_daemon --config daemon.yaml
//
// Config:
//   service: {socket: /run/tutti/daemon.sock}
//   lease:   {heartbeat_timeout_s: 30, reap_interval_ms: 1000}
//   devices:
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
    if (const auto* s = r.get("service"))
        if (const auto* p = s->get("socket")) socket_path = p->scalar;
    if (const auto* l = r.get("lease")) {
        if (const auto* t = l->get("heartbeat_timeout_s")) hb_timeout = yaml::as_int(*t, "lease.heartbeat_timeout_s").value();
        if (const auto* t = l->get("reap_interval_ms")) reap_ms = yaml::as_int(*t, "lease.reap_interval_ms").value();
    }
    std::vector<DeviceInfo> devices;
    const auto* devs = r.get("devices");
    if (!devs || !devs->is_seq()) return fail("config: devices: expected a list");
    for (std::size_t i = 0; i < devs->seq.size(); ++i) {
        const yaml::Node& d = *devs->seq[i];
        const std::string p = "devices[" + std::to_string(i) + "]";
        DeviceInfo info;
        auto id = d.get("id");
        if (!id) return fail(p + ".id: required");
        auto idv = yaml::as_int(*id, p + ".id");
        if (!idv.ok()) return fail(idv.status().to_string());
        info.id = idv.value();
        if (auto k = d.get("kind")) info.kind = k->scalar;
        if (auto m = d.get("mount")) info.mount = m->scalar;
        if (auto c = d.get("pci")) info.pci = c->scalar;
        if (auto q = d.get("queues")) info.queues = static_cast<std::uint32_t>(yaml::as_int(*q, p + ".queues").value());
        if (auto q = d.get("nsid")) info.namespace_id = static_cast<std::uint32_t>(yaml::as_int(*q, p + ".nsid").value());
        if (auto q = d.get("lba_bytes")) info.lba_bytes = static_cast<std::uint32_t>(yaml::as_int(*q, p + ".lba_bytes").value());
        if (auto a = d.get("accelerators")) {
            if (!a->is_seq()) return fail(p + ".accelerators: expected a list of accelerator ids");
            for (std::size_t k = 0; k < a->seq.size(); ++k) {
                auto v = yaml::as_int(*a->seq[k], p + ".accelerators[" + std::to_string(k) + "]");
                if (!v.ok()) return fail(v.status().to_string());
                info.accelerators.push_back(v.value());
            }
        }
        if (info.kind != "emulated" && info.kind != "nvme") return fail(p + ".kind must be emulated or nvme");
        devices.push_back(info);
    }
    LeaseLedger ledger(devices);

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
