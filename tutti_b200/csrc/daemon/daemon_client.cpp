#include "daemon_client.h"

#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include <chrono>
#include <cstdlib>
#include <cstring>

#include "lease_ledger.h"

namespace tutti {
namespace daemon {

namespace {
std::vector<std::string> split(const std::string& s) {
    std::vector<std::string> out;
    std::size_t a = 0;
    while (a <= s.size() && !s.empty()) {
        std::size_t b = s.find(',', a);
        if (b == std::string::npos) b = s.size();
        out.push_back(s.substr(a, b - a));
        a = b + 1;
    }
    return out;
}
}  // namespace

DaemonClient::~DaemonClient() { close(); }

Status DaemonClient::connect(const std::string& path, const std::string& client_name, std::int64_t accel) {
    fd_ = ::socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (fd_ < 0) return {StatusCode::INTERNAL, "socket failed"};
    sockaddr_un addr{};
    addr.sun_family = AF_UNIX;
    std::strncpy(addr.sun_path, path.c_str(), sizeof(addr.sun_path) - 1);
    if (::connect(fd_, reinterpret_cast<sockaddr*>(&addr), sizeof(addr)) != 0) {
        ::close(fd_);
        fd_ = -1;
        return {StatusCode::NOT_FOUND, "cannot reach tutti_daemon at " + path};
    }
    const long pid = static_cast<long>(::getpid());
    auto r = request("HELLO client=" + client_name + " pid=" + std::to_string(pid) +
                     " start_time=" + std::to_string(process_start_time(pid)) +
                     (accel >= 0 ? " accel=" + std::to_string(accel) : std::string()));
    if (!r.ok()) return r.status();
    const Message m = parse_message(r.value());
    session_ = std::strtoull(m.get("session").c_str(), nullptr, 10);
    if (!session_) return {StatusCode::INTERNAL, "daemon returned no session"};
    return Status::Ok();
}

Result<std::string> DaemonClient::request(const std::string& line) {
    std::lock_guard<std::mutex> g(mu_);
    if (fd_ < 0) return Result<std::string>::Failure({StatusCode::NOT_READY, "not connected"});
    const std::string out = line + "\n";
    std::size_t off = 0;
    while (off < out.size()) {
        const ssize_t w = ::write(fd_, out.data() + off, out.size() - off);
        if (w <= 0) return Result<std::string>::Failure({StatusCode::INTERNAL, "daemon write failed"});
        off += static_cast<std::size_t>(w);
    }
    std::string rsp;
    char c;
    while (true) {
        const ssize_t n = ::read(fd_, &c, 1);
        if (n <= 0) return Result<std::string>::Failure({StatusCode::INTERNAL, "daemon closed the connection"});
        if (c == '\n') break;
        rsp += c;
    }
    if (rsp.rfind("OK", 0) != 0)
        return Result<std::string>::Failure({StatusCode::RESOURCE_EXHAUSTED, "daemon: " + rsp});
    return rsp;
}

Result<LeaseGrant> DaemonClient::acquire(const std::vector<std::int64_t>& devices, std::uint32_t queues) {
    std::string ids;
    for (auto d : devices) ids += (ids.empty() ? "" : ",") + std::to_string(d);
    auto r = request("ACQUIRE session=" + std::to_string(session_) + " devices=" + ids +
                     " queues=" + std::to_string(queues));
    if (!r.ok()) return Result<LeaseGrant>::Failure(r.status());
    const Message m = parse_message(r.value());
    LeaseGrant g;
    g.lease = std::strtoull(m.get("lease").c_str(), nullptr, 10);
    for (auto& s : split(m.get("devices"))) g.devices.push_back(std::strtoll(s.c_str(), nullptr, 10));
    g.mounts = split(m.get("mounts"));
    for (auto& s : split(m.get("first_queue"))) g.first_queue.push_back(static_cast<std::uint32_t>(std::strtoul(s.c_str(), nullptr, 10)));
    for (auto& s : split(m.get("lba_bytes"))) g.lba_bytes.push_back(static_cast<std::uint32_t>(std::strtoul(s.c_str(), nullptr, 10)));
    g.queues = static_cast<std::uint32_t>(std::strtoul(m.get("queues").c_str(), nullptr, 10));
    grant_ = g;
    return g;
}

void DaemonClient::start_heartbeat(std::uint32_t interval_ms) {
    if (hb_.joinable() || !grant_.lease) return;
    stop_.store(false);
    hb_ = std::thread([this, interval_ms] {
        while (!stop_.load()) {
            for (std::uint32_t t = 0; t < interval_ms && !stop_.load(); t += 50)
                std::this_thread::sleep_for(std::chrono::milliseconds(50));
            if (stop_.load()) break;
            (void)request("HEARTBEAT lease=" + std::to_string(grant_.lease));
        }
    });
}

Status DaemonClient::release() {
    stop_.store(true);
    if (hb_.joinable()) hb_.join();
    if (!grant_.lease) return Status::Ok();
    auto r = request("RELEASE lease=" + std::to_string(grant_.lease));
    grant_.lease = 0;
    return r.ok() ? Status::Ok() : r.status();
}

void DaemonClient::close() {
    release();
    if (fd_ >= 0) {
        if (session_) (void)request("BYE session=" + std::to_string(session_));
        std::lock_guard<std::mutex> g(mu_);
        ::close(fd_);
        fd_ = -1;
    }
}

}  // namespace daemon
}  // namespace tutti
