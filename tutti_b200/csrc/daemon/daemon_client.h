#pragma once
// Client of tutti_daemon used by the runtime's NVMe resource: opens a session
// (client name, PID and process start time, so the daemon can reap it after a
// crash), acquires a queue lease for a device group, keeps it alive with a
// heartbeat thread and releases it at shutdown.
// Parity: reference nvmeservice_client.h:134 and the NVMe Resource
// (resource/nvme/nvme_resource.cpp:238-431: list / acquire / validate a grant).

#include <atomic>
#include <cstdint>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include <tutti/status.h>

namespace tutti {
namespace daemon {

struct LeaseGrant {
    std::uint64_t lease = 0;
    std::vector<std::int64_t> devices;
    std::vector<std::string> mounts;
    std::vector<std::uint32_t> first_queue;
    std::vector<std::uint32_t> lba_bytes;
    std::uint32_t queues = 0;
};

class DaemonClient {
public:
    DaemonClient() = default;
    ~DaemonClient();
    DaemonClient(const DaemonClient&) = delete;
    DaemonClient& operator=(const DaemonClient&) = delete;

    // `accel`: this process's accelerator, checked against devices' accelerator lists (-1: not given).
    Status connect(const std::string& socket_path, const std::string& client_name, std::int64_t accel = -1);
    Result<LeaseGrant> acquire(const std::vector<std::int64_t>& devices, std::uint32_t queues);
    // Starts a thread that sends HEARTBEAT every `interval_ms`.
    void start_heartbeat(std::uint32_t interval_ms);
    Status release();
    void close();
    Result<std::string> request(const std::string& line);  // raw round trip

private:
    int fd_ = -1;
    std::mutex mu_;
    std::uint64_t session_ = 0;
    LeaseGrant grant_;
    std::thread hb_;
    std::atomic<bool> stop_{false};
};

}  // namespace daemon
}  // namespace tutti
