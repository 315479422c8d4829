#pragma once
// Queue-lease ledger of the device-manager daemon.
//
// The daemon is the host-level owner of the NVMe devices: it knows each
// device's mount and queue budget, and GPU processes lease queues from it.
// A lease names a client session and, per device, a number of I/O queues.
// Leases end by explicit release, by heartbeat expiry, or when the reaper
// finds the client process gone (its PID no longer exists, or exists with a
// different start time, i.e. the PID was reused).
// Parity: reference csrc/device_manager/nvme/nvmeservice (ServiceState
// queue-reservation ledger, leases with heartbeat, PID/starttime reaper:
// nvmeservice_state.h:190, nvmeservice_state.cpp:29-46,138).

#include <chrono>
#include <cstdint>
#include <functional>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include <tutti/status.h>

namespace tutti {
namespace daemon {

struct DeviceInfo {
    std::int64_t id = 0;
    std::string kind = "emulated";  // emulated | nvme
    std::string mount;
    std::string pci;
    std::uint32_t queues = 64;      // queue budget offered to clients
    std::uint32_t namespace_id = 1;
    std::uint32_t lba_bytes = 512;
    std::vector<std::int64_t> accelerators;  // who may lease its queues; empty: any accelerator
    // Filled by the controller's bring-up when the daemon owns it (snvme).
    std::string chrdev;        // the controller's snvme node
    std::string block_device;  // the namespace's block device
    std::uint32_t queue_depth = 0;
    std::uint64_t max_data_size = 0;
    std::uint32_t max_queues_per_group = 32;
    std::uint32_t page_size = 4096;      // the controller's memory page size (CC.MPS)
    std::uint32_t doorbell_stride = 0;   // CAP.DSTRD (doorbells 4 << DSTRD bytes apart)
    std::uint32_t max_user_qid = 0;      // highest QID the driver hands to user queues (0: unknown)
    std::int32_t chrdev_minor = -1;      // the snvme node's minor (-1: none)
    bool available = true;     // false: bring-up or mount failed (see diagnostic); not leased
    std::string diagnostic;
};

// An accelerator and the directory its processes reach the drives through.
struct AcceleratorView {
    std::int64_t id = -1;
    std::string view_root;
};

struct Grant {
    std::int64_t device = 0;
    std::uint32_t queues = 0;
    std::uint32_t first_queue = 0;  // the device's queue range [first, first+queues)
};

struct Lease {
    std::uint64_t id = 0;
    std::uint64_t session = 0;
    std::vector<Grant> grants;
    std::chrono::steady_clock::time_point last_heartbeat;
};

struct Session {
    std::uint64_t id = 0;
    std::string client;
    std::int64_t pid = 0;
    std::uint64_t start_time = 0;  // /proc/<pid>/stat field 22 at HELLO
    std::int64_t accel = -1;       // the client's accelerator (HELLO accel=...), -1 if not given
    bool implicit = false;         // opened by CONNECT / ACQUIRE_SLICES: closed with its lease
};

// Reads /proc/<pid>/stat start time (clock ticks since boot); 0 if the process is gone.
std::uint64_t process_start_time(std::int64_t pid);

class LeaseLedger {
public:
    explicit LeaseLedger(std::vector<DeviceInfo> devices);

    Result<std::uint64_t> open_session(const std::string& client, std::int64_t pid, std::uint64_t start_time,
                                       std::int64_t accel = -1, bool implicit = false);
    // Releases a lease; a session opened only for it is closed too.
    Status release_allocation(std::uint64_t lease);
    Status close_session(std::uint64_t session);  // releases its leases

    // All-or-nothing: either every device gets `queues` queues or nothing changes.
    // A device with an accelerator list is leased only to sessions of those
    // accelerators (PERMISSION_DENIED otherwise).
    Result<Lease> acquire(std::uint64_t session, const std::vector<std::int64_t>& devices, std::uint32_t queues);
    Status heartbeat(std::uint64_t lease);
    // Per-client queue policy: a request for 0 queues gets `default_queues`;
    // one for more than `max_queues` is refused (0: no default / no cap).
    void set_queue_pool(std::uint32_t default_queues, std::uint32_t max_queues) {
        std::lock_guard<std::mutex> g(mu_);
        pool_default_ = default_queues;
        pool_max_ = max_queues;
    }
    Status release(std::uint64_t lease);

    // Releases leases whose heartbeat is older than `timeout`, and sessions
    // whose process is gone according to `alive(pid, start_time)`.
    std::vector<std::uint64_t> reap(std::chrono::steady_clock::duration timeout,
                                    const std::function<bool(std::int64_t, std::uint64_t)>& alive);

    std::vector<DeviceInfo> devices() const;
    std::uint32_t free_queues(std::int64_t device) const;
    void set_accelerators(std::vector<AcceleratorView> a) {
        std::lock_guard<std::mutex> g(mu_);
        accels_ = std::move(a);
    }
    std::vector<AcceleratorView> accelerators() const {
        std::lock_guard<std::mutex> g(mu_);
        return accels_;
    }
    std::string view_root(std::int64_t accel) const;
    void set_lease_timing(std::uint32_t heartbeat_interval_s, std::uint32_t timeout_s) {
        std::lock_guard<std::mutex> g(mu_);
        hb_interval_s_ = heartbeat_interval_s;
        lease_timeout_s_ = timeout_s;
    }
    std::uint32_t heartbeat_interval_s() const { return hb_interval_s_; }
    std::uint32_t lease_timeout_s() const { return lease_timeout_s_; }
    // Available devices `accel` may lease (every device without a list, and those listing it).
    std::vector<std::int64_t> allowed_devices(std::int64_t accel) const;
    std::size_t lease_count() const;
    const DeviceInfo* device(std::int64_t id) const;

private:
    void release_locked(std::uint64_t lease);
    mutable std::mutex mu_;
    std::vector<DeviceInfo> devices_;
    std::map<std::int64_t, std::vector<bool>> used_;  // device -> queue slot in use
    std::map<std::uint64_t, Session> sessions_;
    std::map<std::uint64_t, Lease> leases_;
    std::uint64_t next_ = 1;
    std::uint32_t pool_default_ = 0, pool_max_ = 0;
    std::vector<AcceleratorView> accels_;
    std::uint32_t hb_interval_s_ = 10, lease_timeout_s_ = 30;
};

// Line protocol: "VERB key=value key=value\n" -> "OK key=value ...\n" | "ERR message\n".
// Values carry '%', spaces, tabs and line breaks as %XX.
// Verbs: HELLO, BYE, LIST, ACQUIRE, HEARTBEAT, RELEASE, STATUS (sessions and
// leases), and the service surface of the reference's NvmeService:
// LIST_DEVICES, CONNECT, DISCONNECT, LIST_ACCELERATORS, LIST_RESOURCES,
// ACQUIRE_SLICES (HEARTBEAT and RELEASE also take allocation=). Lists come
// back as indexed keys: devices=2 d0.device_id=... d1.device_id=...
struct Message {
    std::string verb;
    std::map<std::string, std::string> kv;
    std::string get(const std::string& k, const std::string& def = "") const {
        auto it = kv.find(k);
        return it == kv.end() ? def : it->second;
    }
};
Message parse_message(const std::string& line);
std::string format_message(const Message& m);

// Handles one request against the ledger (used by the server and by tests).
std::string handle_request(LeaseLedger& ledger, const std::string& line);

}  // namespace daemon
}  // namespace tutti
