#include "lease_ledger.h"

#include <cctype>
#include <cstdio>
#include <cstdlib>
#include <cstring>


namespace tutti {
namespace daemon {

std::uint64_t process_start_time(std::int64_t pid) {
    if (pid <= 0) return 0;
    char path[64];
    std::snprintf(path, sizeof(path), "/proc/%lld/stat", static_cast<long long>(pid));
    std::FILE* f = std::fopen(path, "r");
    if (!f) return 0;
    char buf[1024];
    const std::size_t n = std::fread(buf, 1, sizeof(buf) - 1, f);
    std::fclose(f);
    buf[n] = '\0';
    // comm may contain spaces: fields resume after the last ')'
    const char* p = std::strrchr(buf, ')');
    if (!p) return 0;
    ++p;
    // after ')' come fields 3.. ; start time is field 22
    int field = 2;
    const char* tok = p;
    while (*tok) {
        while (*tok == ' ') ++tok;
        if (!*tok) break;
        ++field;
        if (field == 22) return std::strtoull(tok, nullptr, 10);
        while (*tok && *tok != ' ') ++tok;
    }
    return 0;
}

LeaseLedger::LeaseLedger(std::vector<DeviceInfo> devices) : devices_(std::move(devices)) {
    for (auto& d : devices_) used_[d.id] = std::vector<bool>(d.queues, false);
}

const DeviceInfo* LeaseLedger::device(std::int64_t id) const {
    for (auto& d : devices_)
        if (d.id == id) return &d;
    return nullptr;
}

std::vector<DeviceInfo> LeaseLedger::devices() const {
    std::lock_guard<std::mutex> g(mu_);
    return devices_;
}

std::uint32_t LeaseLedger::free_queues(std::int64_t device) const {
    std::lock_guard<std::mutex> g(mu_);
    auto it = used_.find(device);
    if (it == used_.end()) return 0;
    std::uint32_t n = 0;
    for (bool u : it->second) n += u ? 0 : 1;
    return n;
}

std::size_t LeaseLedger::lease_count() const {
    std::lock_guard<std::mutex> g(mu_);
    return leases_.size();
}

Result<std::uint64_t> LeaseLedger::open_session(const std::string& client, std::int64_t pid, std::uint64_t start,
                                                std::int64_t accel, bool implicit) {
    std::lock_guard<std::mutex> g(mu_);
    Session s;
    s.id = next_++;
    s.client = client;
    s.pid = pid;
    s.start_time = start;
    s.accel = accel;
    s.implicit = implicit;
    sessions_[s.id] = s;
    return s.id;
}

Status LeaseLedger::release_allocation(std::uint64_t lease) {
    std::lock_guard<std::mutex> g(mu_);
    auto it = leases_.find(lease);
    if (it == leases_.end()) return {StatusCode::NOT_FOUND, "unknown allocation"};
    const std::uint64_t session = it->second.session;
    release_locked(lease);
    auto sit = sessions_.find(session);
    if (sit != sessions_.end() && sit->second.implicit) {
        bool more = false;
        for (auto& kv : leases_) more |= kv.second.session == session;
        if (!more) sessions_.erase(sit);
    }
    return Status::Ok();
}

std::string LeaseLedger::view_root(std::int64_t accel) const {
    std::lock_guard<std::mutex> g(mu_);
    for (const auto& a : accels_)
        if (a.id == accel) return a.view_root;
    return "";
}

std::vector<std::int64_t> LeaseLedger::allowed_devices(std::int64_t accel) const {
    std::lock_guard<std::mutex> g(mu_);
    std::vector<std::int64_t> out;
    for (const auto& d : devices_) {
        bool ok = d.accelerators.empty();
        for (auto a : d.accelerators) ok = ok || a == accel;
        if (ok && d.available) out.push_back(d.id);
    }
    return out;
}

Status LeaseLedger::close_session(std::uint64_t session) {
    std::lock_guard<std::mutex> g(mu_);
    if (!sessions_.count(session)) return {StatusCode::NOT_FOUND, "unknown session"};
    std::vector<std::uint64_t> mine;
    for (auto& kv : leases_)
        if (kv.second.session == session) mine.push_back(kv.first);
    for (auto l : mine) release_locked(l);
    sessions_.erase(session);
    return Status::Ok();
}

Result<Lease> LeaseLedger::acquire(std::uint64_t session, const std::vector<std::int64_t>& devices,
                                   std::uint32_t queues) {
    using R = Result<Lease>;
    std::lock_guard<std::mutex> g(mu_);
    auto sit = sessions_.find(session);
    if (sit == sessions_.end()) return R::Failure({StatusCode::NOT_FOUND, "unknown session"});
    if (queues == 0) queues = pool_default_;
    if (devices.empty() || queues == 0) return R::Failure({StatusCode::INVALID_ARGUMENT, "empty request"});
    if (pool_max_ && queues > pool_max_)
        return R::Failure({StatusCode::RESOURCE_EXHAUSTED, std::to_string(queues) + " queues asked, at most " +
                                                               std::to_string(pool_max_) + " per client"});
    const std::int64_t accel = sit->second.accel;
    for (auto dev : devices) {
        for (const auto& d : devices_)
            if (d.id == dev && !d.available)
                return R::Failure({StatusCode::UNSUPPORTED, "device " + std::to_string(dev) +
                                                                " is unavailable: " + d.diagnostic});
        for (const auto& d : devices_) {
            if (d.id != dev || d.accelerators.empty()) continue;
            bool allowed = false;
            for (auto a : d.accelerators) allowed = allowed || a == accel;
            if (!allowed)
                return R::Failure({StatusCode::PERMISSION_DENIED,
                                   "accelerator " + (accel < 0 ? std::string("(not given)") : std::to_string(accel)) +
                                       " may not use device " + std::to_string(dev)});
        }
    }
    // Contiguous queue ranges per device, all-or-nothing.
    std::vector<Grant> grants;
    for (auto dev : devices) {
        auto it = used_.find(dev);
        if (it == used_.end()) return R::Failure({StatusCode::NOT_FOUND, "unknown device " + std::to_string(dev)});
        auto& u = it->second;
        std::uint32_t run = 0, start = 0;
        bool found = false;
        for (std::uint32_t q = 0; q < u.size(); ++q) {
            if (u[q]) {
                run = 0;
                continue;
            }
            if (run == 0) start = q;
            if (++run == queues) {
                found = true;
                break;
            }
        }
        if (!found)
            return R::Failure({StatusCode::RESOURCE_EXHAUSTED,
                               "device " + std::to_string(dev) + " has no " + std::to_string(queues) + " free queues"});
        grants.push_back({dev, queues, start});
    }
    for (auto& gr : grants)
        for (std::uint32_t q = 0; q < gr.queues; ++q) used_[gr.device][gr.first_queue + q] = true;
    Lease l;
    l.id = next_++;
    l.session = session;
    l.grants = grants;
    l.last_heartbeat = std::chrono::steady_clock::now();
    leases_[l.id] = l;
    return l;
}

Status LeaseLedger::heartbeat(std::uint64_t lease) {
    std::lock_guard<std::mutex> g(mu_);
    auto it = leases_.find(lease);
    if (it == leases_.end()) return {StatusCode::NOT_FOUND, "unknown lease"};
    it->second.last_heartbeat = std::chrono::steady_clock::now();
    return Status::Ok();
}

void LeaseLedger::release_locked(std::uint64_t lease) {
    auto it = leases_.find(lease);
    if (it == leases_.end()) return;
    for (auto& gr : it->second.grants) {
        auto& u = used_[gr.device];
        for (std::uint32_t q = 0; q < gr.queues && gr.first_queue + q < u.size(); ++q) u[gr.first_queue + q] = false;
    }
    leases_.erase(it);
}

Status LeaseLedger::release(std::uint64_t lease) {
    std::lock_guard<std::mutex> g(mu_);
    if (!leases_.count(lease)) return {StatusCode::NOT_FOUND, "unknown lease"};
    release_locked(lease);
    return Status::Ok();
}

std::vector<std::uint64_t> LeaseLedger::reap(std::chrono::steady_clock::duration timeout,
                                             const std::function<bool(std::int64_t, std::uint64_t)>& alive) {
    std::lock_guard<std::mutex> g(mu_);
    std::vector<std::uint64_t> reaped;
    const auto now = std::chrono::steady_clock::now();
    std::vector<std::uint64_t> dead_sessions;
    for (auto& kv : sessions_)
        if (kv.second.pid > 0 && !alive(kv.second.pid, kv.second.start_time)) dead_sessions.push_back(kv.first);
    for (auto& kv : leases_) {
        const bool expired = now - kv.second.last_heartbeat > timeout;
        bool dead = false;
        for (auto s : dead_sessions) dead |= kv.second.session == s;
        if (expired || dead) reaped.push_back(kv.first);
    }
    for (auto l : reaped) release_locked(l);
    for (auto s : dead_sessions) sessions_.erase(s);
    return reaped;
}

namespace {
std::string encode_value(const std::string& v) {
    std::string out;
    for (unsigned char c : v) {
        if (c == '%' || c == ' ' || c == '\t' || c == '\n' || c == '\r') {
            char b[4];
            std::snprintf(b, sizeof(b), "%%%02X", c);
            out += b;
        } else {
            out.push_back(static_cast<char>(c));
        }
    }
    return out;
}
std::string decode_value(const std::string& v) {
    std::string out;
    for (std::size_t i = 0; i < v.size(); ++i) {
        if (v[i] == '%' && i + 2 < v.size() && std::isxdigit(static_cast<unsigned char>(v[i + 1])) &&
            std::isxdigit(static_cast<unsigned char>(v[i + 2]))) {
            out.push_back(static_cast<char>(std::strtol(v.substr(i + 1, 2).c_str(), nullptr, 16)));
            i += 2;
        } else {
            out.push_back(v[i]);
        }
    }
    return out;
}
}  // namespace

Message parse_message(const std::string& line) {
    Message m;
    std::vector<std::string> toks;
    std::size_t i = 0;
    while (i < line.size()) {
        while (i < line.size() && (line[i] == ' ' || line[i] == '\n' || line[i] == '\r' || line[i] == '\t')) ++i;
        std::size_t j = i;
        while (j < line.size() && line[j] != ' ' && line[j] != '\n' && line[j] != '\r' && line[j] != '\t') ++j;
        if (j > i) toks.push_back(line.substr(i, j - i));
        i = j;
    }
    if (toks.empty()) return m;
    m.verb = toks[0];
    for (std::size_t k = 1; k < toks.size(); ++k) {
        const std::string& tok = toks[k];
        const auto eq = tok.find('=');
        if (eq == std::string::npos)
            m.kv[tok] = "";
        else
            m.kv[tok.substr(0, eq)] = decode_value(tok.substr(eq + 1));
    }
    return m;
}


std::string format_message(const Message& m) {
    std::string out = m.verb;
    for (auto& kv : m.kv) out += " " + kv.first + "=" + encode_value(kv.second);
    return out + "\n";
}

namespace {
std::vector<std::int64_t> parse_ids(const std::string& s) {
    std::vector<std::int64_t> out;
    std::size_t a = 0;
    while (a < s.size()) {
        std::size_t b = s.find(',', a);
        if (b == std::string::npos) b = s.size();
        if (b > a) out.push_back(std::strtoll(s.substr(a, b - a).c_str(), nullptr, 10));
        a = b + 1;
    }
    return out;
}
std::string err(const Status& s) { return "ERR " + s.to_string() + "\n"; }

std::string join_ids(const std::vector<std::int64_t>& v, const char* sep = ",") {
    std::string out;
    for (auto x : v) out += (out.empty() ? "" : sep) + std::to_string(x);
    return out;
}

std::uint32_t log2_of(std::uint32_t v) {
    std::uint32_t l = 0;
    while ((1u << (l + 1)) <= v && l < 31) ++l;
    return l;
}

// Fields of one device as the service reports it, under `p` (e.g. "d0.").
void put_device(Message& rsp, const std::string& p, const DeviceInfo& d, const LeaseLedger& ledger) {
    rsp.kv[p + "device_id"] = std::to_string(d.id);
    rsp.kv[p + "pci_addr"] = d.pci;
    rsp.kv[p + "snvme_dev_path"] = d.chrdev;
    rsp.kv[p + "block_path"] = d.block_device;
    rsp.kv[p + "backing_mount_path"] = d.mount;
    rsp.kv[p + "namespace_id"] = std::to_string(d.namespace_id);
    rsp.kv[p + "blk_size"] = std::to_string(d.lba_bytes);
    rsp.kv[p + "blk_size_log"] = std::to_string(log2_of(d.lba_bytes));
    rsp.kv[p + "queue_depth"] = std::to_string(d.queue_depth);
    rsp.kv[p + "max_data_size"] = std::to_string(d.max_data_size);
    rsp.kv[p + "max_queues_per_group"] = std::to_string(d.max_queues_per_group);
    rsp.kv[p + "page_size"] = std::to_string(d.page_size);
    rsp.kv[p + "dstrd"] = std::to_string(d.doorbell_stride);
    rsp.kv[p + "max_user_qid"] = std::to_string(d.max_user_qid);
    rsp.kv[p + "chrdev_minor"] = std::to_string(d.chrdev_minor);
    rsp.kv[p + "allowed_accel_ids"] = d.accelerators.empty() ? "*" : join_ids(d.accelerators);
    rsp.kv[p + "kind"] = d.kind;
    (void)ledger;
}

// One lease as the service reports an allocation: one slice per device.
void put_slices(Message& rsp, const Lease& l, const LeaseLedger& ledger, std::int64_t accel) {
    rsp.kv["allocation_id"] = std::to_string(l.id);
    rsp.kv["slices"] = std::to_string(l.grants.size());
    const std::string root = ledger.view_root(accel);
    for (std::size_t i = 0; i < l.grants.size(); ++i) {
        const Grant& gr = l.grants[i];
        const DeviceInfo* d = ledger.device(gr.device);
        const std::string p = "s" + std::to_string(i) + ".";
        if (d) put_device(rsp, p, *d, ledger);
        rsp.kv[p + "accel_id"] = std::to_string(accel);
        rsp.kv[p + "granted_queues"] = std::to_string(gr.queues);
        rsp.kv[p + "first_queue"] = std::to_string(gr.first_queue);
        rsp.kv[p + "controller_queue_capacity"] = std::to_string(d ? d->queues : 0);
        rsp.kv[p + "view_path"] = root.empty() ? "" : root + "/nvme" + std::to_string(gr.device);
    }
    rsp.kv["heartbeat_interval_sec"] = std::to_string(ledger.heartbeat_interval_s());
    rsp.kv["lease_timeout_sec"] = std::to_string(ledger.lease_timeout_s());
}
}  // namespace

std::string handle_request(LeaseLedger& ledger, const std::string& line) {
    const Message req = parse_message(line);
    Message rsp;
    rsp.verb = "OK";
    if (req.verb == "HELLO") {
        const std::int64_t pid = std::strtoll(req.get("pid", "0").c_str(), nullptr, 10);
        std::uint64_t start = std::strtoull(req.get("start_time", "0").c_str(), nullptr, 10);
        if (start == 0) start = process_start_time(pid);
        const std::int64_t accel = std::strtoll(req.get("accel", "-1").c_str(), nullptr, 10);
        auto s = ledger.open_session(req.get("client", "anonymous"), pid, start, accel);
        if (!s.ok()) return err(s.status());
        rsp.kv["session"] = std::to_string(s.value());
    } else if (req.verb == "BYE") {
        Status s = ledger.close_session(std::strtoull(req.get("session").c_str(), nullptr, 10));
        if (!s.ok()) return err(s);
    } else if (req.verb == "LIST") {
        std::string ids, mounts, free, kinds, acl;
        for (auto& d : ledger.devices()) {
            const std::string sep = ids.empty() ? "" : ",";
            std::string who;
            for (auto a : d.accelerators) who += (who.empty() ? "" : "+") + std::to_string(a);
            acl += sep + (who.empty() ? "*" : who);  // "*": any accelerator
            ids += sep + std::to_string(d.id);
            mounts += sep + d.mount;
            kinds += sep + d.kind;
            free += sep + std::to_string(ledger.free_queues(d.id));
        }
        rsp.kv["devices"] = ids;
        rsp.kv["mounts"] = mounts;
        rsp.kv["kinds"] = kinds;
        rsp.kv["free_queues"] = free;
        rsp.kv["accelerators"] = acl;
    } else if (req.verb == "ACQUIRE") {
        auto l = ledger.acquire(std::strtoull(req.get("session").c_str(), nullptr, 10), parse_ids(req.get("devices")),
                                static_cast<std::uint32_t>(std::strtoul(req.get("queues", "0").c_str(), nullptr, 10)));
        if (!l.ok()) return err(l.status());
        std::string devs, mounts, firsts, lbas, nsids;
        for (auto& gr : l.value().grants) {
            const DeviceInfo* d = ledger.device(gr.device);
            const std::string sep = devs.empty() ? "" : ",";
            devs += sep + std::to_string(gr.device);
            mounts += sep + (d ? d->mount : "");
            firsts += sep + std::to_string(gr.first_queue);
            lbas += sep + std::to_string(d ? d->lba_bytes : 512);
            nsids += sep + std::to_string(d ? d->namespace_id : 1);
        }
        rsp.kv["lease"] = std::to_string(l.value().id);
        rsp.kv["devices"] = devs;
        rsp.kv["mounts"] = mounts;
        rsp.kv["first_queue"] = firsts;
        rsp.kv["queues"] = std::to_string(l.value().grants.empty() ? 0 : l.value().grants[0].queues);
        rsp.kv["lba_bytes"] = lbas;
        rsp.kv["nsid"] = nsids;
    } else if (req.verb == "HEARTBEAT") {
        const std::string id = req.get("lease", req.get("allocation_id", req.get("allocation")));
        Status s = ledger.heartbeat(std::strtoull(id.c_str(), nullptr, 10));
        if (!s.ok()) return err(s);
        rsp.kv["notice"] = "NONE";
    } else if (req.verb == "RELEASE" || req.verb == "DISCONNECT") {
        const std::string id = req.get("lease", req.get("allocation_id", req.get("allocation")));
        Status s = ledger.release_allocation(std::strtoull(id.c_str(), nullptr, 10));
        if (!s.ok()) return err(s);
        rsp.kv["success"] = "true";
    } else if (req.verb == "LIST_DEVICES") {
        const auto devs = ledger.devices();
        rsp.kv["devices"] = std::to_string(devs.size());
        for (std::size_t i = 0; i < devs.size(); ++i) {
            const std::string p = "d" + std::to_string(i) + ".";
            put_device(rsp, p, devs[i], ledger);
            // the mount each allowed accelerator reaches the drive through
            std::string gpus;
            for (auto a : devs[i].accelerators.empty() ? std::vector<std::int64_t>{} : devs[i].accelerators) {
                const std::string root = ledger.view_root(a);
                gpus += (gpus.empty() ? "" : ";") + std::to_string(a) + ":" +
                        (root.empty() ? devs[i].mount : root + "/nvme" + std::to_string(devs[i].id));
            }
            rsp.kv[p + "allowed_gpus"] = gpus;
        }
    } else if (req.verb == "LIST_ACCELERATORS") {
        const auto acc = ledger.accelerators();
        rsp.kv["accelerators"] = std::to_string(acc.size());
        for (std::size_t i = 0; i < acc.size(); ++i) {
            rsp.kv["a" + std::to_string(i) + ".accel_id"] = std::to_string(acc[i].id);
            rsp.kv["a" + std::to_string(i) + ".view_root"] = acc[i].view_root;
        }
    } else if (req.verb == "LIST_RESOURCES") {
        const auto devs = ledger.devices();
        rsp.kv["resources"] = std::to_string(devs.size());
        for (std::size_t i = 0; i < devs.size(); ++i) {
            const std::string p = "r" + std::to_string(i) + ".";
            put_device(rsp, p, devs[i], ledger);
            const std::uint32_t freeq = ledger.free_queues(devs[i].id);
            rsp.kv[p + "controller_queue_capacity"] = std::to_string(devs[i].queues);
            rsp.kv[p + "available_queues"] = std::to_string(devs[i].available ? freeq : 0);
            rsp.kv[p + "reserved_queues"] = std::to_string(devs[i].queues - freeq);
            rsp.kv[p + "available"] = devs[i].available ? "true" : "false";
            rsp.kv[p + "diagnostic"] = devs[i].diagnostic;
        }
        rsp.kv["heartbeat_interval_sec"] = std::to_string(ledger.heartbeat_interval_s());
        rsp.kv["lease_timeout_sec"] = std::to_string(ledger.lease_timeout_s());
    } else if (req.verb == "CONNECT" || req.verb == "ACQUIRE_SLICES") {
        // A session of its own (closed with the allocation) unless one is named.
        const std::int64_t accel = std::strtoll(req.get("accel", req.get("cuda_device", req.get("accel_id", "-1"))).c_str(),
                                                nullptr, 10);
        const std::int64_t pid = std::strtoll(req.get("pid", req.get("client_pid", "0")).c_str(), nullptr, 10);
        std::vector<std::int64_t> devs;
        if (req.verb == "CONNECT") {
            devs.push_back(std::strtoll(req.get("device", req.get("device_id", "-1")).c_str(), nullptr, 10));
        } else {
            const std::string mode = req.get("selection", "allowed");
            if (mode == "explicit") {
                devs = parse_ids(req.get("devices", req.get("device_ids")));
                if (devs.empty()) return err({StatusCode::INVALID_ARGUMENT, "explicit selection names no devices"});
            } else if (mode == "allowed" || mode == "striped") {
                devs = ledger.allowed_devices(accel);
                if (mode == "striped" && devs.size() < 2)
                    return err({StatusCode::RESOURCE_EXHAUSTED, "striping needs two or more devices for this accelerator"});
                if (devs.empty()) return err({StatusCode::PERMISSION_DENIED, "no device is allowed for this accelerator"});
            } else {
                return err({StatusCode::INVALID_ARGUMENT, "selection must be allowed, explicit or striped"});
            }
        }
        std::uint64_t session = std::strtoull(req.get("session", "0").c_str(), nullptr, 10);
        bool opened = false;
        if (session == 0) {
            auto sr = ledger.open_session(req.get("client", "pid" + std::to_string(pid)), pid, process_start_time(pid),
                                          accel, /*implicit=*/true);
            if (!sr.ok()) return err(sr.status());
            session = sr.value();
            opened = true;
        }
        const auto queues = static_cast<std::uint32_t>(
            std::strtoul(req.get("queues", req.get("num_queues", req.get("queues_per_controller", "0"))).c_str(), nullptr, 10));
        auto l = ledger.acquire(session, devs, queues);
        if (!l.ok()) {
            if (opened) (void)ledger.close_session(session);
            return err(l.status());
        }
        put_slices(rsp, l.value(), ledger, accel);
        if (req.verb == "CONNECT" && !l.value().grants.empty()) {
            // the single-device answer carries the slice's fields unprefixed
            const Grant& gr = l.value().grants[0];
            if (const DeviceInfo* d = ledger.device(gr.device)) {
                put_device(rsp, "", *d, ledger);
                rsp.kv["mount_path"] = rsp.kv["s0.view_path"].empty() ? d->mount : rsp.kv["s0.view_path"];
            }
            rsp.kv["granted_queues"] = std::to_string(gr.queues);
            rsp.kv["first_queue"] = std::to_string(gr.first_queue);
        }
    } else if (req.verb == "STATUS") {
        rsp.kv["leases"] = std::to_string(ledger.lease_count());
        rsp.kv["devices"] = std::to_string(ledger.devices().size());
    } else {
        return err({StatusCode::INVALID_ARGUMENT, "unknown verb '" + req.verb + "'"});
    }
    return format_message(rsp);
}

}  // namespace daemon
}  // namespace tutti
