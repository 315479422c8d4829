#include "lease_ledger.h"

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
                                                std::int64_t accel) {
    std::lock_guard<std::mutex> g(mu_);
    Session s;
    s.id = next_++;
    s.client = client;
    s.pid = pid;
    s.start_time = start;
    s.accel = accel;
    sessions_[s.id] = s;
    return s.id;
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
            m.kv[tok.substr(0, eq)] = tok.substr(eq + 1);
    }
    return m;
}

std::string format_message(const Message& m) {
    std::string out = m.verb;
    for (auto& kv : m.kv) out += " " + kv.first + "=" + kv.second;
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
        Status s = ledger.heartbeat(std::strtoull(req.get("lease").c_str(), nullptr, 10));
        if (!s.ok()) return err(s);
    } else if (req.verb == "RELEASE") {
        Status s = ledger.release(std::strtoull(req.get("lease").c_str(), nullptr, 10));
        if (!s.ok()) return err(s);
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
