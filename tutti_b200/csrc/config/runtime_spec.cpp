#include "runtime_spec.h"

#include <set>

namespace tutti {

namespace {

using yaml::Node;

Status field_error(const Node& n, const std::string& path, const std::string& what) {
    return {StatusCode::INVALID_ARGUMENT, "config line " + std::to_string(n.line) + ": " + path + ": " + what};
}

// Rejects any key not in `allowed`.
Status only_fields(const Node& n, const std::string& path, std::initializer_list<const char*> allowed) {
    if (n.kind == Node::Kind::Null) return Status::Ok();
    if (!n.is_map()) return field_error(n, path, "expected a mapping");
    for (const auto& kv : n.map) {
        bool ok = false;
        for (const char* a : allowed)
            if (kv.first == a) ok = true;
        if (!ok) return field_error(*kv.second, path + "." + kv.first, "unknown field");
    }
    return Status::Ok();
}

template <typename T>
Status get_uint(const Node& m, const char* key, const std::string& path, T& out) {
    const Node* v = m.get(key);
    if (!v || v->kind == Node::Kind::Null) return Status::Ok();
    auto r = yaml::as_int(*v, path + "." + key);
    if (!r.ok()) return r.status();
    if (r.value() < 0) return field_error(*v, path + "." + key, "must be >= 0");
    out = static_cast<T>(r.value());
    return Status::Ok();
}

Status get_str(const Node& m, const char* key, const std::string& path, std::string& out, bool required = false) {
    const Node* v = m.get(key);
    if (!v || v->kind == Node::Kind::Null) {
        if (required) return field_error(m, path + "." + key, "required");
        return Status::Ok();
    }
    auto r = yaml::as_string(*v, path + "." + key);
    if (!r.ok()) return r.status();
    out = r.value();
    return Status::Ok();
}

Status get_bool(const Node& m, const char* key, const std::string& path, bool& out) {
    const Node* v = m.get(key);
    if (!v || v->kind == Node::Kind::Null) return Status::Ok();
    auto r = yaml::as_bool(*v, path + "." + key);
    if (!r.ok()) return r.status();
    out = r.value();
    return Status::Ok();
}

Status parse_resource(const Node& n, const std::string& p, ResourceSpec& r) {
    TUTTI_RETURN_IF_ERROR(only_fields(n, p, {"id", "type", "provider", "allocation", "config"}));
    TUTTI_RETURN_IF_ERROR(get_str(n, "id", p, r.id, true));
    TUTTI_RETURN_IF_ERROR(get_str(n, "type", p, r.type, true));
    if (const Node* prov = n.get("provider")) {
        TUTTI_RETURN_IF_ERROR(only_fields(*prov, p + ".provider", {"type", "endpoint", "client"}));
        TUTTI_RETURN_IF_ERROR(get_str(*prov, "type", p + ".provider", r.provider, true));
        TUTTI_RETURN_IF_ERROR(get_str(*prov, "endpoint", p + ".provider", r.endpoint));
        TUTTI_RETURN_IF_ERROR(get_str(*prov, "client", p + ".provider", r.client));
    }
    if (const Node* a = n.get("allocation")) {
        const std::string ap = p + ".allocation";
        TUTTI_RETURN_IF_ERROR(only_fields(*a, ap, {"selection", "device_ids", "queues_per_controller"}));
        TUTTI_RETURN_IF_ERROR(get_str(*a, "selection", ap, r.selection));
        TUTTI_RETURN_IF_ERROR(get_uint(*a, "queues_per_controller", ap, r.queues_per_controller));
        if (const Node* ids = a->get("device_ids")) {
            if (!ids->is_seq()) return field_error(*ids, ap + ".device_ids", "expected a list");
            for (std::size_t i = 0; i < ids->seq.size(); ++i) {
                auto v = yaml::as_int(*ids->seq[i], ap + ".device_ids[" + std::to_string(i) + "]");
                if (!v.ok()) return v.status();
                r.device_ids.push_back(v.value());
            }
        }
    }
    if (const Node* c = n.get("config")) {
        const std::string cp = p + ".config";
        TUTTI_RETURN_IF_ERROR(only_fields(*c, cp, {"mounts", "queue_depth", "mdts_bytes", "lba_bytes",
                                                   "controller_threads", "direct_io"}));
        if (const Node* m = c->get("mounts")) {
            if (!m->is_seq()) return field_error(*m, cp + ".mounts", "expected a list");
            for (std::size_t i = 0; i < m->seq.size(); ++i) {
                auto v = yaml::as_string(*m->seq[i], cp + ".mounts[" + std::to_string(i) + "]");
                if (!v.ok()) return v.status();
                r.mounts.push_back(v.value());
            }
        }
        TUTTI_RETURN_IF_ERROR(get_uint(*c, "queue_depth", cp, r.queue_depth));
        TUTTI_RETURN_IF_ERROR(get_uint(*c, "mdts_bytes", cp, r.mdts_bytes));
        TUTTI_RETURN_IF_ERROR(get_uint(*c, "lba_bytes", cp, r.lba_bytes));
        TUTTI_RETURN_IF_ERROR(get_uint(*c, "controller_threads", cp, r.controller_threads));
        TUTTI_RETURN_IF_ERROR(get_bool(*c, "direct_io", cp, r.direct_io));
    }
    return Status::Ok();
}

Status parse_resolver(const Node& n, const std::string& p, ResolverSpec& r) {
    TUTTI_RETURN_IF_ERROR(only_fields(n, p, {"id", "type", "scheme", "config"}));
    TUTTI_RETURN_IF_ERROR(get_str(n, "id", p, r.id, true));
    TUTTI_RETURN_IF_ERROR(get_str(n, "type", p, r.type, true));
    TUTTI_RETURN_IF_ERROR(get_str(n, "scheme", p, r.scheme));
    if (const Node* c = n.get("config")) {
        const std::string cp = p + ".config";
        TUTTI_RETURN_IF_ERROR(only_fields(*c, cp, {"topology", "mapping", "md", "sysfs_root"}));
        TUTTI_RETURN_IF_ERROR(get_str(*c, "topology", cp, r.topology));
        TUTTI_RETURN_IF_ERROR(get_str(*c, "mapping", cp, r.mapping));
        TUTTI_RETURN_IF_ERROR(get_str(*c, "md", cp, r.md));
        TUTTI_RETURN_IF_ERROR(get_str(*c, "sysfs_root", cp, r.sysfs_root));
    }
    return Status::Ok();
}

Status parse_datapath(const Node& n, const std::string& p, DataPathSpec& d) {
    TUTTI_RETURN_IF_ERROR(only_fields(n, p, {"id", "type", "config"}));
    TUTTI_RETURN_IF_ERROR(get_str(n, "id", p, d.id, true));
    TUTTI_RETURN_IF_ERROR(get_str(n, "type", p, d.type, true));
    if (const Node* c = n.get("config")) {
        const std::string cp = p + ".config";
        TUTTI_RETURN_IF_ERROR(only_fields(*c, cp, {"leases", "max_ctas_per_op", "slots_per_lease", "slot_bytes",
                                                   "timeout_ms", "threads", "direct_io", "async_completion"}));
        TUTTI_RETURN_IF_ERROR(get_uint(*c, "leases", cp, d.leases));
        TUTTI_RETURN_IF_ERROR(get_uint(*c, "max_ctas_per_op", cp, d.max_ctas_per_op));
        TUTTI_RETURN_IF_ERROR(get_uint(*c, "slots_per_lease", cp, d.slots_per_lease));
        TUTTI_RETURN_IF_ERROR(get_uint(*c, "slot_bytes", cp, d.slot_bytes));
        TUTTI_RETURN_IF_ERROR(get_uint(*c, "timeout_ms", cp, d.timeout_ms));
        TUTTI_RETURN_IF_ERROR(get_uint(*c, "threads", cp, d.threads));
        TUTTI_RETURN_IF_ERROR(get_bool(*c, "direct_io", cp, d.direct_io));
        TUTTI_RETURN_IF_ERROR(get_bool(*c, "async_completion", cp, d.async_completion));
    }
    return Status::Ok();
}

Status parse_backend(const Node& n, const std::string& p, BackendSpec& b) {
    TUTTI_RETURN_IF_ERROR(only_fields(n, p, {"id", "contract", "resolver", "datapath", "resource", "config"}));
    TUTTI_RETURN_IF_ERROR(get_str(n, "id", p, b.id, true));
    TUTTI_RETURN_IF_ERROR(get_str(n, "contract", p, b.contract, true));
    TUTTI_RETURN_IF_ERROR(get_str(n, "resolver", p, b.resolver, true));
    TUTTI_RETURN_IF_ERROR(get_str(n, "datapath", p, b.datapath, true));
    TUTTI_RETURN_IF_ERROR(get_str(n, "resource", p, b.resource));
    if (const Node* c = n.get("config")) TUTTI_RETURN_IF_ERROR(only_fields(*c, p + ".config", {}));
    return Status::Ok();
}

template <typename T, typename F>
Status parse_list(const Node& parent, const char* key, const std::string& path, std::vector<T>& out, F fn) {
    const Node* l = parent.get(key);
    if (!l || l->kind == Node::Kind::Null) return Status::Ok();
    if (!l->is_seq()) return field_error(*l, path + "." + key, "expected a list");
    for (std::size_t i = 0; i < l->seq.size(); ++i) {
        T item;
        TUTTI_RETURN_IF_ERROR(fn(*l->seq[i], path + "." + key + "[" + std::to_string(i) + "]", item));
        out.push_back(std::move(item));
    }
    return Status::Ok();
}

}  // namespace

const ResourceSpec* TuttiRuntimeSpec::resource(const std::string& id) const {
    for (auto& r : resources)
        if (r.id == id) return &r;
    return nullptr;
}
const ResolverSpec* TuttiRuntimeSpec::resolver(const std::string& id) const {
    for (auto& r : resolvers)
        if (r.id == id) return &r;
    return nullptr;
}
const DataPathSpec* TuttiRuntimeSpec::datapath(const std::string& id) const {
    for (auto& d : datapaths)
        if (d.id == id) return &d;
    return nullptr;
}

Result<TuttiRuntimeSpec> parse_runtime_spec(const yaml::Node& root) {
    using R = Result<TuttiRuntimeSpec>;
    TuttiRuntimeSpec s;
    TUTTI_RETURN_IF_ERROR_R(R, only_fields(root, "$", {"accelerator", "runtime", "storage"}));
    if (const Node* a = root.get("accelerator")) {
        TUTTI_RETURN_IF_ERROR_R(R, only_fields(*a, "accelerator", {"profile"}));
        TUTTI_RETURN_IF_ERROR_R(R, get_str(*a, "profile", "accelerator", s.profile));
    }
    if (const Node* r = root.get("runtime")) {
        TUTTI_RETURN_IF_ERROR_R(R, only_fields(*r, "runtime", {"accel_id", "max_terminal_results"}));
        TUTTI_RETURN_IF_ERROR_R(R, get_uint(*r, "accel_id", "runtime", s.accel_id));
        TUTTI_RETURN_IF_ERROR_R(R, get_uint(*r, "max_terminal_results", "runtime", s.max_terminal_results));
    }
    const Node* st = root.get("storage");
    if (!st) return R::Failure({StatusCode::INVALID_ARGUMENT, "config: storage: required"});
    TUTTI_RETURN_IF_ERROR_R(R, only_fields(*st, "storage", {"resources", "resolvers", "datapaths", "backends"}));
    TUTTI_RETURN_IF_ERROR_R(R, parse_list(*st, "resources", "storage", s.resources, parse_resource));
    TUTTI_RETURN_IF_ERROR_R(R, parse_list(*st, "resolvers", "storage", s.resolvers, parse_resolver));
    TUTTI_RETURN_IF_ERROR_R(R, parse_list(*st, "datapaths", "storage", s.datapaths, parse_datapath));
    TUTTI_RETURN_IF_ERROR_R(R, parse_list(*st, "backends", "storage", s.backends, parse_backend));
    return s;
}

Result<TuttiRuntimeSpec> parse_runtime_config_file(const std::string& path) {
    auto n = yaml::parse_file(path);
    if (!n.ok()) return Result<TuttiRuntimeSpec>::Failure(n.status());
    return parse_runtime_spec(*n.value());
}

Result<TuttiRuntimeSpec> parse_runtime_config_text(const std::string& text) {
    auto n = yaml::parse(text);
    if (!n.ok()) return Result<TuttiRuntimeSpec>::Failure(n.status());
    return parse_runtime_spec(*n.value());
}

Status validate_runtime_spec(const TuttiRuntimeSpec& s) {
    auto bad = [](const std::string& m) { return Status(StatusCode::INVALID_ARGUMENT, "spec: " + m); };
    if (s.profile != "CUDA") return bad("accelerator.profile must be CUDA (this build targets sm_100a)");
    std::set<std::string> ids;
    auto unique = [&](const std::string& id, const char* what) -> Status {
        if (id.empty()) return bad(std::string(what) + " without id");
        if (!ids.insert(id).second) return bad("duplicate id '" + id + "'");
        return Status::Ok();
    };
    for (auto& r : s.resources) {
        TUTTI_RETURN_IF_ERROR(unique(r.id, "resource"));
        if (r.type != "nvme" && r.type != "memory") return bad("resource " + r.id + ": type must be nvme or memory");
        if (r.type == "nvme") {
            if (r.provider != "emulated" && r.provider != "nvme-service")
                return bad("resource " + r.id + ": provider must be emulated or nvme-service");
            if (r.provider == "nvme-service" && r.endpoint.empty())
                return bad("resource " + r.id + ": nvme-service needs provider.endpoint");
            if (r.provider == "emulated" && r.mounts.empty())
                return bad("resource " + r.id + ": emulated provider needs config.mounts");
            if (r.provider == "emulated" && !r.device_ids.empty() && r.device_ids.size() != r.mounts.size())
                return bad("resource " + r.id + ": one mount per device id");
            // "explicit" is Tutti's name for an explicit list of device ids
            if (r.selection != "device-group" && r.selection != "single" && r.selection != "explicit")
                return bad("resource " + r.id + ": selection must be device-group, single or explicit");
        }
    }
    for (auto& r : s.resolvers) {
        TUTTI_RETURN_IF_ERROR(unique(r.id, "resolver"));
        if (r.type != "local-file") return bad("resolver " + r.id + ": type must be local-file");
        if (r.topology != "single" && r.topology != "multi-mount" && r.topology != "raid0")
            return bad("resolver " + r.id + ": topology must be single, multi-mount or raid0");
        if (r.mapping != "auto" && r.mapping != "fiemap" && r.mapping != "synthetic")
            return bad("resolver " + r.id + ": mapping must be auto, fiemap or synthetic");
    }
    for (auto& d : s.datapaths) {
        TUTTI_RETURN_IF_ERROR(unique(d.id, "datapath"));
        if (d.type != "nvme-device-group" && d.type != "local-nvme" && d.type != "posix")
            return bad("datapath " + d.id + ": type must be nvme-device-group, local-nvme or posix");
        if (d.slots_per_lease == 0 || d.slots_per_lease > 16) return bad("datapath " + d.id + ": slots_per_lease 1..16");
        if (d.leases == 0) return bad("datapath " + d.id + ": leases must be > 0");
    }
    for (auto& b : s.backends) TUTTI_RETURN_IF_ERROR(unique(b.id, "backend"));
    if (s.backends.size() != 1) return bad("exactly one backend is required");
    const BackendSpec& b = s.backends[0];
    const ResolverSpec* rs = s.resolver(b.resolver);
    const DataPathSpec* ds = s.datapath(b.datapath);
    const ResourceSpec* res = b.resource.empty() ? nullptr : s.resource(b.resource);
    if (!rs) return bad("backend " + b.id + ": unknown resolver '" + b.resolver + "'");
    if (!ds) return bad("backend " + b.id + ": unknown datapath '" + b.datapath + "'");
    if (!b.resource.empty() && !res) return bad("backend " + b.id + ": unknown resource '" + b.resource + "'");
    if (b.contract == "nvme-device-group") {
        if (ds->type != "nvme-device-group" && ds->type != "local-nvme")
            return bad("contract nvme-device-group needs an nvme datapath");
        if (!res || res->type != "nvme") return bad("contract nvme-device-group needs an nvme resource");
    } else if (b.contract == "ext4-local-nvme") {
        if (ds->type != "local-nvme") return bad("contract ext4-local-nvme needs a local-nvme datapath");
        if (rs->topology != "single") return bad("contract ext4-local-nvme needs a single-mount resolver");
        if (!res || res->type != "nvme") return bad("contract ext4-local-nvme needs an nvme resource");
        const std::size_t ndev = res->provider == "emulated" ? res->mounts.size() : res->device_ids.size();
        if (ndev != 1) return bad("contract ext4-local-nvme needs exactly one device");
    } else if (b.contract == "posix") {
        if (ds->type != "posix") return bad("contract posix needs a posix datapath");
        if (res && res->type == "nvme" && res->provider == "nvme-service")
            return bad("contract posix cannot lease NVMe queues");
    } else {
        return bad("backend " + b.id + ": unknown contract '" + b.contract + "'");
    }
    return Status::Ok();
}

}  // namespace tutti
