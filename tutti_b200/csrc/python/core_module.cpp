// tutti_b200._core: Python bindings of the native runtime.
//
// Parity: reference csrc/python/src/_core.cpp:254-293 (submit), :824-853
// (preset factories), :1222-1312 (module: Runtime, ObjectStore, make_*_runtime).
// Handles cross the boundary as packed 64-bit integers (slot << 32 | generation).

#include <execinfo.h>
#include <fcntl.h>
#include <signal.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <sys/stat.h>
#include <unistd.h>

#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <tutti/storage_runtime.h>

#include "../datapaths/gpu_nvme_data_path.h"
#include "../datapaths/posix_data_path.h"
#include "../nvme/controller.h"
#include "../objects/digest.h"
#include "../objects/object_store.h"
#include "../config/runtime_spec.h"
#include "../daemon/lease_ledger.h"
#include "../resolvers/file_resolvers.h"
#include "../runtime/tutti_runtime.h"
#include "presets.h"

namespace py = pybind11;
using namespace tutti;

namespace {

[[noreturn]] void raise(const Status& s) {
    if (s.code() == StatusCode::NOT_FOUND) throw py::key_error(s.to_string());
    if (s.code() == StatusCode::INVALID_ARGUMENT || s.code() == StatusCode::OUT_OF_RANGE)
        throw py::value_error(s.to_string());
    throw std::runtime_error(s.to_string());
}
template <typename T>
T unwrap(Result<T> r) {
    if (!r.ok()) raise(r.status());
    return std::move(r).value();
}
void check(const Status& s) {
    if (!s.ok()) raise(s);
}

template <typename H>
std::uint64_t pack(const H& h) {
    return (std::uint64_t(h.slot()) << 32) | (h.generation() & 0xFFFFFFFFull);
}
template <typename H>
H unpack(std::uint32_t rid, std::uint64_t v) {
    return H::from_raw(rid, static_cast<std::uint32_t>(v >> 32), v & 0xFFFFFFFFull);
}

const char* state_name(IoState s) {
    return s == IoState::IN_FLIGHT ? "in_flight" : s == IoState::COMPLETED ? "completed" : "failed";
}
const char* kind_name(IoFailureKind k) {
    switch (k) {
        case IoFailureKind::NONE: return "none";
        case IoFailureKind::RESOLVE_LBA: return "resolve_lba";
        case IoFailureKind::CQ_TIMEOUT: return "cq_timeout";
        case IoFailureKind::NVME_CQ_ERROR: return "nvme_cq_error";
        case IoFailureKind::CUDA_QUERY_ERROR: return "cuda_query_error";
        case IoFailureKind::STATUS_D2H_ERROR: return "status_d2h_error";
        default: return "unknown";
    }
}

py::dict result_dict(const IoResult& r) {
    py::dict d;
    d["state"] = state_name(r.state);
    d["ok"] = r.state == IoState::COMPLETED;
    d["status"] = r.status.to_string();
    d["confirmed_bytes"] = r.detail.confirmed_bytes;
    d["timeout_seen"] = r.detail.timeout_seen;
    d["failure_kind"] = kind_name(r.detail.failure_kind);
    d["raw_cq_status"] = r.detail.raw_cq_status;
    d["failed_request_indices"] = r.detail.failed_request_indices;
    return d;
}

MemoryKind parse_kind(const std::string& k) {
    if (k == "device") return MemoryKind::DEVICE;
    if (k == "pinned") return MemoryKind::PINNED_HOST;
    if (k == "host") return MemoryKind::HOST;
    if (k == "managed") return MemoryKind::MANAGED;
    throw py::value_error("memory kind must be device|pinned|host|managed");
}

// Python-facing runtime: owns the StorageRuntime and anything its components need.
struct PyRuntime {
    std::shared_ptr<TuttiRuntime> assembly;  // spec-assembled runtimes: lease + controllers (outlive rt)
    std::unique_ptr<StorageRuntime> rt;
    PresetExtras extras;
    std::uint32_t rid() const {
        // runtime id is carried by every handle minted; recover it from a probe
        return rid_;
    }
    std::uint32_t rid_ = 0;
};

std::shared_ptr<PyRuntime> wrap(PresetResult pr) {
    auto r = std::make_shared<PyRuntime>();
    r->rt = std::move(pr.runtime);
    r->extras = std::move(pr.extras);
    // Mint-and-discard to learn the runtime id (handles carry it).
    r->rid_ = pr.runtime_id;
    return r;
}

void segv_trace(int sig) {
    void* frames[64];
    int n = backtrace(frames, 64);
    backtrace_symbols_fd(frames, n, 2);
    signal(sig, SIG_DFL);
    ::raise(sig);
}

}  // namespace

PYBIND11_MODULE(_core, m) {
    // Debug aid: TUTTI_SEGV_TRACE=1 prints a native backtrace on SIGSEGV/SIGBUS.
    if (std::getenv("TUTTI_SEGV_TRACE")) {
        signal(SIGSEGV, segv_trace);
        signal(SIGBUS, segv_trace);
    }
    m.doc() = "tutti_b200 native runtime (StorageRuntime, object store, NVMe data paths)";

    py::class_<PyRuntime, std::shared_ptr<PyRuntime>>(m, "Runtime")
        .def_property_readonly("accel_id", [](PyRuntime& r) { return r.rt->accel_id(); })
        .def("caps",
             [](PyRuntime& r) {
                 py::list out;
                 for (auto& c : r.rt->data_path_capabilities()) {
                     py::dict d;
                     d["name"] = c.name;
                     d["device_execution"] = c.supports_device_execution;
                     d["host_execution"] = c.supports_host_execution;
                     d["target_alignment"] = c.target_alignment_bytes;
                     d["memory_alignment"] = c.memory_alignment_bytes;
                     d["length_alignment"] = c.length_alignment_bytes;
                     d["max_single_io_bytes"] = c.max_single_io_bytes;
                     d["max_batch_requests"] = c.max_batch_requests;
                     d["bound_accel_id"] = c.bound_accel_id;
                     d["features"] = c.optional_target_features;
                     out.append(d);
                 }
                 return out;
             })
        .def(
            "register_memory",
            [](PyRuntime& r, std::uintptr_t ptr, std::uint64_t size, const std::string& kind, int accel,
               std::uint64_t granularity) {
                MemoryView v;
                v.address = reinterpret_cast<void*>(ptr);
                v.size = size;
                v.expected_kind = parse_kind(kind);
                v.expected_accel_id = accel;
                v.io_granularity = granularity;
                return pack(unwrap(r.rt->register_memory(v)));
            },
            py::arg("ptr"), py::arg("size"), py::arg("kind") = "device", py::arg("accel_id") = -1,
            py::arg("io_granularity") = 0)
        .def("unregister_memory",
             [](PyRuntime& r, std::uint64_t h) { check(r.rt->unregister_memory(unpack<MemoryHandle>(r.rid_, h))); })
        .def("allocate_memory",
             [](PyRuntime& r, std::uint64_t size, const std::string& kind) {
                 MemorySpec s;
                 s.size = size;
                 s.kind = parse_kind(kind);
                 auto a = unwrap(r.rt->allocate_memory(s));
                 return py::make_tuple(pack(a.handle), reinterpret_cast<std::uintptr_t>(a.address), a.size);
             })
        .def("free_memory",
             [](PyRuntime& r, std::uint64_t h) { check(r.rt->free_memory(unpack<MemoryHandle>(r.rid_, h))); })
        .def("query_memory",
             [](PyRuntime& r, std::uint64_t h) {
                 auto i = unwrap(r.rt->query_memory(unpack<MemoryHandle>(r.rid_, h)));
                 py::dict d;
                 d["size"] = i.size;
                 d["address"] = reinterpret_cast<std::uintptr_t>(i.address);
                 d["inflight"] = i.inflight_count;
                 d["runtime_owned"] = i.ownership == MemoryOwnership::RUNTIME_OWNED;
                 return d;
             })
        .def("open", [](PyRuntime& r, const std::string& uri) { return pack(unwrap(r.rt->open(uri))); })
        .def(
            "open_batch",
            [](PyRuntime& r, const std::vector<std::string>& uris, bool strict) {
                std::vector<Result<TargetHandle>> res;
                {
                    py::gil_scoped_release nogil;
                    res = r.rt->open_batch(uris);
                }
                py::list out;
                for (auto& x : res) {
                    if (x.ok())
                        out.append(pack(x.value()));
                    else if (strict)
                        raise(x.status());
                    else
                        out.append(py::str(x.status().to_string()));
                }
                return out;
            },
            py::arg("uris"), py::arg("strict") = true)
        .def("close", [](PyRuntime& r, std::uint64_t h) { check(r.rt->close(unpack<TargetHandle>(r.rid_, h))); })
        .def("query_target",
             [](PyRuntime& r, std::uint64_t h) {
                 auto t = unwrap(r.rt->query_target(unpack<TargetHandle>(r.rid_, h)));
                 py::dict d;
                 d["uri"] = t.uri;
                 d["size"] = t.logical_size;
                 d["inflight"] = t.inflight_count;
                 d["data_path"] = t.data_path_key;
                 return d;
             })
        .def(
            "submit_arrays",
            [](PyRuntime& r, const std::string& direction, py::array_t<std::uint64_t, py::array::c_style> mem,
               py::array_t<std::uint64_t, py::array::c_style> mem_off,
               py::array_t<std::uint64_t, py::array::c_style> tgt,
               py::array_t<std::uint64_t, py::array::c_style> tgt_off,
               py::array_t<std::uint64_t, py::array::c_style> len, std::uintptr_t stream, bool host_exec,
               py::array_t<std::uint8_t, py::array::c_style> directions) {
                const std::size_t n = static_cast<std::size_t>(len.size());
                if (mem_off.size() != static_cast<py::ssize_t>(n) || tgt_off.size() != static_cast<py::ssize_t>(n) ||
                    (mem.size() != 1 && mem.size() != static_cast<py::ssize_t>(n)) ||
                    (tgt.size() != 1 && tgt.size() != static_cast<py::ssize_t>(n)))
                    throw py::value_error("array lengths differ");
                // "mixed": directions[i] is 0 (read) or 1 (write) per request
                const bool mixed = direction == "mixed";
                const IoDirection dir = direction == "read" ? IoDirection::READ : IoDirection::WRITE;
                if (direction != "read" && direction != "write" && !mixed)
                    throw py::value_error("direction read|write|mixed");
                if (mixed && directions.size() != static_cast<py::ssize_t>(n))
                    throw py::value_error("mixed: one direction per request");
                std::vector<IoRequest> reqs(n);
                auto pm = mem.unchecked<1>(), pmo = mem_off.unchecked<1>(), pt = tgt.unchecked<1>(),
                     pto = tgt_off.unchecked<1>(), pl = len.unchecked<1>();
                const bool one_mem = mem.size() == 1, one_tgt = tgt.size() == 1;
                const std::uint8_t* pd = mixed ? directions.data() : nullptr;
                for (std::size_t i = 0; i < n; ++i) {
                    reqs[i].direction = mixed ? (pd[i] ? IoDirection::WRITE : IoDirection::READ) : dir;
                    reqs[i].memory = unpack<MemoryHandle>(r.rid_, pm(one_mem ? 0 : i));
                    reqs[i].memory_offset = pmo(i);
                    reqs[i].target = unpack<TargetHandle>(r.rid_, pt(one_tgt ? 0 : i));
                    reqs[i].target_offset = pto(i);
                    reqs[i].length = pl(i);
                }
                HostSubmitContext ctx;
                ctx.execution_domain = host_exec ? ExecutionDomain::HOST_EXECUTION : ExecutionDomain::DEVICE_EXECUTION;
                ctx.accel_id = -1;
                ctx.stream = reinterpret_cast<cudaStream_t>(stream);
                IoSubmitOutcome o;
                const auto t_built = std::chrono::steady_clock::now();
                {
                    py::gil_scoped_release nogil;
                    o = r.rt->submit(reqs.data(), n, ctx);
                }
                const auto t_sub = std::chrono::steady_clock::now();
                py::dict d;
                if (std::getenv("TUTTI_SUBMIT_PROFILE")) {
                    d["runtime_submit_ms"] =
                        std::chrono::duration<double, std::milli>(t_sub - t_built).count();
                    if (r.extras.gpu_path) {
                        const auto sp = r.extras.gpu_path->last_submit_profile();
                        d["dp_coalesce_ms"] = sp.coalesce_ms;
                        d["dp_launch_ms"] = sp.launch_ms;
                        d["dp_commands"] = sp.commands;
                    }
                }
                d["io"] = o.io ? py::cast(pack(*o.io)) : py::none();
                d["status"] = o.status.to_string();
                d["ok"] = o.status.ok();
                std::vector<std::uint32_t> rejected;
                std::vector<std::string> reasons;
                for (std::size_t i = 0; i < n; ++i)
                    if (o.initial_states[i].state == IoRequestState::REJECTED) {
                        rejected.push_back(static_cast<std::uint32_t>(i));
                        if (reasons.size() < 8) reasons.push_back(o.initial_states[i].status.to_string());
                    }
                d["rejected"] = rejected;
                d["reasons"] = reasons;
                return d;
            },
            py::arg("direction"), py::arg("mem"), py::arg("mem_offsets"), py::arg("targets"),
            py::arg("target_offsets"), py::arg("lengths"), py::arg("stream") = 0, py::arg("host_exec") = false,
            py::arg("directions") = py::array_t<std::uint8_t>())
        .def(
            "submit_paged",
            [](PyRuntime& r, const std::string& direction, std::uint64_t mem,
               py::array_t<std::uint64_t, py::array::c_style> chunk_targets,
               py::array_t<std::uint64_t, py::array::c_style> chunk_offsets,
               py::array_t<std::int64_t, py::array::c_style> block_ids, py::array_t<std::int64_t, py::array::c_style> layers,
               py::dict geo, std::uintptr_t stream, bool host_exec,
               py::array_t<std::uint64_t, py::array::c_style> layer_mems,
               py::array_t<std::uint64_t, py::array::c_style> chunk_mems,
               py::array_t<std::uint64_t, py::array::c_style> chunk_layer_mems) {
                // layer_mems (optional): one memory handle per model layer, for engines that
                // allocate each layer's KV separately; offsets then omit the layer term.
                // chunk_mems (optional): one whole-pool memory handle per chunk (e.g. the
                // pool of the TP rank that chunk is restored for, reached over NVLink).
                // chunk_layer_mems (optional, [chunks, model layers]): per-layer caches of
                // the rank each chunk lands in; one submission can then serve several
                // ranks, and chunks named for several ranks are read once (replica merge).
                const bool per_chunk_layer = chunk_layer_mems.size() > 0;
                const bool per_layer = layer_mems.size() > 0 || per_chunk_layer;
                const bool per_chunk = chunk_mems.size() > 0;
                if (per_chunk && chunk_mems.size() != chunk_targets.size())
                    throw py::value_error("chunk_mems needs one handle per chunk");
                if (per_chunk_layer && (per_chunk || layer_mems.size() > 0 || chunk_layer_mems.ndim() != 2 ||
                                        chunk_layer_mems.shape(0) != chunk_targets.size()))
                    throw py::value_error("chunk_layer_mems is [chunks, layers] and excludes layer_mems and chunk_mems");
                auto lm = layer_mems.unchecked<1>();
                auto cm = chunk_mems.unchecked<1>();
                const std::size_t clm_layers = per_chunk_layer ? static_cast<std::size_t>(chunk_layer_mems.shape(1)) : 0;
                const std::uint64_t* clm = per_chunk_layer ? chunk_layer_mems.data() : nullptr;
                // Requests of a paged restore/store in (chunk, layer, block, plane) order:
                //   target_offset = chunk_offset + layer*segment + j*block_layer + plane*plane_bytes
                //   memory_offset = ((layer*planes + plane)*num_blocks + block) * plane_bytes
                const std::uint64_t planes = geo["planes"].cast<std::uint64_t>();
                const std::uint64_t plane_bytes = geo["plane_bytes"].cast<std::uint64_t>();
                const std::uint64_t segment = geo["segment_bytes"].cast<std::uint64_t>();
                const std::uint64_t block_layer = geo["block_layer_bytes"].cast<std::uint64_t>();
                const std::uint64_t num_blocks = geo["num_blocks"].cast<std::uint64_t>();
                // Stored format (optional): with the fp8 block transform the target-side
                // plane and block strides are the stored (33/64) sizes.
                const std::uint32_t transform = geo.contains("transform") ? geo["transform"].cast<std::uint32_t>() : 0u;
                const std::uint64_t splane =
                    geo.contains("stored_plane_bytes") ? geo["stored_plane_bytes"].cast<std::uint64_t>() : plane_bytes;
                const std::uint64_t sblock = geo.contains("stored_block_layer_bytes")
                                                 ? geo["stored_block_layer_bytes"].cast<std::uint64_t>()
                                                 : block_layer;
                const std::size_t n = static_cast<std::size_t>(chunk_targets.size());
                if (chunk_offsets.size() != static_cast<py::ssize_t>(n) || block_ids.ndim() != 2 ||
                    block_ids.shape(0) != static_cast<py::ssize_t>(n))
                    throw py::value_error("chunk arrays / block table shape mismatch");
                const std::size_t bpc = static_cast<std::size_t>(block_ids.shape(1));
                const std::size_t nl = static_cast<std::size_t>(layers.size());
                if (direction != "read" && direction != "write") throw py::value_error("direction read|write");
                const IoDirection dir = direction == "read" ? IoDirection::READ : IoDirection::WRITE;
                auto ct = chunk_targets.unchecked<1>();
                auto co = chunk_offsets.unchecked<1>();
                auto bt = block_ids.unchecked<2>();
                auto ly = layers.unchecked<1>();
                std::vector<IoRequest> reqs(n * nl * bpc * planes);
                const MemoryHandle mh = unpack<MemoryHandle>(r.rid_, mem);
                std::size_t k = 0;
                for (std::size_t c = 0; c < n; ++c) {
                    const TargetHandle th = unpack<TargetHandle>(r.rid_, ct(c));
                    for (std::size_t l = 0; l < nl; ++l) {
                        const std::uint64_t L = static_cast<std::uint64_t>(ly(l));
                        if (per_chunk_layer ? L >= clm_layers
                                            : (per_layer && !per_chunk && L >= static_cast<std::uint64_t>(layer_mems.size())))
                            throw py::value_error("layer beyond layer_mems");
                        const MemoryHandle lmh = per_chunk_layer ? unpack<MemoryHandle>(r.rid_, clm[c * clm_layers + L])
                                                 : per_chunk     ? unpack<MemoryHandle>(r.rid_, cm(c))
                                                 : per_layer     ? unpack<MemoryHandle>(r.rid_, lm(L))
                                                                 : mh;
                        const std::uint64_t lterm = (per_layer && !per_chunk) ? 0 : L * planes;
                        for (std::size_t j = 0; j < bpc; ++j) {
                            const std::int64_t b = bt(c, j);
                            if (b < 0 || static_cast<std::uint64_t>(b) >= num_blocks)
                                throw py::value_error("block id out of range");
                            for (std::uint64_t p = 0; p < planes; ++p) {
                                IoRequest& q = reqs[k++];
                                q.direction = dir;
                                q.memory = lmh;
                                q.memory_offset = ((lterm + p) * num_blocks + static_cast<std::uint64_t>(b)) * plane_bytes;
                                q.target = th;
                                q.target_offset = co(c) + L * segment + j * sblock + p * splane;
                                q.length = plane_bytes;
                            }
                        }
                    }
                }
                HostSubmitContext ctx;
                ctx.execution_domain = host_exec ? ExecutionDomain::HOST_EXECUTION : ExecutionDomain::DEVICE_EXECUTION;
                ctx.accel_id = -1;
                ctx.stream = reinterpret_cast<cudaStream_t>(stream);
                if (transform > 1) throw py::value_error("transform: 0 (none) or 1 (fp8 e4m3, 1x128 scales)");
                ctx.transform = static_cast<IoTransform>(transform);
                IoSubmitOutcome o;
                {
                    py::gil_scoped_release nogil;
                    o = r.rt->submit(reqs.data(), reqs.size(), ctx);
                }
                py::dict d;
                d["io"] = o.io ? py::cast(pack(*o.io)) : py::none();
                d["status"] = o.status.to_string();
                d["ok"] = o.status.ok();
                d["count"] = reqs.size();
                std::vector<std::uint32_t> rejected;
                std::vector<std::string> reasons;
                for (std::size_t i = 0; i < reqs.size(); ++i)
                    if (o.initial_states[i].state == IoRequestState::REJECTED) {
                        rejected.push_back(static_cast<std::uint32_t>(i));
                        if (reasons.size() < 8) reasons.push_back(o.initial_states[i].status.to_string());
                    }
                d["rejected"] = rejected;
                d["reasons"] = reasons;
                return d;
            },
            py::arg("direction"), py::arg("mem"), py::arg("chunk_targets"), py::arg("chunk_offsets"),
            py::arg("block_ids"), py::arg("layers"), py::arg("geometry"), py::arg("stream") = 0,
            py::arg("host_exec") = false, py::arg("layer_mems") = py::array_t<std::uint64_t>(),
            py::arg("chunk_mems") = py::array_t<std::uint64_t>(),
            py::arg("chunk_layer_mems") = py::array_t<std::uint64_t>())
        .def("query_io",
             [](PyRuntime& r, std::uint64_t io) {
                 auto s = unwrap(r.rt->query(unpack<IoHandle>(r.rid_, io)));
                 return std::string(state_name(s.state));
             })
        .def(
            "wait",
            [](PyRuntime& r, std::uint64_t io, std::uint64_t timeout_ms) -> py::object {
                WaitOutcome w;
                {
                    py::gil_scoped_release nogil;
                    w = r.rt->wait(unpack<IoHandle>(r.rid_, io), timeout_ms);
                }
                if (w.observation_status.code() == StatusCode::TIMEOUT) return py::none();
                if (!w.observation_status.ok()) raise(w.observation_status);
                return result_dict(*w.result);
            },
            py::arg("io"), py::arg("timeout_ms") = 60000)
        .def("release_io", [](PyRuntime& r, std::uint64_t io) { check(r.rt->release_io(unpack<IoHandle>(r.rid_, io))); })
        .def("enqueue_wait",
             [](PyRuntime& r, const std::vector<std::uint64_t>& ios, std::uintptr_t stream) {
                 std::vector<IoHandle> hs;
                 for (auto v : ios) hs.push_back(unpack<IoHandle>(r.rid_, v));
                 check(r.rt->enqueue_wait(hs.data(), hs.size(), reinterpret_cast<cudaStream_t>(stream)));
             })
        .def("unreleased_terminal_results", [](PyRuntime& r) { return r.rt->unreleased_terminal_results(); })
        .def(
            "testing_force_complete",
            [](PyRuntime& r, std::uint64_t io, const std::string& state) {
                // stub runtimes only: their IOs have no DataPath to complete them
                IoState terminal;
                if (state == "COMPLETED")
                    terminal = IoState::COMPLETED;
                else if (state == "FAILED")
                    terminal = IoState::FAILED;
                else
                    throw py::value_error("state must be 'COMPLETED' or 'FAILED', got '" + state + "'");
                check(r.rt->testing_force_complete(unpack<IoHandle>(r.rid_, io), terminal));
            },
            py::arg("io"), py::arg("state"))
        .def(
            "shutdown",
            [](PyRuntime& r, std::uint64_t timeout_ms) {
                Status st;
                {
                    py::gil_scoped_release nogil;
                    st = r.rt->shutdown(timeout_ms);
                }
                check(st);
            },
            py::arg("timeout_ms") = 10000)
        .def("state",
             [](PyRuntime& r) {
                 auto s = r.rt->state();
                 return std::string(s == RuntimeState::RUNNING ? "running" : s == RuntimeState::DRAINING ? "draining" : "stopped");
             })
        .def("flush_devices",
             [](PyRuntime& r) {
                 // every completed WRITE durable in its file (drives with a write cache write back)
                 py::gil_scoped_release nogil;
                 for (auto& c : r.extras.controllers) {
                     Status s = c->flush();
                     if (!s.ok()) throw std::runtime_error(s.to_string());
                 }
             })
        .def("controller_stats",
             [](PyRuntime& r) {
                 py::list out;
                 for (auto& c : r.extras.controllers) {
                     auto s = c->stats();
                     py::dict d;
                     d["name"] = c->info().name;
                     d["kind"] = c->info().kind;
                     d["emulated"] = c->emulated_drive() != nullptr;  // the drive's DMA runs in this process
                     d["queues"] = c->info().num_io_queues;
                     d["commands"] = s.commands;
                     d["read_bytes"] = s.read_bytes;
                     d["write_bytes"] = s.write_bytes;
                     d["errors"] = s.errors;
                     d["injected"] = s.injected;
                     d["dma_copies"] = s.dma_copies;
                     d["green_streams"] = s.green_streams;
                     d["image_bytes"] = s.image_bytes;
                     d["load_ms"] = s.load_ns / 1e6;
                     d["file_ms"] = s.file_ns / 1e6;
                     d["sync_ms"] = s.sync_ns / 1e6;
                     d["max_command_ms"] = s.max_command_ns / 1e6;
                     d["device_dma"] = c->info().device_dma;
                     out.append(d);
                 }
                 return out;
             })
        .def(
            "inject",
            [](PyRuntime& r, int device, const std::string& kind, std::uint32_t count, std::uint32_t delay_us,
               std::uint32_t status) {
                if (device < 0 || device >= static_cast<int>(r.extras.controllers.size()))
                    throw py::index_error("device index");
                auto* emu = r.extras.controllers[device]->emulated_drive();
                if (!emu) throw py::value_error("injection needs an emulated controller");
                nvme::InjectKind k = kind == "media_error"     ? nvme::InjectKind::MEDIA_ERROR
                                     : kind == "drop_completion" ? nvme::InjectKind::DROP_COMPLETION
                                     : kind == "delay"           ? nvme::InjectKind::DELAY
                                                                 : nvme::InjectKind::NONE;
                emu->inject(k, count, delay_us, status);
            },
            py::arg("device"), py::arg("kind"), py::arg("count") = 1, py::arg("delay_us") = 0, py::arg("status") = 0)
        .def(
            "testing_inject_data_path",
            [](PyRuntime& r, const std::string& kind, std::uint32_t count) {
                if (!r.extras.gpu_path) throw py::value_error("data-path injection needs the nvme-gpu data path");
                using F = GpuNvmeDataPath::TestFault;
                F f = kind == "launch_failure"         ? F::LAUNCH_FAILURE
                      : kind == "event_record_failure" ? F::EVENT_RECORD_FAILURE
                      : kind == "query_error"          ? F::QUERY_ERROR
                                                       : throw py::value_error("unknown injection " + kind);
                r.extras.gpu_path->test_inject(f, count);
            },
            py::arg("kind"), py::arg("count") = 1)
        .def("memfs_usage",
             [](PyRuntime& r) {
                 if (!r.extras.memfs_budget) throw py::value_error("not a memfs runtime");
                 py::dict d;
                 d["capacity"] = r.extras.memfs_budget->capacity();
                 d["used"] = r.extras.memfs_budget->used();
                 return d;
             })
        .def("memfs_remove",
             [](PyRuntime& r, const std::string& name) {
                 if (!r.extras.memfs_resolver) throw py::value_error("not a memfs runtime");
                 check(r.extras.memfs_resolver->remove(name));
             })
        .def("last_submit_profile",
             [](PyRuntime& r) {
                 py::dict d;
                 if (!r.extras.gpu_path) return d;
                 const auto sp = r.extras.gpu_path->last_submit_profile();
                 d["coalesce_ms"] = sp.coalesce_ms;
                 d["launch_ms"] = sp.launch_ms;
                 d["commands"] = sp.commands;
                 d["requests"] = sp.requests;
                 d["h2d_bytes"] = sp.h2d_bytes;
                 d["d2h_bytes"] = sp.d2h_bytes;
                 return d;
             })
        .def("io_timing",
             [](PyRuntime& r) {
                 py::dict d;
                 if (!r.extras.gpu_path) return d;
                 auto t = r.extras.gpu_path->last_timing();
                 d["commands"] = t.commands;
                 d["queue_wait_us_p50"] = t.queue_wait_us_p50;
                 d["device_us_p50"] = t.device_us_p50;
                 d["device_us_p99"] = t.device_us_p99;
                 d["move_us_p50"] = t.move_us_p50;
                 d["total_us_p50"] = t.total_us_p50;
                 d["total_us_p99"] = t.total_us_p99;
                 return d;
             })
        .def("staging_on_device",
             [](PyRuntime& r) { return r.extras.gpu_path ? r.extras.gpu_path->staging_on_device() : false; })
        .def("free_leases", [](PyRuntime& r) {
            return r.extras.gpu_path ? r.extras.gpu_path->free_leases() : 0u;
        })
        // For the allocation-free C entry point: the GPU DataPath's address and
        // the DataPath target row behind a target handle.
        .def("gpu_path_address",
             [](PyRuntime& r) { return reinterpret_cast<std::uintptr_t>(r.extras.gpu_path.get()); })
        .def("target_row", [](PyRuntime& r, std::uint64_t h) {
            return unwrap(r.rt->data_path_target(unpack<TargetHandle>(r.rid_, h))).token;
        });

    m.def(
        "make_emulated_nvme_runtime",
        [](int accel_id, const std::vector<std::string>& mounts, py::dict opts) {
            EmulatedPresetOptions o;
            o.accel_id = accel_id;
            o.mounts = mounts;
            if (opts.contains("queues")) o.queues = opts["queues"].cast<std::uint32_t>();
            if (opts.contains("queue_depth")) o.queue_depth = opts["queue_depth"].cast<std::uint32_t>();
            if (opts.contains("mdts_bytes")) o.mdts_bytes = opts["mdts_bytes"].cast<std::uint32_t>();
            if (opts.contains("lba_bytes")) o.lba_bytes = opts["lba_bytes"].cast<std::uint32_t>();
            if (opts.contains("controller_threads")) o.controller_threads = opts["controller_threads"].cast<std::uint32_t>();
            if (opts.contains("direct_io")) o.direct_io = opts["direct_io"].cast<bool>();
            if (opts.contains("emulator_skip_data")) o.skip_data = opts["emulator_skip_data"].cast<bool>();
            if (opts.contains("emulator_idle_spins")) o.idle_spin_iters = opts["emulator_idle_spins"].cast<std::uint32_t>();
            if (opts.contains("emulator_reads")) {
                const std::string how = opts["emulator_reads"].cast<std::string>();
                if (how != "mmap" && how != "pread") throw py::value_error("emulator_reads: mmap|pread");
                o.map_reads = how == "mmap";
            }
            if (opts.contains("emulator_media")) o.media = opts["emulator_media"].cast<std::string>();
            if (opts.contains("nvme_provider")) o.provider = opts["nvme_provider"].cast<std::string>();
            if (opts.contains("snvme_nodes")) o.snvme_nodes = opts["snvme_nodes"].cast<std::vector<std::string>>();
            if (opts.contains("snvme_rings_in_gpu_memory"))
                o.snvme_rings_in_gpu_memory = opts["snvme_rings_in_gpu_memory"].cast<bool>();
            if (opts.contains("image_budget_bytes")) o.image_budget_bytes = opts["image_budget_bytes"].cast<std::uint64_t>();
            if (opts.contains("emulator_write_back")) o.write_back = opts["emulator_write_back"].cast<bool>();
            if (opts.contains("drive_gbps")) o.drive_gbps = opts["drive_gbps"].cast<double>();
            if (opts.contains("staging")) {
                const std::string where = opts["staging"].cast<std::string>();
                if (where == "auto") o.gpu.staging = GpuNvmeConfig::Staging::AUTO;
                else if (where == "host") o.gpu.staging = GpuNvmeConfig::Staging::HOST;
                else if (where == "device") o.gpu.staging = GpuNvmeConfig::Staging::DEVICE;
                else throw py::value_error("staging: auto|host|device");
            }
            if (opts.contains("leases")) o.gpu.leases = opts["leases"].cast<std::uint32_t>();
            if (opts.contains("max_ctas_per_op")) o.gpu.max_ctas_per_op = opts["max_ctas_per_op"].cast<std::uint32_t>();
            if (opts.contains("slots_per_lease")) o.gpu.slots_per_lease = opts["slots_per_lease"].cast<std::uint32_t>();
            if (opts.contains("slot_bytes")) o.gpu.slot_bytes = opts["slot_bytes"].cast<std::uint32_t>();
            if (opts.contains("timeout_ms")) o.gpu.timeout_ns = opts["timeout_ms"].cast<std::uint64_t>() * 1000000ull;
            if (opts.contains("timing")) o.gpu.timing = opts["timing"].cast<bool>();
            {
                const char* env = std::getenv("TUTTI_ASYNC_COMPLETION");
                o.gpu.async_completion = env && *env && std::strcmp(env, "0") != 0;
            }
            if (opts.contains("async_completion")) o.gpu.async_completion = opts["async_completion"].cast<bool>();
            if (opts.contains("direct_reads")) o.gpu.direct_reads = opts["direct_reads"].cast<bool>();
            if (opts.contains("staging_write_combined"))
                o.gpu.staging_write_combined = opts["staging_write_combined"].cast<bool>();
            if (opts.contains("async_fallback_us"))
                o.gpu.async_fallback_us = opts["async_fallback_us"].cast<std::uint32_t>();
            if (opts.contains("mapping")) o.mapping = opts["mapping"].cast<std::string>();
            if (opts.contains("raid0_md")) o.raid0_md = opts["raid0_md"].cast<std::string>();
            if (opts.contains("sysfs_root")) o.sysfs_root = opts["sysfs_root"].cast<std::string>();
            if (opts.contains("max_terminal_results"))
                o.max_terminal_results = opts["max_terminal_results"].cast<std::uint64_t>();
            Result<PresetResult> pr = Result<PresetResult>::Failure({StatusCode::INTERNAL, "unset"});
            {
                py::gil_scoped_release nogil;
                pr = make_emulated_nvme_runtime(o);
            }
            return wrap(unwrap(std::move(pr)));
        },
        py::arg("accel_id"), py::arg("mounts"), py::arg("options") = py::dict());

    m.def(
        "make_posix_runtime",
        [](int accel_id, const std::vector<std::string>& mounts, py::dict opts) {
            PosixPresetOptions o;
            o.accel_id = accel_id;
            o.mounts = mounts;
            if (opts.contains("threads")) o.posix.threads = opts["threads"].cast<std::uint32_t>();
            if (opts.contains("direct_io")) o.posix.direct_io = opts["direct_io"].cast<bool>();
            if (opts.contains("inject_fail_every")) o.posix.inject_fail_every = opts["inject_fail_every"].cast<std::uint64_t>();
            if (opts.contains("max_terminal_results"))
                o.max_terminal_results = opts["max_terminal_results"].cast<std::uint64_t>();
            return wrap(unwrap(make_posix_runtime(o)));
        },
        py::arg("accel_id"), py::arg("mounts"), py::arg("options") = py::dict());

    m.def(
        "make_memfs_runtime",
        [](int accel_id, std::uint64_t capacity_bytes, std::uint64_t max_terminal_results) {
            MemfsPresetOptions o;
            o.accel_id = accel_id;
            o.capacity_bytes = capacity_bytes;
            o.max_terminal_results = max_terminal_results;
            return wrap(unwrap(make_memfs_runtime(o)));
        },
        py::arg("accel_id") = -1, py::arg("capacity_bytes") = 1ull << 30, py::arg("max_terminal_results") = 64);

    m.def(
        "parse_runtime_config",
        [](const std::string& text, bool validate) {
            auto s = unwrap(parse_runtime_config_text(text));
            if (validate) check(validate_runtime_spec(s));
            py::dict d;
            d["profile"] = s.profile;
            d["accel_id"] = s.accel_id;
            py::list res, rsl, dps, bes;
            for (auto& r : s.resources) {
                py::dict x;
                x["id"] = r.id;
                x["type"] = r.type;
                x["provider"] = r.provider;
                x["endpoint"] = r.endpoint;
                x["device_ids"] = r.device_ids;
                x["queues_per_controller"] = r.queues_per_controller;
                x["mounts"] = r.mounts;
                res.append(x);
            }
            for (auto& r : s.resolvers) {
                py::dict x;
                x["id"] = r.id;
                x["type"] = r.type;
                x["scheme"] = r.scheme;
                x["topology"] = r.topology;
                x["mapping"] = r.mapping;
                x["md"] = r.md;
                rsl.append(x);
            }
            for (auto& p : s.datapaths) {
                py::dict x;
                x["id"] = p.id;
                x["type"] = p.type;
                x["leases"] = p.leases;
                x["slots_per_lease"] = p.slots_per_lease;
                dps.append(x);
            }
            for (auto& b : s.backends) {
                py::dict x;
                x["id"] = b.id;
                x["contract"] = b.contract;
                x["resolver"] = b.resolver;
                x["datapath"] = b.datapath;
                x["resource"] = b.resource;
                bes.append(x);
            }
            d["resources"] = res;
            d["resolvers"] = rsl;
            d["datapaths"] = dps;
            d["backends"] = bes;
            return d;
        },
        py::arg("text"), py::arg("validate") = true);

    m.def(
        "make_runtime_from_config",
        [](const std::string& text_or_path, bool is_path) {
            Result<TuttiRuntimeSpec> spec = is_path ? parse_runtime_config_file(text_or_path)
                                                    : parse_runtime_config_text(text_or_path);
            if (!spec.ok()) raise(spec.status());
            Result<std::unique_ptr<TuttiRuntime>> tr = Result<std::unique_ptr<TuttiRuntime>>::Failure({StatusCode::INTERNAL, "unset"});
            {
                py::gil_scoped_release nogil;
                tr = TuttiRuntime::create(spec.value());
            }
            std::shared_ptr<TuttiRuntime> asmbl(unwrap(std::move(tr)).release());
            auto r = std::make_shared<PyRuntime>();
            r->assembly = asmbl;
            r->extras.controllers = asmbl->controllers;
            r->extras.gpu_path = asmbl->gpu_path;
            r->extras.posix_path = asmbl->posix_path;
            r->rt = asmbl->take_storage();
            r->rid_ = r->rt->runtime_id();
            return r;
        },
        py::arg("config"), py::arg("is_path") = false);

    m.def(
        "daemon_handle_request_selftest",
        [](const std::vector<std::string>& lines, py::list devices, py::list accelerators) {
            // Runs lines through an in-process ledger (protocol tests without a socket).
            std::vector<tutti::daemon::DeviceInfo> devs;
            for (auto item : devices) {
                auto d = item.cast<py::dict>();
                tutti::daemon::DeviceInfo info;
                info.id = d["id"].cast<std::int64_t>();
                info.mount = d["mount"].cast<std::string>();
                info.queues = d["queues"].cast<std::uint32_t>();
                if (d.contains("accelerators")) info.accelerators = d["accelerators"].cast<std::vector<std::int64_t>>();
                if (d.contains("pci")) info.pci = d["pci"].cast<std::string>();
                if (d.contains("chrdev")) info.chrdev = d["chrdev"].cast<std::string>();
                if (d.contains("available")) info.available = d["available"].cast<bool>();
                if (d.contains("diagnostic")) info.diagnostic = d["diagnostic"].cast<std::string>();
                if (d.contains("lba_bytes")) info.lba_bytes = d["lba_bytes"].cast<std::uint32_t>();
                devs.push_back(info);
            }
            tutti::daemon::LeaseLedger ledger(devs);
            std::vector<tutti::daemon::AcceleratorView> views;
            for (auto item : accelerators) {
                auto a = item.cast<py::dict>();
                views.push_back({a["accel_id"].cast<std::int64_t>(), a["view_root"].cast<std::string>()});
            }
            ledger.set_accelerators(views);
            std::vector<std::string> out;
            for (auto& l : lines) out.push_back(tutti::daemon::handle_request(ledger, l));
            return out;
        },
        py::arg("lines"), py::arg("devices"), py::arg("accelerators") = py::list());

    m.def("make_stub_runtime", [](int accel_id) {
        RuntimeConfig c;
        c.accel_id = accel_id;
        PresetResult pr;
        pr.runtime = StorageRuntime::create_stub(c);
        pr.runtime_id = probe_runtime_id(*pr.runtime);
        return wrap(std::move(pr));
    });

    // ---- object store ----
    py::class_<SegmentFileObjectStore, std::shared_ptr<SegmentFileObjectStore>>(m, "ObjectStore")
        .def(py::init<>())
        .def(
            "open",
            [](SegmentFileObjectStore& s, py::dict c) {
                StoreConfig cfg;
                cfg.uri = c["uri"].cast<std::string>();
                cfg.layout.segment_bytes = c["segment_bytes"].cast<std::uint64_t>();
                cfg.layout.segment_count = c["segment_count"].cast<std::uint32_t>();
                cfg.segment_file_slots = c["segment_file_slots"].cast<std::uint64_t>();
                cfg.segment_header_bytes = c["segment_header_bytes"].cast<std::uint64_t>();
                if (c.contains("capacity_slots")) cfg.capacity_slots = c["capacity_slots"].cast<std::uint64_t>();
                if (c.contains("capacity_bytes")) cfg.capacity_bytes = c["capacity_bytes"].cast<std::uint64_t>();
                if (c.contains("fingerprint")) {
                    std::string f = c["fingerprint"].cast<std::string>();
                    cfg.namespace_fingerprint.assign(f.begin(), f.end());
                }
                if (c.contains("mounts"))
                    for (auto& mp : c["mounts"].cast<std::vector<std::string>>()) {
                        StoreDevice d;
                        d.mount_path = mp;
                        cfg.devices.push_back(d);
                    }
                if (c.contains("rank_id")) cfg.rank_id = c["rank_id"].cast<std::uint32_t>();
                if (c.contains("rank_count")) cfg.rank_count = c["rank_count"].cast<std::uint32_t>();
                if (c.contains("read_only")) cfg.read_only = c["read_only"].cast<bool>();
                if (c.contains("materialize")) cfg.materialize = c["materialize"].cast<std::string>();
                if (c.contains("recover_full_scan")) cfg.recover_full_scan = c["recover_full_scan"].cast<bool>();
                if (c.contains("adopt_namespace_meta"))
                    cfg.adopt_namespace_meta = c["adopt_namespace_meta"].cast<bool>();
                Status st;
                {
                    py::gil_scoped_release nogil;
                    st = s.open(cfg);
                }
                check(st);
            })
        .def("close", [](SegmentFileObjectStore& s) { check(s.close()); })
        .def("reserve",
             [](SegmentFileObjectStore& s, const std::vector<py::bytes>& keys) {
                 std::vector<ObjectKey> ks(keys.size());
                 for (std::size_t i = 0; i < keys.size(); ++i) {
                     std::string b = keys[i];
                     ks[i].bytes.assign(b.begin(), b.end());
                 }
                 auto o = unwrap(s.reserve(ks.data(), ks.size()));
                 py::list acc;
                 for (std::size_t i = 0; i < o.accepted.size(); ++i) {
                     const auto& p = o.accepted[i];
                     std::string k(o.accepted_keys[i].bytes.begin(), o.accepted_keys[i].bytes.end());
                     acc.append(py::make_tuple(py::bytes(k), p.uri, p.offset, p.slot, p.generation));
                 }
                 return py::make_tuple(acc, o.rejected_count);
             })
        .def("commit",
             [](SegmentFileObjectStore& s, const std::vector<py::bytes>& keys) {
                 std::vector<ObjectKey> ks(keys.size());
                 for (std::size_t i = 0; i < keys.size(); ++i) {
                     std::string b = keys[i];
                     ks[i].bytes.assign(b.begin(), b.end());
                 }
                 Status st;
                 {
                     py::gil_scoped_release nogil;
                     st = s.commit(ks.data(), ks.size());
                 }
                 check(st);
             })
        .def("abort",
             [](SegmentFileObjectStore& s, const std::vector<py::bytes>& keys) {
                 std::vector<ObjectKey> ks(keys.size());
                 for (std::size_t i = 0; i < keys.size(); ++i) {
                     std::string b = keys[i];
                     ks[i].bytes.assign(b.begin(), b.end());
                 }
                 check(s.abort(ks.data(), ks.size()));
             })
        .def("release",
             [](SegmentFileObjectStore& s, const std::vector<py::bytes>& keys) {
                 std::vector<ObjectKey> ks(keys.size());
                 for (std::size_t i = 0; i < keys.size(); ++i) {
                     std::string b = keys[i];
                     ks[i].bytes.assign(b.begin(), b.end());
                 }
                 return unwrap(s.release(ks.data(), ks.size()));
             })
        .def("pin",
             [](SegmentFileObjectStore& s, const std::vector<py::bytes>& keys) {
                 std::vector<ObjectKey> ks(keys.size());
                 for (std::size_t i = 0; i < keys.size(); ++i) {
                     std::string b = keys[i];
                     ks[i].bytes.assign(b.begin(), b.end());
                 }
                 check(s.pin(ks.data(), ks.size()));
             })
        .def("unpin",
             [](SegmentFileObjectStore& s, const std::vector<py::bytes>& keys) {
                 std::vector<ObjectKey> ks(keys.size());
                 for (std::size_t i = 0; i < keys.size(); ++i) {
                     std::string b = keys[i];
                     ks[i].bytes.assign(b.begin(), b.end());
                 }
                 check(s.unpin(ks.data(), ks.size()));
             })
        .def("contains",
             [](SegmentFileObjectStore& s, py::bytes key) {
                 std::string b = key;
                 ObjectKey k;
                 k.bytes.assign(b.begin(), b.end());
                 return s.contains(k);
             })
        .def("contains_prefix",
             [](SegmentFileObjectStore& s, const std::vector<py::bytes>& keys, bool all_ranks) {
                 std::vector<ObjectKey> ks(keys.size());
                 for (std::size_t i = 0; i < keys.size(); ++i) {
                     std::string b = keys[i];
                     ks[i].bytes.assign(b.begin(), b.end());
                 }
                 return all_ranks ? s.contains_prefix_all_ranks(ks.data(), ks.size())
                                  : s.contains_prefix(ks.data(), ks.size());
             },
             py::arg("keys"), py::arg("all_ranks") = false)
        .def("lookup",
             [](SegmentFileObjectStore& s, py::bytes key) -> py::object {
                 std::string b = key;
                 ObjectKey k;
                 k.bytes.assign(b.begin(), b.end());
                 auto r = s.lookup(k);
                 if (!r.ok()) return py::none();
                 auto& p = r.value();
                 return py::make_tuple(p.uri, p.offset, p.slot, p.generation);
             })
        .def("recover",
             [](SegmentFileObjectStore& s) {
                 Result<std::vector<ObjectKey>> rr = Result<std::vector<ObjectKey>>::Failure({StatusCode::INTERNAL, "unset"});
                 {
                     py::gil_scoped_release nogil;
                     rr = s.recover();
                 }
                 std::vector<ObjectKey> keys = unwrap(std::move(rr));
                 py::list out;
                 for (auto& k : keys) out.append(py::bytes(std::string(k.bytes.begin(), k.bytes.end())));
                 return out;
             })
        .def("checkpoint", [](SegmentFileObjectStore& s) { check(s.checkpoint()); })
        .def("precreate_step",
             [](SegmentFileObjectStore& s, std::uint64_t headroom) {
                 Result<std::uint64_t> r = Result<std::uint64_t>::Failure({StatusCode::INTERNAL, "unset"});
                 {
                     py::gil_scoped_release nogil;
                     r = s.precreate_step(headroom);
                 }
                 return unwrap(std::move(r));
             })
        .def("usage",
             [](SegmentFileObjectStore& s) {
                 auto u = s.usage();
                 py::dict d;
                 d["capacity_bytes"] = u.capacity_bytes;
                 d["committed_bytes"] = u.committed_bytes;
                 d["reserved_bytes"] = u.reserved_bytes;
                 d["usable_bytes"] = u.usable_bytes;
                 d["per_device_bytes"] = u.per_device_bytes;
                 return d;
             })
        .def_property_readonly("ready_slots", &SegmentFileObjectStore::ready_slots)
        .def_property_readonly("precreated_slots", &SegmentFileObjectStore::precreated_slots)
        .def_property_readonly("precreate_target", &SegmentFileObjectStore::precreate_target)
        .def_property_readonly("total_slots", &SegmentFileObjectStore::total_slots)
        .def_property_readonly("slot_bytes", &SegmentFileObjectStore::slot_bytes)
        .def_property_readonly("file_bytes", &SegmentFileObjectStore::file_bytes)
        .def("slot_uri", &SegmentFileObjectStore::slot_uri)
        .def("slot_path", &SegmentFileObjectStore::slot_path)
        .def("slot_generation", &SegmentFileObjectStore::slot_generation)
        .def("header_offset_for_slot", &SegmentFileObjectStore::header_offset_for_slot)
        .def("payload_offset_for_slot", &SegmentFileObjectStore::payload_offset_for_slot);

    // ---- digests and resolver helpers ----
    m.def("crc32c", [](py::bytes b) {
        std::string s = b;
        return crc32c(s.data(), s.size());
    });
    m.def("object_identity", [](py::bytes b) {
        std::string s = b;
        return object_identity(s.data(), s.size());
    });
    m.def("fiemap", [](const std::string& path) {
        int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
        if (fd < 0) throw py::key_error("cannot open " + path);
        struct stat st {};
        fstat(fd, &st);
        auto r = fiemap_extents(fd, static_cast<std::uint64_t>(st.st_size), true);
        ::close(fd);
        if (!r.ok()) raise(r.status());
        py::list out;
        for (auto& e : r.value()) out.append(py::make_tuple(e.logical, e.physical, e.length, e.flags));
        return out;
    });
    m.def("resolve_file",
          [](const std::string& path, const std::string& mapping, int device_index, std::uint32_t block_bytes) {
              MountBinding b;
              b.mount_path = "/";
              b.device_index = device_index;
              b.mapping = mapping;
              b.block_bytes = block_bytes;
              b.controller = "probe";
              LocalFileResolver r(b);
              auto p = unwrap(r.build_payload(path));
              py::dict d;
              d["size"] = p->file_size;
              d["mapping"] = p->mapping;
              py::list ex;
              for (auto& e : p->extents) ex.append(py::make_tuple(e.logical, e.physical, e.length, e.device));
              d["extents"] = ex;
              return d;
          },
          py::arg("path"), py::arg("mapping") = "auto", py::arg("device_index") = 0, py::arg("block_bytes") = 512);
    m.def("find_md_array", [](const std::string& sysfs_root, const std::string& path) {
        return unwrap(find_md_array(sysfs_root, path));
    });
    m.def("probe_md_raid0", [](const std::string& sysfs_root, const std::string& md) {
        auto g = unwrap(probe_md_raid0(sysfs_root, md));
        py::dict d;
        d["chunk_bytes"] = g.chunk_bytes;
        py::list mem;
        for (auto& x : g.members) mem.append(py::make_tuple(x.device_index, x.data_offset_bytes, x.name));
        d["members"] = mem;
        return d;
    });
    m.def("raid0_map", [](std::uint64_t chunk_bytes, const std::vector<std::uint64_t>& data_offsets, std::uint64_t off) {
        Raid0Geometry g;
        g.chunk_bytes = chunk_bytes;
        for (std::size_t i = 0; i < data_offsets.size(); ++i)
            g.members.push_back({static_cast<std::uint32_t>(i), data_offsets[i], ""});
        auto l = raid0_map(g, off);
        return py::make_tuple(l.member, l.offset, l.contiguous);
    });
    m.attr("cuda_device_present") = py::cpp_function([] { return cuda_device_present(); });
}
