// C++ contract tests of the native runtime (no GPU, no NVMe).
// Suites: StorageRuntime against the mock DataPath kit (partial commit,
// lifecycle, budgets, failure attribution), stub runtime, object store
// format and recovery, config spec validation, and the emulated NVMe
// controller's queue protocol driven by a host submitter.
// Parity: reference tests/storage_runtime/contract/storage_runtime_contract_test.cpp,
// tests/storage_objects/*, tests/config/{parser,spec}.
//
//   tutti_native_tests [--filter substring]

#include <fcntl.h>
#include <unistd.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <string>
#include <vector>

#include <tutti/storage_runtime.h>

#include "../config/runtime_spec.h"
#include "../datapaths/upload_plan.h"
#include "../nvme/controller.h"
#include "../objects/digest.h"
#include "../objects/object_store.h"
#include "../samples/memfs/memfs.h"
#include "../testing/mock_data_path.h"
#include "harness.h"

using namespace tutti;
using namespace tutti::testing;
using namespace tutti::native_tests;


TEST(runtime_read_write_roundtrip) {
    Fixture f;
    IoRequest r[2] = {f.req(0, 4096), f.req(8192, 4096)};
    auto o = f.rt->submit(r, 2, f.ctx());
    CHECK(o.status.ok() && o.io.has_value());
    auto w = f.rt->wait(*o.io, 1000);
    CHECK(w.observation_status.ok() && w.result->state == IoState::COMPLETED);
    CHECK(w.result->detail.confirmed_bytes == 8192);
    CHECK(f.buf[100] == static_cast<char>(100 * 7));
    CHECK(f.rt->release_io(*o.io).ok());
}

TEST(runtime_partial_commit) {
    Fixture f;
    f.dp.set_reject_at_index(1);
    IoRequest r[3] = {f.req(0, 512), f.req(512, 512), f.req(1024, 512)};
    auto o = f.rt->submit(r, 3, f.ctx());
    CHECK(o.io.has_value());
    CHECK(!o.status.ok());
    CHECK(o.initial_states[0].state == IoRequestState::ACCEPTED);
    CHECK(o.initial_states[1].state == IoRequestState::REJECTED);
    CHECK(o.initial_states[2].state == IoRequestState::ACCEPTED);
    auto w = f.rt->wait(*o.io, 1000);
    CHECK(w.result->detail.confirmed_bytes == 1024);
}

TEST(runtime_enforces_the_data_path_batch_width) {
    Fixture f;
    f.dp.mutable_caps().max_batch_requests = 3;
    IoRequest r[5] = {f.req(0, 4096), f.req(4096, 4096), f.req(8192, 4096), f.req(12288, 4096), f.req(16384, 4096)};
    auto o = f.rt->submit(r, 5, f.ctx());
    CHECK(o.io.has_value());
    CHECK(o.initial_states[2].state == IoRequestState::ACCEPTED);
    CHECK(o.initial_states[3].state == IoRequestState::REJECTED &&
          o.initial_states[3].status.code() == StatusCode::RESOURCE_EXHAUSTED);
    CHECK(f.rt->wait(*o.io, 1000).result->detail.confirmed_bytes == 3 * 4096);
    CHECK(f.rt->release_io(*o.io).ok());
    f.dp.mutable_caps().max_batch_requests = 0;
    f.dp.mutable_caps().max_batch_bytes = 8192;  // by bytes: two 4 KiB requests per batch
    o = f.rt->submit(r, 3, f.ctx());
    CHECK(o.initial_states[1].state == IoRequestState::ACCEPTED && o.initial_states[2].state == IoRequestState::REJECTED);
    CHECK(f.rt->wait(*o.io, 1000).observation_status.ok());
    CHECK(f.rt->release_io(*o.io).ok());
}

TEST(runtime_all_rejected_has_no_io) {
    Fixture f;
    IoRequest r[1] = {f.req(0, 1 << 20)};  // beyond the target
    auto o = f.rt->submit(r, 1, f.ctx());
    CHECK(!o.io.has_value());
    CHECK(o.initial_states[0].status.code() == StatusCode::OUT_OF_RANGE);
    auto o2 = f.rt->submit(r, 0, f.ctx());
    CHECK(!o2.io.has_value() && o2.status.ok() && o2.initial_states.empty());
}

TEST(runtime_wait_timeout_and_release_busy) {
    Fixture f;
    f.dp.set_manual_mode(true);
    IoRequest r[1] = {f.req(0, 4096)};
    auto o = f.rt->submit(r, 1, f.ctx());
    auto w = f.rt->wait(*o.io, 10);
    CHECK(w.observation_status.code() == StatusCode::TIMEOUT && !w.result);
    CHECK(f.rt->release_io(*o.io).code() == StatusCode::BUSY);
    CHECK(f.rt->close(f.tgt).code() == StatusCode::BUSY);
    CHECK(f.rt->unregister_memory(f.mem).code() == StatusCode::BUSY);
    f.dp.complete_all();
    CHECK(f.rt->wait(*o.io, 1000).observation_status.ok());
    CHECK(f.rt->release_io(*o.io).ok());
    CHECK(f.rt->close(f.tgt).ok());
}

TEST(runtime_terminal_result_budget) {
    Fixture f(2);
    IoRequest r[1] = {f.req(0, 512)};
    auto a = f.rt->submit(r, 1, f.ctx());
    auto b = f.rt->submit(r, 1, f.ctx());
    f.rt->wait(*a.io, 1000);
    f.rt->wait(*b.io, 1000);
    auto c = f.rt->submit(r, 1, f.ctx());
    CHECK(!c.io && c.status.code() == StatusCode::RESOURCE_EXHAUSTED);
    CHECK(f.rt->release_io(*a.io).ok());
    auto d = f.rt->submit(r, 1, f.ctx());
    CHECK(d.io.has_value());
}

TEST(runtime_failure_attribution) {
    Fixture f;
    f.dp.set_fail_request(2);
    IoRequest r[4] = {f.req(0, 512), f.req(512, 512), f.req(1024, 512), f.req(1536, 512)};
    auto o = f.rt->submit(r, 4, f.ctx());
    auto res = f.rt->wait_detail(*o.io, 1000);
    CHECK(res.ok());
    CHECK(res.value().state == IoState::FAILED);
    CHECK(res.value().detail.failure_scope == IoFailureScope::REQUEST_INDICES);
    CHECK(res.value().detail.failed_request_indices.size() == 1 && res.value().detail.failed_request_indices[0] == 2);
    CHECK(res.value().detail.confirmed_bytes == 1536);
}

TEST(runtime_handles_are_runtime_scoped_and_generational) {
    Fixture f, g;
    IoRequest r[1] = {IoRequest{IoDirection::READ, g.mem, 0, f.tgt, 0, 512}};
    auto o = f.rt->submit(r, 1, f.ctx());
    CHECK(!o.io && o.initial_states[0].status.code() == StatusCode::NOT_FOUND);
    CHECK(f.rt->close(f.tgt).ok());
    CHECK(f.rt->close(f.tgt).code() == StatusCode::NOT_FOUND);  // stale generation
    auto t2 = f.rt->open("mem://a");
    CHECK(t2.ok() && t2.value() != f.tgt);
}

TEST(runtime_execution_domain_and_accel_checks) {
    Fixture f;
    IoRequest r[1] = {f.req(0, 512)};
    HostSubmitContext dev{ExecutionDomain::DEVICE_EXECUTION, -1, nullptr};
    auto o = f.rt->submit(r, 1, dev);
    CHECK(!o.io && o.initial_states[0].status.code() == StatusCode::UNSUPPORTED);
    HostSubmitContext other{ExecutionDomain::HOST_EXECUTION, 3, nullptr};
    auto o2 = f.rt->submit(r, 1, other);
    CHECK(!o2.io && o2.status.code() == StatusCode::INVALID_ARGUMENT);
}

TEST(runtime_open_batch_per_item_results) {
    Fixture f;
    auto v = f.rt->open_batch({"mem://a", "mem://missing", "nfs://x", "mem://a"});
    CHECK(v.size() == 4);
    CHECK(v[0].ok() && v[3].ok() && v[0].value() != v[3].value());
    CHECK(!v[1].ok() && v[1].status().code() == StatusCode::NOT_FOUND);
    CHECK(!v[2].ok());
}

TEST(runtime_overlapping_registration_refused) {
    Fixture f;
    MemoryView v;
    v.address = f.buf.data() + 100;
    v.size = 10;
    v.expected_kind = MemoryKind::HOST;
    CHECK(f.rt->register_memory(v).status().code() == StatusCode::INVALID_ARGUMENT);
}

TEST(runtime_shutdown_drains_and_stops) {
    Fixture f;
    IoRequest r[1] = {f.req(0, 512)};
    auto o = f.rt->submit(r, 1, f.ctx());
    CHECK(o.io.has_value());
    CHECK(f.rt->shutdown(1000).ok());
    CHECK(f.rt->state() == RuntimeState::STOPPED);
    CHECK(f.dp.shut_down);
    MemoryView v;
    v.address = f.buf.data();
    v.size = 16;
    CHECK(f.rt->register_memory(v).status().code() == StatusCode::NOT_READY);
}

TEST(runtime_shutdown_times_out_with_inflight_io) {
    Fixture f;
    f.dp.set_manual_mode(true);
    IoRequest r[1] = {f.req(0, 512)};
    auto o = f.rt->submit(r, 1, f.ctx());
    CHECK(f.rt->shutdown(20).code() == StatusCode::TIMEOUT);
    f.dp.complete_all();
    CHECK(f.rt->shutdown(1000).ok());
}

TEST(memfs_sample_plugs_into_an_unmodified_runtime) {
    // a backend written only against the SPI: resolver + payload + DataPath + budget
    auto budget = std::make_shared<samples::memfs::MemoryResource>(1 << 20);
    samples::memfs::Resolver resolver(budget);
    samples::memfs::MemfsDataPath dp;
    RuntimeConfig c;
    c.accel_id = 0;
    RuntimeComponents comps;
    comps.resolvers.push_back({"memfs", &resolver});
    comps.data_paths.push_back({"memfs", &dp, DataPathConfig{"memfs"}});
    auto rt = StorageRuntime::create(c, comps).value();
    std::vector<char> src(8192), dst(8192, 0);
    for (std::size_t i = 0; i < src.size(); ++i) src[i] = static_cast<char>(i * 13 + 1);
    MemoryView v;
    v.address = src.data();
    v.size = src.size();
    v.expected_kind = MemoryKind::HOST;
    auto ms = rt->register_memory(v).value();
    v.address = dst.data();
    auto md = rt->register_memory(v).value();
    auto t = rt->open("memfs://obj?size=64K");
    CHECK(t.ok() && budget->used() == 65536);
    const HostSubmitContext ctx{ExecutionDomain::HOST_EXECUTION, -1, nullptr};
    IoRequest w{IoDirection::WRITE, ms, 0, t.value(), 4096, 8192};
    auto o = rt->submit(&w, 1, ctx);
    CHECK(o.status.ok() && o.io.has_value());
    CHECK(rt->wait(*o.io, 1000).result->state == IoState::COMPLETED);
    CHECK(rt->release_io(*o.io).ok());
    IoRequest r[2] = {{IoDirection::READ, md, 0, t.value(), 4096, 8192},
                      {IoDirection::READ, md, 0, t.value(), 65536 - 100, 200}};  // past the end
    o = rt->submit(r, 2, ctx);
    CHECK(o.io.has_value() && o.initial_states[1].state == IoRequestState::REJECTED);
    auto res = rt->wait(*o.io, 1000);
    CHECK(res.result->state == IoState::COMPLETED && res.result->detail.confirmed_bytes == 8192);
    CHECK(std::memcmp(src.data(), dst.data(), src.size()) == 0);
    CHECK(rt->release_io(*o.io).ok());
    CHECK(!rt->open("memfs://big?size=2M").ok());  // over budget
}

TEST(upload_runs_merge_within_an_allocation_only) {
    static char arena[1024];
    char* a = arena;        // allocation A: [0, 64)
    char* b = arena + 64;   // allocation B starts right after A
    auto up = [](const char* alloc, char* dst, std::vector<char> v) { return DeviceUpload{alloc, dst, std::move(v)}; };
    std::vector<DeviceUpload> ups;
    ups.push_back(up(b, b + 400, {7, 7}));          // B, far: its own run
    ups.push_back(up(a, a + 40, {3, 3, 3, 3}));     // A, after the next one (input order does not matter)
    ups.push_back(up(a, a + 0, {1, 1, 1, 1, 1, 1, 1, 1}));
    ups.push_back(up(b, b + 0, {5, 5}));            // B at A's end: never merged with A
    ups.push_back(up(a, a + 42, {9}));              // overlaps an earlier upload: later wins
    auto runs = coalesce_uploads(ups, 255);
    CHECK(runs.size() == 3);
    CHECK(runs[0].dst == a && runs[0].bytes.size() == 44);  // [0, 44) with the gap zero-filled
    CHECK(runs[0].bytes[0] == 1 && runs[0].bytes[8] == 0 && runs[0].bytes[39] == 0 && runs[0].bytes[40] == 3);
    CHECK(runs[0].bytes[42] == 9 && runs[0].bytes[43] == 3);
    CHECK(runs[1].dst == b && runs[1].bytes.size() == 2 && runs[1].bytes[0] == 5);
    CHECK(runs[2].dst == b + 400 && runs[2].bytes.size() == 2);
    std::vector<DeviceUpload> rows;  // consecutive 32-byte rows: one run
    for (int r = 0; r < 5; ++r) rows.push_back(up(a, a + 32 * r, std::vector<char>(32, static_cast<char>(r))));
    runs = coalesce_uploads(rows, 255);
    CHECK(runs.size() == 1 && runs[0].bytes.size() == 160 && runs[0].bytes[159] == 4);
}

TEST(stub_runtime_ios_wait_for_a_forced_completion) {
    RuntimeConfig c;
    auto rt = StorageRuntime::create_stub(c);
    std::vector<char> b(64);
    MemoryView v;
    v.address = b.data();
    v.size = b.size();
    v.expected_kind = MemoryKind::HOST;
    auto h = rt->register_memory(v);
    CHECK(h.ok());
    CHECK(rt->query_memory(h.value()).value().size == 64);
    auto t = rt->open("file:///anything");  // any URI: a 1 GiB stub target
    CHECK(t.ok());
    IoRequest reqs[3];
    for (auto& r : reqs) {
        r.direction = IoDirection::READ;
        r.memory = h.value();
        r.memory_offset = 0;
        r.target = t.value();
        r.target_offset = 4096;
        r.length = 64;
    }
    reqs[1].length = 65;  // past the registration: rejected, the others accepted
    HostSubmitContext ctx;
    auto o = rt->submit(reqs, 3, ctx);
    CHECK(o.io.has_value());
    CHECK(o.initial_states[0].state == IoRequestState::ACCEPTED);
    CHECK(o.initial_states[1].state == IoRequestState::REJECTED);
    CHECK(o.initial_states[1].status.code() == StatusCode::OUT_OF_RANGE);
    CHECK(rt->query(*o.io).value().state == IoState::IN_FLIGHT);
    CHECK(rt->wait(*o.io, 5).observation_status.code() == StatusCode::TIMEOUT);
    CHECK(rt->release_io(*o.io).code() == StatusCode::BUSY);
    CHECK(rt->unregister_memory(h.value()).code() != StatusCode::OK);  // in use
    CHECK(rt->testing_force_complete(*o.io, IoState::IN_FLIGHT).code() == StatusCode::INVALID_ARGUMENT);
    CHECK(rt->testing_force_complete(*o.io, IoState::FAILED, Status(StatusCode::DEVICE_ERROR, "media")).ok());
    CHECK(rt->testing_force_complete(*o.io, IoState::COMPLETED).code() == StatusCode::INVALID_ARGUMENT);
    auto w = rt->wait(*o.io, 0);
    CHECK(w.observation_status.ok() && w.result->state == IoState::FAILED);
    CHECK(w.result->status.code() == StatusCode::DEVICE_ERROR);
    CHECK((w.result->detail.failed_request_indices == std::vector<std::uint32_t>{0, 2}));
    CHECK(rt->unreleased_terminal_results() == 1);
    CHECK(rt->release_io(*o.io).ok());
    CHECK(rt->testing_force_complete(*o.io, IoState::COMPLETED).code() == StatusCode::NOT_FOUND);
    auto o2 = rt->submit(reqs, 1, ctx);
    CHECK(rt->testing_force_complete(*o2.io, IoState::COMPLETED).ok());
    CHECK(rt->wait(*o2.io, 0).result->state == IoState::COMPLETED);
    CHECK(rt->release_io(*o2.io).ok());
    CHECK(rt->unregister_memory(h.value()).ok());
}

TEST(digest_check_values) {
    CHECK(crc32c("123456789", 9) == 0xE3069283u);
    CHECK(object_identity(nullptr, 0) == object_identity("", 0));
    CHECK(object_identity("a", 1) != object_identity("b", 1));
}

TEST(object_store_commit_recover) {
    char tmpl[] = "/tmp/tutti_native_XXXXXX";
    const char* dir = mkdtemp(tmpl);
    CHECK(dir != nullptr);
    StoreConfig c;
    c.uri = dir;
    c.layout.segment_bytes = 8192;
    c.layout.segment_count = 2;
    c.segment_file_slots = 4;
    c.segment_header_bytes = 4096;
    c.capacity_slots = 8;
    {
        SegmentFileObjectStore s;
        CHECK(s.open(c).ok());
        ObjectKey k{{1, 2, 3}};
        CHECK(s.reserve(&k, 1).ok());
        CHECK(s.commit(&k, 1).ok());
        CHECK(s.contains(k));
        CHECK(s.close().ok());
    }
    {
        SegmentFileObjectStore s;
        CHECK(s.open(c).ok());
        auto keys = s.recover();
        CHECK(keys.ok() && keys.value().size() == 1 && keys.value()[0].bytes == std::vector<std::uint8_t>({1, 2, 3}));
        CHECK(s.close().ok());
    }
    c.namespace_fingerprint = {9};
    SegmentFileObjectStore s3;
    CHECK(s3.open(c).code() == StatusCode::INVALID_ARGUMENT);
    std::string cmd = std::string("rm -rf ") + dir;
    CHECK(std::system(cmd.c_str()) == 0);
}

TEST(config_spec_contract_matrix) {
    const char* ok = R"(
storage:
  resources:
    - {id: r, type: nvme, provider: {type: emulated}, config: {mounts: [/a]}}
  resolvers:
    - {id: f, type: local-file, config: {topology: single}}
  datapaths:
    - {id: d, type: local-nvme}
  backends:
    - {id: b, contract: ext4-local-nvme, resolver: f, datapath: d, resource: r}
)";
    auto s = parse_runtime_config_text(ok);
    CHECK(s.ok());
    CHECK(validate_runtime_spec(s.value()).ok());
    std::string two = ok;
    two.replace(two.find("[/a]"), 4, "[/a, /b]");
    auto s2 = parse_runtime_config_text(two);
    CHECK(s2.ok() && !validate_runtime_spec(s2.value()).ok());
    auto s3 = parse_runtime_config_text(std::string(ok) + "  extra: 1\n");
    CHECK(!s3.ok());
}


// ---- emulated NVMe controller, host submitter ----
namespace {
void controller_roundtrip(bool direct_io, bool map_reads = false, bool memory_media = false,
                          std::uint64_t image_budget = 0) {
    char path[] = "/tmp/tutti_emu_XXXXXX";
    const int fd = mkstemp(path);
    CHECK(fd >= 0);
    const std::size_t fbytes = 4u << 20;
    std::vector<unsigned char> pattern(fbytes);
    for (std::size_t i = 0; i < fbytes; ++i) pattern[i] = static_cast<unsigned char>((i * 131u + 7u) >> 3);
    CHECK(::pwrite(fd, pattern.data(), fbytes, 0) == static_cast<ssize_t>(fbytes));
    ::fsync(fd);
    ::close(fd);
    nvme::EmulatedControllerConfig cfg;
    cfg.num_io_queues = 2;
    cfg.queue_depth = 16;
    cfg.worker_threads = 1;
    cfg.direct_io = direct_io;
    cfg.map_reads = map_reads;
    if (memory_media) {
        cfg.media = nvme::EmulatedControllerConfig::Media::MEMORY;
        cfg.image_chunk_bytes = 1u << 20;  // the 4 MiB file is four image chunks
        cfg.image_budget_bytes = image_budget;
    }
    auto ctl = nvme::EmulatedNvmeController::create(cfg);
    CHECK(ctl.ok());
    auto& c = *ctl.value();
    // namespace [1 MiB, 5 MiB) is the file
    CHECK(c.attach_file(path, {{1u << 20, fbytes, 0}}).ok());
    void* buf = nullptr;
    void* lst = nullptr;
    CHECK(posix_memalign(&buf, 4096, 256 << 10) == 0 && posix_memalign(&lst, 4096, 4096) == 0);
    auto iova = c.map_window(buf, 256 << 10, false);
    auto liova = c.map_window(lst, 4096, false);
    CHECK(iova.ok() && liova.ok());
    HostSubmitter hs{c.host_queue(0)};
    // 8 KiB read: PRP1 + PRP2 page
    nvme::Sqe e{};
    const std::uint64_t lba = 512;
    nvme::build_rw_sqe(e, nvme::kOpRead, 1, 1, ((1u << 20) + 8192) / lba, 8192 / lba, iova.value(),
                       iova.value() + 4096);
    CHECK(hs.run(e) == 0);
    CHECK(std::memcmp(buf, pattern.data() + 8192, 8192) == 0);
    // 40 more single-page reads: the 16-entry CQ wraps and its phase bit flips (2.5 laps)
    for (std::uint32_t k = 0; k < 40; ++k) {
        const std::uint64_t off = (k * 7u % 64u) * 4096u;
        nvme::build_rw_sqe(e, nvme::kOpRead, 1, 1, ((1u << 20) + off) / lba, 4096 / lba, iova.value(), 0);
        CHECK(hs.run(e) == 0);
        CHECK(std::memcmp(buf, pattern.data() + off, 4096) == 0);
    }
    // 64 KiB read through a PRP list (pages in reverse order)
    auto* l = static_cast<std::uint64_t*>(lst);
    for (int k = 0; k < 15; ++k) l[k] = iova.value() + (15 - k) * 4096ull;
    nvme::build_rw_sqe(e, nvme::kOpRead, 2, 1, ((1u << 20) + 65536) / lba, 65536 / lba, iova.value(), liova.value());
    CHECK(hs.run(e) == 0);
    auto* b = static_cast<unsigned char*>(buf);
    CHECK(std::memcmp(b, pattern.data() + 65536, 4096) == 0);
    for (int k = 0; k < 15; ++k) CHECK(std::memcmp(b + (15 - k) * 4096, pattern.data() + 65536 + (k + 1) * 4096, 4096) == 0);
    // write 4 KiB, then read it back through the controller
    std::memset(buf, 0xA5, 4096);
    nvme::build_rw_sqe(e, nvme::kOpWrite, 3, 1, ((1u << 20) + 12288) / lba, 8, iova.value(), 0);
    CHECK(hs.run(e) == 0);
    std::memset(buf, 0, 8192);
    nvme::build_rw_sqe(e, nvme::kOpRead, 4, 1, ((1u << 20) + 12288) / lba, 8, iova.value(), 0);
    CHECK(hs.run(e) == 0);
    CHECK(b[0] == 0xA5 && b[4095] == 0xA5);
    {  // a WRITE's CQE means the bytes are in the backing file (memory media write through)
        unsigned char back[4096];
        const int rfd = ::open(path, O_RDONLY);
        CHECK(rfd >= 0 && ::pread(rfd, back, 4096, 12288) == 4096);
        ::close(rfd);
        CHECK(back[0] == 0xA5 && back[4095] == 0xA5);
    }
    if (memory_media) {
        const auto st = c.stats();
        CHECK(image_budget == 0 ? st.image_bytes >= (1u << 20) : st.image_bytes <= image_budget);
    }
    // outside the backed namespace range, an unmapped buffer, an injected media error
    nvme::build_rw_sqe(e, nvme::kOpRead, 5, 1, 0, 8, iova.value(), 0);
    CHECK(hs.run(e) == nvme::make_status(0, nvme::kScLbaOutOfRange));
    nvme::build_rw_sqe(e, nvme::kOpRead, 6, 1, (1u << 20) / lba, 8, 0x1000, 0);
    CHECK(hs.run(e) == nvme::make_status(0, nvme::kScDataTransferError));
    c.inject(nvme::InjectKind::MEDIA_ERROR, 1);
    nvme::build_rw_sqe(e, nvme::kOpRead, 7, 1, (1u << 20) / lba, 8, iova.value(), 0);
    CHECK(hs.run(e) == nvme::make_status(nvme::kSctMedia, nvme::kScUnrecoveredRead));
    nvme::build_rw_sqe(e, nvme::kOpRead, 8, 1, (1u << 20) / lba, 8, iova.value(), 0);
    CHECK(hs.run(e) == 0);
    // an injected error can carry any CQE status (here: type 2, code 0x85)
    c.inject(nvme::InjectKind::MEDIA_ERROR, 1, 0, nvme::make_status(2, 0x85));
    nvme::build_rw_sqe(e, nvme::kOpRead, 9, 1, (1u << 20) / lba, 8, iova.value(), 0);
    CHECK(hs.run(e) == nvme::make_status(2, 0x85));
    nvme::build_rw_sqe(e, nvme::kOpRead, 10, 1, (1u << 20) / lba, 8, iova.value(), 0);
    CHECK(hs.run(e) == 0);
    c.stop();
    free(buf);
    free(lst);
    ::unlink(path);
}
}  // namespace

TEST(emulated_controller_page_cached_reads_writes_and_errors) { controller_roundtrip(false); }
TEST(emulated_controller_mapped_reads_writes_and_errors) { controller_roundtrip(false, true); }
TEST(emulated_controller_direct_io_reads_writes_and_errors) { controller_roundtrip(true); }
TEST(emulated_controller_memory_media_reads_writes_and_errors) { controller_roundtrip(false, false, true); }
TEST(emulated_controller_memory_media_over_budget_serves_from_files) {
    controller_roundtrip(false, false, true, 1u << 20);  // one chunk fits; the rest is read from the file
}

int main(int argc, char** argv) {
    const char* filter = nullptr;
    for (int i = 1; i + 1 < argc; ++i)
        if (std::string(argv[i]) == "--filter") filter = argv[i + 1];
    int run = 0;
    for (auto& t : registry()) {
        if (filter && !std::strstr(t.name, filter)) continue;
        const int before = g_failures;
        t.fn();
        ++run;
        std::printf("%s %s\n", g_failures == before ? "PASS" : "FAIL", t.name);
    }
    std::printf("%d test(s), %d failure(s)\n", run, g_failures);
    return g_failures ? 1 : 0;
}
