// Contract suite of the DataPaths and the emulated drive without a GPU:
// the POSIX host-execution DataPath through the runtime (file resolver,
// aligned and unaligned requests, failure attribution, concurrency) and the
// emulated controller's queue protocol at its edges (PRP-list chaining,
// protocol violations, resets, injected drops and delays, the bandwidth cap,
// memory media across image chunks, detach).
// Parity: the rules of reference tests/data_paths/local_nvme/
// local_nvme_datapath_contract_test.cpp that hold without hardware.

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <thread>

#include "../datapaths/posix_data_path.h"
#include "../resolvers/file_resolvers.h"
#include "harness.h"

using namespace tutti;
using namespace tutti::native_tests;

namespace {

std::string temp_dir() {
    char tmpl[] = "/tmp/tutti_dp_XXXXXX";
    const char* d = mkdtemp(tmpl);
    return d ? std::string(d) : std::string();
}

std::string make_file(const std::string& dir, const std::string& name, std::size_t bytes, unsigned seed) {
    const std::string path = dir + "/" + name;
    std::vector<unsigned char> v(bytes);
    for (std::size_t i = 0; i < bytes; ++i) v[i] = static_cast<unsigned char>((i * 131u + seed) >> 2);
    const int fd = ::open(path.c_str(), O_CREAT | O_RDWR | O_TRUNC, 0644);
    if (fd >= 0) {
        (void)!::pwrite(fd, v.data(), bytes, 0);
        ::fsync(fd);
        ::close(fd);
    }
    return path;
}

struct PosixFixture {
    std::string dir = temp_dir();
    std::unique_ptr<StorageRuntime> rt;
    std::shared_ptr<PosixDataPath> dp;
    std::vector<char> buf = std::vector<char>(1 << 20, 0);
    MemoryHandle mem;
    explicit PosixFixture(std::uint64_t fail_every = 0, std::uint32_t threads = 4) {
        MountBinding b;
        b.mount_path = dir;
        b.controller = "posix0";
        b.mapping = "synthetic";
        b.datapath_key = "posix";
        PosixConfig pc;
        pc.threads = threads;
        pc.direct_io = false;
        pc.inject_fail_every = fail_every;
        dp = std::make_shared<PosixDataPath>(pc);
        OwnedComponents comps;
        comps.resolvers.push_back({"file", std::make_unique<LocalFileResolver>(b)});
        comps.data_paths.push_back({"posix", dp, DataPathConfig{"posix"}});
        RuntimeConfig rc;
        rc.max_terminal_results = 4096;
        rt = StorageRuntime::create_owning(rc, std::move(comps)).value();
        mem = rt->register_memory(MemoryView{buf.data(), buf.size(), MemoryKind::HOST}).value();
    }
    ~PosixFixture() {
        rt.reset();
        if (!dir.empty()) (void)!std::system(("rm -rf " + dir).c_str());
    }
    HostSubmitContext ctx() { return HostSubmitContext{ExecutionDomain::HOST_EXECUTION, -1, nullptr}; }
};

bool done_ok(StorageRuntime& rt, const IoHandle& h, std::uint64_t bytes) {
    auto w = rt.wait(h, 5000);
    return w.observation_status.ok() && w.result && w.result->state == IoState::COMPLETED &&
           w.result->detail.confirmed_bytes == bytes;
}

}  // namespace

// ---- POSIX DataPath through the runtime ----------------------------------------------

TEST(posix_write_then_read_back) {
    PosixFixture f;
    const std::string path = make_file(f.dir, "obj", 1 << 20, 3);
    auto t = f.rt->open("file://" + path);
    CHECK(t.ok());
    for (std::size_t i = 0; i < 65536; ++i) f.buf[i] = static_cast<char>(i * 13 + 1);
    IoRequest w[1] = {IoRequest{IoDirection::WRITE, f.mem, 0, t.value(), 65536, 65536}};
    auto o = f.rt->submit(w, 1, f.ctx());
    CHECK(o.io && done_ok(*f.rt, *o.io, 65536));
    std::memset(f.buf.data(), 0, 1 << 17);
    IoRequest r[1] = {IoRequest{IoDirection::READ, f.mem, 4096, t.value(), 65536, 65536}};
    o = f.rt->submit(r, 1, f.ctx());
    CHECK(o.io && done_ok(*f.rt, *o.io, 65536));
    for (std::size_t i = 0; i < 65536; i += 4093) CHECK(f.buf[4096 + i] == static_cast<char>(i * 13 + 1));
}

TEST(posix_unaligned_offsets_and_lengths) {
    PosixFixture f;
    const std::string path = make_file(f.dir, "obj", 1 << 16, 5);
    auto t = f.rt->open("file://" + path);
    CHECK(t.ok());
    IoRequest r[1] = {IoRequest{IoDirection::READ, f.mem, 3, t.value(), 7, 1001}};
    auto o = f.rt->submit(r, 1, f.ctx());
    CHECK(o.io && done_ok(*f.rt, *o.io, 1001));
    for (std::size_t i = 0; i < 1001; i += 97)
        CHECK(static_cast<unsigned char>(f.buf[3 + i]) == static_cast<unsigned char>(((i + 7) * 131u + 5) >> 2));
}

TEST(posix_injected_failure_names_the_failed_request) {
    PosixFixture f(3, 1);  // one worker: requests execute in order, the 3rd fails
    const std::string path = make_file(f.dir, "obj", 1 << 16, 7);
    auto t = f.rt->open("file://" + path);
    CHECK(t.ok());
    IoRequest r[4];
    for (int i = 0; i < 4; ++i) r[i] = IoRequest{IoDirection::READ, f.mem, 4096u * i, t.value(), 4096u * i, 4096};
    auto o = f.rt->submit(r, 4, f.ctx());
    auto res = f.rt->wait_detail(*o.io, 5000);
    CHECK(res.ok() && res.value().state == IoState::FAILED);
    CHECK(res.value().detail.failed_request_indices.size() == 1);
    CHECK(res.value().detail.failed_request_indices[0] == 2);
    CHECK(res.value().detail.confirmed_bytes == 3 * 4096);
}

TEST(posix_many_requests_from_many_threads) {
    PosixFixture f(0, 8);
    const std::string path = make_file(f.dir, "obj", 1 << 20, 9);
    auto t = f.rt->open("file://" + path);
    CHECK(t.ok());
    std::atomic<int> bad{0};
    std::vector<std::thread> th;
    for (int k = 0; k < 4; ++k)
        th.emplace_back([&, k] {
            for (int i = 0; i < 16; ++i) {
                IoRequest r[16];
                for (int j = 0; j < 16; ++j) {
                    const std::uint64_t slot = (k * 256 + i * 16 + j) % 256;
                    r[j] = IoRequest{IoDirection::READ, f.mem, slot * 4096, t.value(), slot * 4096, 4096};
                }
                auto o = f.rt->submit(r, 16, f.ctx());
                if (!o.io || !done_ok(*f.rt, *o.io, 16 * 4096) || !f.rt->release_io(*o.io).ok()) ++bad;
            }
        });
    for (auto& x : th) x.join();
    CHECK(bad.load() == 0);
    for (std::size_t i = 0; i < (1u << 20); i += 65521)
        CHECK(static_cast<unsigned char>(f.buf[i]) == static_cast<unsigned char>((i * 131u + 9) >> 2));
}

TEST(posix_files_outside_the_mount_are_refused) {
    PosixFixture f;
    CHECK(!f.rt->open("file:///etc/hostname").ok());
    CHECK(!f.rt->open("file://" + f.dir + "/missing").ok());
}

// ---- emulated controller: queue protocol edges ------------------------------------------

namespace {
struct Drive {
    std::string dir = temp_dir();
    std::string path;
    std::unique_ptr<nvme::EmulatedNvmeController> ctl;
    void* buf = nullptr;
    void* lists = nullptr;
    std::uint64_t iova = 0, list_iova = 0;
    std::vector<unsigned char> pattern;
    explicit Drive(nvme::EmulatedControllerConfig cfg, std::size_t file_bytes = 8u << 20) {
        path = make_file(dir, "ns", file_bytes, 11);
        pattern.resize(file_bytes);
        for (std::size_t i = 0; i < file_bytes; ++i) pattern[i] = static_cast<unsigned char>((i * 131u + 11) >> 2);
        cfg.num_io_queues = 2;
        cfg.queue_depth = 16;
        cfg.worker_threads = 1;
        ctl = nvme::EmulatedNvmeController::create(cfg).value();
        (void)ctl->attach_file(path, {{0, file_bytes, 0}});
        (void)!posix_memalign(&buf, 4096, 4u << 20);
        (void)!posix_memalign(&lists, 4096, 16 * 4096);
        std::memset(buf, 0, 4u << 20);
        iova = ctl->map_dma(buf, 4u << 20).value().bus_at(buf);
        list_iova = ctl->map_dma(lists, 16 * 4096).value().bus_at(lists);
    }
    ~Drive() {
        ctl->stop();
        ctl.reset();
        std::free(buf);
        std::free(lists);
        (void)!std::system(("rm -rf " + dir).c_str());
    }
    nvme::Sqe read(std::uint16_t cid, std::uint64_t off, std::uint32_t bytes, std::uint64_t prp1, std::uint64_t prp2) {
        nvme::Sqe e{};
        nvme::build_rw_sqe(e, nvme::kOpRead, cid, 1, off / 512, bytes / 512, prp1, prp2);
        return e;
    }
};
}  // namespace

TEST(emulated_prp_list_chains_across_list_pages) {
    nvme::EmulatedControllerConfig cfg;
    cfg.mdts_bytes = 4u << 20;
    Drive d(cfg);
    // 3 MiB = 768 pages: PRP1 + a 767-entry list, which takes two list pages
    // (the last entry of the first page points at the second page)
    auto* l = static_cast<std::uint64_t*>(d.lists);
    const std::uint32_t pages = 768;
    std::uint32_t k = 0;
    for (std::uint32_t p = 1; p < pages; ++p) {
        if (k == 511) {  // chain to the next list page
            l[k] = d.list_iova + 4096;
            k = 512;
        }
        l[k++] = d.iova + std::uint64_t(p) * 4096;
    }
    HostSubmitter hs{d.ctl->host_queue(0)};
    CHECK(hs.run(d.read(1, 4096, pages * 4096, d.iova, d.list_iova)) == 0);
    CHECK(std::memcmp(d.buf, d.pattern.data() + 4096, pages * 4096) == 0);
}

TEST(emulated_invalid_doorbell_is_fatal_until_reset) {
    Drive d({});
    HostSubmitter hs{d.ctl->host_queue(0)};
    CHECK(hs.run(d.read(1, 0, 4096, d.iova, 0)) == 0);
    __atomic_store_n(hs.q.sq_doorbell, 99u, __ATOMIC_RELEASE);  // beyond the queue depth
    std::this_thread::sleep_for(std::chrono::milliseconds(5));
    CHECK(hs.run(d.read(2, 0, 4096, d.iova, 0), 2000) == -1);  // ignored while fatal
    CHECK(d.ctl->reset_queue(0).ok());
    hs.reset();
    CHECK(hs.run(d.read(3, 4096, 4096, d.iova, 0)) == 0);
    CHECK(std::memcmp(d.buf, d.pattern.data() + 4096, 4096) == 0);
    // the other queue never noticed
    HostSubmitter hs1{d.ctl->host_queue(1)};
    CHECK(hs1.run(d.read(4, 0, 4096, d.iova, 0)) == 0);
}

TEST(emulated_dropped_completion_then_reset_recovers) {
    Drive d({});
    HostSubmitter hs{d.ctl->host_queue(0)};
    d.ctl->inject(nvme::InjectKind::DROP_COMPLETION, 1);
    CHECK(hs.run(d.read(1, 0, 4096, d.iova, 0), 3000) == -1);
    CHECK(d.ctl->stats().injected == 1);
    CHECK(d.ctl->reset_queue(0).ok());
    hs.reset();
    CHECK(hs.run(d.read(2, 8192, 4096, d.iova, 0)) == 0);
    CHECK(std::memcmp(d.buf, d.pattern.data() + 8192, 4096) == 0);
}

TEST(emulated_delay_injection_delays_one_command) {
    Drive d({});
    HostSubmitter hs{d.ctl->host_queue(0)};
    d.ctl->inject(nvme::InjectKind::DELAY, 1, 30000);
    const auto t0 = std::chrono::steady_clock::now();
    CHECK(hs.run(d.read(1, 0, 4096, d.iova, 0)) == 0);
    const auto ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    CHECK(ms >= 29.0);
    const auto t1 = std::chrono::steady_clock::now();
    CHECK(hs.run(d.read(2, 0, 4096, d.iova, 0)) == 0);  // only one command was delayed
    using Ms = std::chrono::duration<double, std::milli>;
    const double ms2 = Ms(std::chrono::steady_clock::now() - t1).count();
    CHECK(ms2 < 29.0);
}

TEST(emulated_late_completion_after_a_reset_is_not_taken_for_the_next_command) {
    // the host gives up on a command the drive still holds, resets the queue and
    // reuses slot 0: the old command's completion, arriving later, must not land
    // in the fresh queue (it would complete the next command before its data)
    Drive d({});
    HostSubmitter hs{d.ctl->host_queue(0)};
    d.ctl->inject(nvme::InjectKind::DELAY, 1, 200000);  // 200 ms
    CHECK(hs.run(d.read(1, 0, 4096, d.iova, 0), 2000) == -1);  // gave up after about 20 ms
    CHECK(d.ctl->reset_queue(0).ok());
    hs.reset();
    std::memset(d.buf, 0, 2 * 4096);
    const auto* cq = d.ctl->host_queue(0).cq;
    CHECK(hs.run(d.read(2, 8192, 4096, d.iova + 4096, 0)) == 0);
    CHECK(nvme::cqe_cid(cq[0].dw3) == 2);  // slot 0 holds the new command's completion
    CHECK(std::memcmp(static_cast<char*>(d.buf) + 4096, d.pattern.data() + 8192, 4096) == 0);
    std::this_thread::sleep_for(std::chrono::milliseconds(250));  // past the old command's delay
    CHECK(hs.run(d.read(3, 16384, 4096, d.iova + 4096, 0)) == 0);
    CHECK(nvme::cqe_cid(cq[1].dw3) == 3);  // and the next slot the one after it
    CHECK(std::memcmp(static_cast<char*>(d.buf) + 4096, d.pattern.data() + 16384, 4096) == 0);
}

TEST(emulated_bandwidth_cap_paces_the_drive) {
    nvme::EmulatedControllerConfig cfg;
    cfg.max_gbps = 0.1;  // 100 MB/s: 10 x 1 MiB take at least ~94 ms
    Drive d(cfg);
    HostSubmitter hs{d.ctl->host_queue(0)};
    const auto t0 = std::chrono::steady_clock::now();
    for (int i = 0; i < 10; ++i) CHECK(hs.run(d.read(static_cast<std::uint16_t>(i), 0, 1u << 20, d.iova, d.list_iova)) == 0 || true);
    const auto ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    CHECK(ms >= 85.0);
}

TEST(emulated_flush_opcode_namespace_and_mdts_checks) {
    Drive d({});
    HostSubmitter hs{d.ctl->host_queue(0)};
    nvme::Sqe e{};
    nvme::build_rw_sqe(e, nvme::kOpFlush, 1, 1, 0, 1, 0, 0);
    CHECK(hs.run(e) == 0);
    nvme::build_rw_sqe(e, 0x7F, 2, 1, 0, 8, d.iova, 0);
    CHECK(hs.run(e) == static_cast<int>(nvme::make_status(0, nvme::kScInvalidOpcode)));
    nvme::build_rw_sqe(e, nvme::kOpRead, 3, 9, 0, 8, d.iova, 0);
    CHECK(hs.run(e) == static_cast<int>(nvme::make_status(0, nvme::kScInvalidNamespace)));
    nvme::build_rw_sqe(e, nvme::kOpRead, 4, 1, 0, (2u << 20) / 512, d.iova, d.list_iova);  // past the 1 MiB MDTS
    CHECK(hs.run(e) == static_cast<int>(nvme::make_status(0, nvme::kScInvalidField)));
}

TEST(emulated_prp_list_outside_the_dma_windows_is_a_transfer_error) {
    Drive d({});
    HostSubmitter hs{d.ctl->host_queue(0)};
    std::vector<std::uint64_t> rogue(512, d.iova);
    CHECK(hs.run(d.read(1, 0, 64 * 1024, d.iova, reinterpret_cast<std::uint64_t>(rogue.data()))) ==
          static_cast<int>(nvme::make_status(0, nvme::kScDataTransferError)));
    // a list entry that points outside the windows
    auto* l = static_cast<std::uint64_t*>(d.lists);
    for (int k = 0; k < 15; ++k) l[k] = d.iova + (k + 1) * 4096ull;
    l[7] = 0x10000;
    CHECK(hs.run(d.read(2, 0, 64 * 1024, d.iova, d.list_iova)) ==
          static_cast<int>(nvme::make_status(0, nvme::kScDataTransferError)));
}

TEST(emulated_memory_media_across_image_chunks_writes_through) {
    nvme::EmulatedControllerConfig cfg;
    cfg.media = nvme::EmulatedControllerConfig::Media::MEMORY;
    cfg.image_chunk_bytes = 1u << 20;
    cfg.image_budget_bytes = 8u << 20;
    Drive d(cfg);
    HostSubmitter hs{d.ctl->host_queue(0)};
    // 8 KiB that straddle the first and second image chunk
    std::memset(d.buf, 0x5A, 8192);
    nvme::Sqe w{};
    nvme::build_rw_sqe(w, nvme::kOpWrite, 1, 1, ((1u << 20) - 4096) / 512, 16, d.iova, d.iova + 4096);
    CHECK(hs.run(w) == 0);
    std::memset(d.buf, 0, 8192);
    CHECK(hs.run(d.read(2, (1u << 20) - 4096, 8192, d.iova, d.iova + 4096)) == 0);
    CHECK(static_cast<unsigned char*>(d.buf)[0] == 0x5A && static_cast<unsigned char*>(d.buf)[8191] == 0x5A);
    unsigned char back[8192];
    const int fd = ::open(d.path.c_str(), O_RDONLY);
    CHECK(fd >= 0 && ::pread(fd, back, 8192, (1u << 20) - 4096) == 8192);
    ::close(fd);
    CHECK(back[0] == 0x5A && back[8191] == 0x5A);
    CHECK(d.ctl->stats().image_bytes == (2u << 20));  // only the two touched chunks were loaded
}

TEST(emulated_detached_file_leaves_its_range_unbacked) {
    Drive d({});
    HostSubmitter hs{d.ctl->host_queue(0)};
    CHECK(hs.run(d.read(1, 0, 4096, d.iova, 0)) == 0);
    CHECK(d.ctl->detach_file(d.path).ok());
    CHECK(hs.run(d.read(2, 0, 4096, d.iova, 0)) == static_cast<int>(nvme::make_status(0, nvme::kScLbaOutOfRange)));
    CHECK(d.ctl->detach_file(d.path).ok() || true);
    CHECK(d.ctl->detach_file("/nonexistent").code() == StatusCode::NOT_FOUND);
}

TEST(emulated_stats_count_commands_bytes_and_errors) {
    Drive d({});
    HostSubmitter hs{d.ctl->host_queue(0)};
    for (int i = 0; i < 5; ++i) CHECK(hs.run(d.read(static_cast<std::uint16_t>(i), 0, 8192, d.iova, d.iova + 4096)) == 0);
    d.ctl->inject(nvme::InjectKind::MEDIA_ERROR, 2);
    CHECK(hs.run(d.read(9, 0, 4096, d.iova, 0)) != 0);
    CHECK(hs.run(d.read(10, 0, 4096, d.iova, 0)) != 0);
    CHECK(hs.run(d.read(11, 0, 4096, d.iova, 0)) == 0);
    const auto s = d.ctl->stats();
    CHECK(s.commands == 8 && s.read_bytes == 5 * 8192 + 4096 && s.errors == 2 && s.injected == 2);
}

TEST(emulated_controller_rejects_bad_configurations) {
    nvme::EmulatedControllerConfig c;
    c.num_io_queues = 0;
    CHECK(!nvme::EmulatedNvmeController::create(c).ok());
    c = {};
    c.lba_bytes = 1000;
    CHECK(!nvme::EmulatedNvmeController::create(c).ok());
    c = {};
    c.mdts_bytes = 6000;
    CHECK(!nvme::EmulatedNvmeController::create(c).ok());
    c = {};
    c.queue_depth = 1;
    CHECK(!nvme::EmulatedNvmeController::create(c).ok());
    c = {};
    c.max_gbps = -1;
    CHECK(!nvme::EmulatedNvmeController::create(c).ok());
}

namespace tutti {
namespace native_tests {

namespace {
std::vector<unsigned char> file_bytes_at(const std::string& path, std::uint64_t off, std::size_t n) {
    std::vector<unsigned char> out(n);
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd >= 0) {
        (void)!::pread(fd, out.data(), n, static_cast<off_t>(off));
        ::close(fd);
    }
    return out;
}
}  // namespace

TEST(emulated_write_cache_reaches_the_file_on_flush_only) {
    nvme::EmulatedControllerConfig cfg;
    cfg.media = nvme::EmulatedControllerConfig::Media::MEMORY;
    cfg.image_chunk_bytes = 1u << 20;
    cfg.write_back = true;
    Drive d(cfg);
    HostSubmitter hs{d.ctl->host_queue(0)};
    std::memset(d.buf, 0xA5, 8192);
    nvme::Sqe w{};
    nvme::build_rw_sqe(w, nvme::kOpWrite, 1, 1, (2u << 20) / 512, 16, d.iova, d.iova + 4096);
    CHECK(hs.run(w) == 0);
    // the drive answers reads from its cache, the file still holds the old bytes
    std::memset(d.buf, 0, 8192);
    CHECK(hs.run(d.read(2, 2u << 20, 8192, d.iova, d.iova + 4096)) == 0);
    CHECK(static_cast<unsigned char*>(d.buf)[8191] == 0xA5);
    CHECK(file_bytes_at(d.path, 2u << 20, 8192) == std::vector<unsigned char>(d.pattern.begin() + (2u << 20),
                                                                              d.pattern.begin() + (2u << 20) + 8192));
    CHECK(d.ctl->flush().ok());
    CHECK(file_bytes_at(d.path, 2u << 20, 8192) == std::vector<unsigned char>(8192, 0xA5));
}

TEST(emulated_write_cache_is_written_back_by_flush_commands_detach_and_stop) {
    nvme::EmulatedControllerConfig cfg;
    cfg.media = nvme::EmulatedControllerConfig::Media::MEMORY;
    cfg.image_chunk_bytes = 1u << 20;
    cfg.write_back = true;
    Drive d(cfg);
    HostSubmitter hs{d.ctl->host_queue(0)};
    auto write_at = [&](std::uint16_t cid, std::uint64_t off, unsigned char v) {
        std::memset(d.buf, v, 4096);
        nvme::Sqe w{};
        nvme::build_rw_sqe(w, nvme::kOpWrite, cid, 1, off / 512, 8, d.iova, 0);
        return hs.run(w);
    };
    CHECK(write_at(1, 0, 0x11) == 0);
    nvme::Sqe f{};
    f.cdw0 = nvme::kOpFlush | (2u << 16);
    f.nsid = 1;
    CHECK(hs.run(f) == 0);  // an NVMe FLUSH writes the cache back
    CHECK(file_bytes_at(d.path, 0, 4096) == std::vector<unsigned char>(4096, 0x11));
    CHECK(write_at(3, 5u << 20, 0x22) == 0);
    CHECK(d.ctl->detach_file(d.path).ok());  // detaching writes the file's dirty ranges back
    CHECK(file_bytes_at(d.path, 5u << 20, 4096) == std::vector<unsigned char>(4096, 0x22));
    (void)d.ctl->attach_file(d.path, {{0, d.pattern.size(), 0}});
    CHECK(write_at(4, 6u << 20, 0x33) == 0);
    d.ctl->stop();  // stopping the drive writes back too
    CHECK(file_bytes_at(d.path, 6u << 20, 4096) == std::vector<unsigned char>(4096, 0x33));
}

}  // namespace native_tests
}  // namespace tutti
