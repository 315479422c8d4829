// tutti_snvme_smoke: bring-up check of one controller behind the snvme driver.
//
//   tutti_snvme_smoke --node /dev/snvm0 [--queues N] [--lba L] [--bytes B] [--rounds R] [--write]
//   tutti_snvme_smoke --fake [...]      (the fake driver over an emulated drive and a temporary file)
//
// Steps, each reported on its own line:
//   1. attach: the driver's handshake (ABI version, capabilities), device
//      information, BAR0 mapped for doorbells; queue groups and N user queue
//      pairs created through the driver (SnvmeController);
//   2. mapping: a page-aligned host buffer and a PRP-list page mapped for DMA
//      through the driver (per-page bus addresses);
//   3. rounds on every queue in turn: without --write, two READs of the same
//      range must return the same bytes (nothing on the drive changes); with
//      --write (destroys the range's data), a position pattern is written,
//      read back and compared.
// The last line is one JSON object: {"ok": ..., "node": ..., "rounds": ...,
// "read_us": [...], "write_us": [...]}. Exit code 0 when every round passed.
// A GPU round is the runtime's io kernel over the same driver
// (`bench.py --provider snvme`, `kernels io`), not repeated here.
//
// Parity: reference kernel_modules/test/snvme_smoke*.c and run_snvme_smoke.sh
// (bind, add queue, queue group, CPU IO rounds against one drive).

#include <unistd.h>

#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "nvme/nvme_spec.h"
#include "nvme/snvme_client.h"
#include "testing/fake_snvme.h"

namespace {

using tutti::nvme::QueuePairView;

struct Args {
    std::string node;
    bool fake = false;
    std::uint32_t queues = 1;
    std::uint64_t lba = 0;
    std::uint64_t bytes = 64 << 10;
    std::uint32_t rounds = 4;
    bool write = false;
};

void usage() {
    std::fprintf(stderr,
                 "usage: tutti_snvme_smoke (--node PATH | --fake) [--queues N] [--lba L] [--bytes B] "
                 "[--rounds R] [--write]\n");
}

bool parse(int argc, char** argv, Args& a) {
    for (int i = 1; i < argc; ++i) {
        const std::string k = argv[i];
        auto val = [&](const char* what) -> const char* {
            if (i + 1 >= argc) {
                std::fprintf(stderr, "%s needs a value\n", what);
                return nullptr;
            }
            return argv[++i];
        };
        if (k == "--fake") {
            a.fake = true;
        } else if (k == "--write") {
            a.write = true;
        } else if (k == "--node" || k == "--queues" || k == "--lba" || k == "--bytes" || k == "--rounds") {
            const char* v = val(k.c_str());
            if (!v) return false;
            if (k == "--node")
                a.node = v;
            else if (k == "--queues")
                a.queues = static_cast<std::uint32_t>(std::strtoul(v, nullptr, 0));
            else if (k == "--lba")
                a.lba = std::strtoull(v, nullptr, 0);
            else if (k == "--bytes")
                a.bytes = std::strtoull(v, nullptr, 0);
            else
                a.rounds = static_cast<std::uint32_t>(std::strtoul(v, nullptr, 0));
        } else {
            std::fprintf(stderr, "unknown argument %s\n", k.c_str());
            return false;
        }
    }
    if (a.fake == !a.node.empty()) {
        std::fprintf(stderr, "give exactly one of --node PATH and --fake\n");
        return false;
    }
    if (a.queues == 0 || a.rounds == 0 || a.bytes == 0) {
        std::fprintf(stderr, "--queues, --rounds and --bytes must be positive\n");
        return false;
    }
    return true;
}

// One command at a time on a host-visible queue pair, bounded wait for its CQE.
struct HostQueue {
    QueuePairView q;
    std::uint32_t tail = 0, head = 0, phase = 1;
    std::uint16_t cid = 1;

    // status field of the CQE; -1 when none arrived within `timeout_ms`
    int run(const tutti::nvme::Sqe& cmd, int timeout_ms) {
        tutti::nvme::Sqe e = cmd;
        e.cdw0 = (e.cdw0 & 0xFFFFu) | (static_cast<std::uint32_t>(cid++) << 16);
        volatile tutti::nvme::Sqe* slot = q.sq + tail;
        std::memcpy(const_cast<tutti::nvme::Sqe*>(slot), &e, sizeof e);
        tail = (tail + 1) % q.depth;
        __atomic_thread_fence(__ATOMIC_SEQ_CST);  // the SQE before the doorbell
        *reinterpret_cast<volatile std::uint32_t*>(q.sq_doorbell) = tail;
        const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
        for (;;) {
            const std::uint32_t dw3 = __atomic_load_n(&q.cq[head].dw3, __ATOMIC_ACQUIRE);
            if (tutti::nvme::cqe_phase(dw3) == phase) {
                head = (head + 1) % q.depth;
                if (head == 0) phase ^= 1u;
                *reinterpret_cast<volatile std::uint32_t*>(q.cq_doorbell) = head;
                return static_cast<int>(tutti::nvme::cqe_status(dw3));
            }
            if (std::chrono::steady_clock::now() > deadline) return -1;
            usleep(5);
        }
    }
};

struct Aligned {
    void* p = nullptr;
    Aligned(std::size_t align, std::size_t bytes) {
        if (posix_memalign(&p, align, bytes) != 0) p = nullptr;
        if (p) std::memset(p, 0, bytes);
    }
    ~Aligned() { std::free(p); }
};

double elapsed_us(std::chrono::steady_clock::time_point t0) {
    return std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - t0).count();
}

}  // namespace

int main(int argc, char** argv) {
    using namespace tutti;
    Args a;
    if (!parse(argc, argv, a)) {
        usage();
        return 2;
    }
    std::shared_ptr<testing::FakeSnvmeDriver> fake;
    std::string backing;
    nvme::SnvmeControllerConfig cc;
    cc.num_io_queues = a.queues;
    cc.node = a.node;
    if (a.fake) {
        testing::FakeSnvmeConfig fc;
        fc.drive.name = "smoke0";
        fc.drive.num_io_queues = a.queues;
        fc.drive.queue_depth = 64;
        fc.drive.worker_threads = 1;
        fc.drive.idle_sleep_us = 20;
        auto f = testing::FakeSnvmeDriver::create(fc);
        if (!f.ok()) {
            std::printf("attach: fake driver failed: %s\n", f.status().to_string().c_str());
            return 1;
        }
        fake = std::shared_ptr<testing::FakeSnvmeDriver>(std::move(f).value());
        cc.node = fc.node;
        char path[] = "/tmp/tutti_snvme_smoke_XXXXXX";
        const int fd = mkstemp(path);
        const std::uint64_t span = a.lba * 512 + (a.bytes + 4095) / 4096 * 4096 + 4096;
        if (fd < 0 || ftruncate(fd, static_cast<off_t>(span)) != 0) {
            std::printf("attach: cannot create the backing file\n");
            return 1;
        }
        close(fd);
        backing = path;
        if (!fake->emulated_drive()->attach_file(backing, {{0, span, 0}}).ok()) {
            std::printf("attach: the backing file was refused\n");
            return 1;
        }
    }
    auto ctl = a.fake ? nvme::SnvmeController::create(cc, fake) : nvme::SnvmeController::create(cc);
    if (!ctl.ok()) {
        std::printf("attach: %s: %s\n", cc.node.c_str(), ctl.status().to_string().c_str());
        return 1;
    }
    std::unique_ptr<nvme::SnvmeController> owned = std::move(ctl).value();
    auto& c = *owned;
    const auto& info = c.info();
    std::printf("attach: %s (%s): %u queue pairs in %u group(s), depth %u, LBA %u bytes, MDTS %u bytes, %s doorbells\n",
                cc.node.c_str(), info.name.c_str(), info.num_io_queues, c.groups(), info.queue_depth,
                info.lba_bytes, info.mdts_bytes, c.host_queue(0).flags ? "MMIO" : "host-memory");
    const std::uint64_t lba_bytes = info.lba_bytes;
    std::uint64_t bytes = (a.bytes + 4095) / 4096 * 4096;
    if (bytes > info.mdts_bytes) bytes = info.mdts_bytes / 4096 * 4096;
    if (bytes % lba_bytes) {
        std::printf("mapping: %llu bytes is not a whole number of %llu-byte LBAs\n",
                    static_cast<unsigned long long>(bytes), static_cast<unsigned long long>(lba_bytes));
        return 1;
    }
    const std::uint64_t pages = bytes / 4096;
    Aligned buf(4096, bytes), ref(4096, bytes), list(4096, 4096);
    if (!buf.p || !ref.p || !list.p || pages > 513 || bytes / lba_bytes > 65536) {
        std::printf("mapping: cannot allocate %llu bytes (at most 2 MiB per command)\n",
                    static_cast<unsigned long long>(bytes));
        return 1;
    }
    auto m = c.map_dma(buf.p, bytes);
    auto lm = c.map_dma(list.p, 4096);
    if (!m.ok() || !lm.ok()) {
        std::printf("mapping: %s\n", (!m.ok() ? m.status() : lm.status()).to_string().c_str());
        return 1;
    }
    // PRP1 names the first page; PRP2 the second page, or a list of pages 2..n
    std::uint64_t prp2 = 0;
    if (pages == 2) {
        prp2 = m.value().bus_at(static_cast<char*>(buf.p) + 4096);
    } else if (pages > 2) {
        auto* l = static_cast<std::uint64_t*>(list.p);
        for (std::uint64_t k = 1; k < pages; ++k) l[k - 1] = m.value().bus_at(static_cast<char*>(buf.p) + k * 4096);
        prp2 = lm.value().bus_at(list.p);
    }
    std::printf("mapping: %llu bytes in %llu page(s), PRP %s\n", static_cast<unsigned long long>(bytes),
                static_cast<unsigned long long>(pages), pages > 2 ? "list" : pages == 2 ? "pair" : "single");
    const std::uint32_t nlb = static_cast<std::uint32_t>(bytes / lba_bytes);
    std::vector<HostQueue> qs;
    for (std::uint32_t i = 0; i < info.num_io_queues; ++i) qs.push_back(HostQueue{c.host_queue(i)});
    std::vector<double> read_us, write_us;
    bool ok = true;
    auto rw = [&](HostQueue& hq, std::uint8_t op, const char* what, std::vector<double>& times) {
        nvme::Sqe e{};
        nvme::build_rw_sqe(e, op, 0, info.nsid, a.lba, nlb, m.value().bus_at(buf.p), prp2);
        const auto t0 = std::chrono::steady_clock::now();
        const int st = hq.run(e, 5000);
        times.push_back(elapsed_us(t0));
        if (st != 0) {
            std::printf("round: %s on qid %u %s\n", what, hq.q.qid,
                        st < 0 ? "timed out after 5 s" : ("failed, status 0x" + std::to_string(st)).c_str());
            ok = false;
        }
        return st == 0;
    };
    for (std::uint32_t r = 0; r < a.rounds && ok; ++r) {
        HostQueue& hq = qs[r % qs.size()];
        auto* b = static_cast<unsigned char*>(buf.p);
        if (a.write) {
            for (std::uint64_t i = 0; i < bytes; ++i) b[i] = static_cast<unsigned char>((i * 131 + r * 7 + 1) & 0xFF);
            std::memcpy(ref.p, buf.p, bytes);
            if (!rw(hq, nvme::kOpWrite, "WRITE", write_us)) break;
            std::memset(buf.p, 0, bytes);
            if (!rw(hq, nvme::kOpRead, "READ", read_us)) break;
        } else {
            if (!rw(hq, nvme::kOpRead, "READ", read_us)) break;
            std::memcpy(ref.p, buf.p, bytes);
            std::memset(buf.p, 0xA5, bytes);
            if (!rw(hq, nvme::kOpRead, "READ", read_us)) break;
        }
        const bool same = std::memcmp(buf.p, ref.p, bytes) == 0;
        std::printf("round %u: qid %u, %s %s\n", r, hq.q.qid, a.write ? "write + read back" : "read twice",
                    same ? "match" : "MISMATCH");
        ok = ok && same;
    }
    (void)c.unmap_dma(m.value());
    (void)c.unmap_dma(lm.value());
    auto join = [](const std::vector<double>& v) {
        std::string s = "[";
        for (std::size_t i = 0; i < v.size(); ++i) s += (i ? ", " : "") + std::to_string(static_cast<long long>(v[i]));
        return s + "]";
    };
    std::printf("{\"ok\": %s, \"node\": \"%s\", \"fake\": %s, \"queues\": %u, \"bytes\": %llu, \"rounds\": %u, "
                "\"write\": %s, \"read_us\": %s, \"write_us\": %s}\n",
                ok ? "true" : "false", cc.node.c_str(), a.fake ? "true" : "false", info.num_io_queues,
                static_cast<unsigned long long>(bytes), a.rounds, a.write ? "true" : "false", join(read_us).c_str(),
                join(write_us).c_str());
    owned.reset();  // the controller's queues and mappings before the fake driver
    if (fake) fake->emulated_drive()->stop();
    if (!backing.empty()) unlink(backing.c_str());
    return ok ? 0 : 1;
}
