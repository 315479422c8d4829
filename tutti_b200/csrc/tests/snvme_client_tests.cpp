// Contract tests of the snvme client (the host side of a real NVMe provider)
// against the fake driver: ABI handshake, queue-group lifecycle, mapping
// rules, queue creation and teardown, error propagation, and a controller
// whose driver-created queues serve READ/WRITE commands from the host.
//
// Parity: the reference's UAPI contract test (tests/device_manager/uapi/
// uapi_contract_test.cpp: ioctl numbers and layouts) and its queue-group
// bring-up (csrc/data_paths/local_nvme/io/nvme_queue_group.cu:131-217).

#include <cerrno>
#include <cstdlib>
#include <fcntl.h>
#include <set>

#include "harness.h"

#include "../nvme/snvme_client.h"
#include "../testing/fake_snvme.h"

namespace tutti {
namespace native_tests {

namespace uapi = snvme::uapi;
using nvme::SnvmeClient;
using nvme::SnvmeController;
using nvme::SnvmeControllerConfig;
using nvme::SnvmeMemory;
using testing::FakeSnvmeConfig;
using testing::FakeSnvmeDriver;

namespace {

FakeSnvmeConfig small_fake(std::uint32_t queues = 8, std::uint32_t depth = 64) {
    FakeSnvmeConfig c;
    c.drive.name = "fake0";
    c.drive.num_io_queues = queues;
    c.drive.queue_depth = depth;
    c.drive.worker_threads = 1;
    c.drive.idle_sleep_us = 20;
    return c;
}

std::shared_ptr<FakeSnvmeDriver> make_fake(const FakeSnvmeConfig& c) {
    auto f = FakeSnvmeDriver::create(c);
    return f.ok() ? std::shared_ptr<FakeSnvmeDriver>(std::move(f).value()) : nullptr;
}

bool nothing_held(const FakeSnvmeDriver& f) {
    const auto c = f.counts();
    return c.files == 0 && c.groups == 0 && c.queues == 0 && c.ring_maps == 0 && c.data_maps == 0 &&
           c.bar_maps == 0 && c.registered == 0;
}

struct AlignedBuf {
    void* p = nullptr;
    AlignedBuf(std::size_t align, std::size_t bytes) {
        if (posix_memalign(&p, align, bytes) == 0) std::memset(p, 0, bytes);
    }
    ~AlignedBuf() { std::free(p); }
    char* c() const { return static_cast<char*>(p); }
};

}  // namespace

TEST(snvme_uapi_numbers_encode_type_number_size_and_direction) {
    CHECK(_IOC_TYPE(uapi::kMapHostMemory) == 0x80 && _IOC_NR(uapi::kMapHostMemory) == 1);
    CHECK(_IOC_SIZE(uapi::kMapHostMemory) == 40 && _IOC_DIR(uapi::kMapHostMemory) == _IOC_WRITE);
    CHECK(_IOC_NR(uapi::kGetDevInfo) == 9 && _IOC_DIR(uapi::kGetDevInfo) == _IOC_READ);
    CHECK(_IOC_SIZE(uapi::kGetDevInfo) == 104);
    CHECK(_IOC_NR(uapi::kCreateQueueGroup) == 12 && _IOC_DIR(uapi::kCreateQueueGroup) == (_IOC_READ | _IOC_WRITE));
    CHECK(_IOC_SIZE(uapi::kDestroyQueueGroup) == 4 && _IOC_NR(uapi::kDestroyQueueGroup) == 13);
    // ABI 2: the add-queue payload holds 32 pairs, and its size is part of the number
    CHECK(_IOC_SIZE(uapi::kAddUserQueue) == 1056 && _IOC_NR(uapi::kAddUserQueue) == 14);
    CHECK(_IOC_SIZE(uapi::kUnmapDeviceMemory) == 8 && _IOC_NR(uapi::kUnmapDeviceMemory) == 5);
    CHECK(_IOC_TYPE(uapi::kDeviceBind) == 0x90 && _IOC_NR(uapi::kChrdevRemove) == 4);
    CHECK(_IOC_SIZE(uapi::kRawAdminCmd) == 92 && _IOC_SIZE(uapi::kSetIoqNum) == 160);
}

TEST(snvme_attach_reads_device_info_and_maps_bar0) {
    auto fake = make_fake(small_fake());
    CHECK(fake != nullptr);
    {
        auto c = SnvmeClient::attach("/dev/ssnvme0", *fake, /*for_gpu=*/false);
        CHECK(c.ok());
        const auto& in = c.value()->info();
        CHECK(in.abi_version == uapi::kAbiVersion);
        CHECK(in.queue_depth == 64 && in.lba_bytes == 512 && in.max_transfer_bytes == (1u << 20));
        CHECK(in.first_user_qid == 1 && in.last_user_qid == 8 && in.max_queues_per_group == 32);
        CHECK(in.doorbell_stride == 4 && in.disk_name == "fake0n1");
        CHECK(fake->counts().files == 1 && fake->counts().bar_maps == 1 && fake->counts().registered == 0);
        // doorbell addresses are BAR0 + offset
        CHECK(c.value()->doorbell_host(0x1008) ==
              reinterpret_cast<std::uint32_t*>(static_cast<char*>(fake->emulated_drive()->bar0_host()) + 0x1008));
        CHECK(c.value()->doorbell_device(0x1008) == nullptr);  // not registered for a GPU
    }
    CHECK(nothing_held(*fake));
}

TEST(snvme_attach_for_gpu_registers_bar0_once_and_releases_it) {
    auto fake = make_fake(small_fake());
    CHECK(fake != nullptr);
    {
        auto c = SnvmeClient::attach("/dev/ssnvme0", *fake, /*for_gpu=*/true);
        CHECK(c.ok());
        CHECK(fake->counts().registered == 1);
        CHECK(c.value()->doorbell_device(0x1008) != nullptr);
        CHECK(!c.value()->mmio_doorbells());  // the fake's registers are host memory
    }
    CHECK(nothing_held(*fake));
}

TEST(snvme_attach_refuses_an_unknown_node) {
    auto fake = make_fake(small_fake());
    CHECK(fake != nullptr);
    auto c = SnvmeClient::attach("/dev/ssnvme7", *fake, false);
    CHECK(!c.ok() && c.status().code() == StatusCode::NOT_FOUND);
    CHECK(nothing_held(*fake));
}

TEST(snvme_attach_refuses_a_driver_before_the_handshake) {
    auto cfg = small_fake();
    cfg.abi_version = 0;
    auto fake = make_fake(cfg);
    CHECK(fake != nullptr);
    auto c = SnvmeClient::attach("/dev/ssnvme0", *fake, false);
    CHECK(!c.ok() && c.status().code() == StatusCode::UNSUPPORTED);
    CHECK(c.status().message().find("predates") != std::string::npos);
    CHECK(nothing_held(*fake));  // the file is closed again
}

TEST(snvme_attach_refuses_another_abi_version) {
    auto cfg = small_fake();
    cfg.abi_version = 3;
    auto fake = make_fake(cfg);
    CHECK(fake != nullptr);
    auto c = SnvmeClient::attach("/dev/ssnvme0", *fake, false);
    CHECK(!c.ok() && c.status().message().find("ABI 3") != std::string::npos);
    CHECK(nothing_held(*fake));
}

TEST(snvme_attach_refuses_a_driver_without_user_queues) {
    auto cfg = small_fake();
    cfg.capabilities = uapi::kCapQueueGroups | uapi::kCapMapKindTag;
    auto fake = make_fake(cfg);
    CHECK(fake != nullptr);
    auto c = SnvmeClient::attach("/dev/ssnvme0", *fake, false);
    CHECK(!c.ok() && c.status().code() == StatusCode::UNSUPPORTED);
}

TEST(snvme_attach_reports_a_node_that_is_not_an_snvme_controller) {
    auto fake = make_fake(small_fake());
    CHECK(fake != nullptr);
    fake->fail_next(uapi::kGetDevInfo, ENOTTY);
    auto c = SnvmeClient::attach("/dev/ssnvme0", *fake, false);
    CHECK(!c.ok() && c.status().message().find("not an snvme controller") != std::string::npos);
    CHECK(nothing_held(*fake));
}

TEST(snvme_one_queue_group_per_open_file) {
    auto fake = make_fake(small_fake());
    CHECK(fake != nullptr);
    auto c = SnvmeClient::attach("/dev/ssnvme0", *fake, false);
    CHECK(c.ok());
    std::uint32_t cap = 0;
    auto g = c.value()->create_group(&cap);
    CHECK(g.ok() && g.value() != 0 && cap == 32);
    auto g2 = c.value()->create_group();
    CHECK(!g2.ok() && g2.status().code() == StatusCode::RESOURCE_EXHAUSTED);
    // the driver enforces the same rule on a raw request
    const int fd = fake->open_node("/dev/ssnvme0");
    uapi::QueueGroup q{};
    CHECK(fake->ioctl_node(fd, uapi::kCreateQueueGroup, &q) == 0);
    uapi::QueueGroup q2{};
    CHECK(fake->ioctl_node(fd, uapi::kCreateQueueGroup, &q2) == -EBUSY);
    uapi::QueueGroup bad{};
    bad.flags = 1;  // must be zero
    const int fd2 = fake->open_node("/dev/ssnvme0");
    CHECK(fake->ioctl_node(fd2, uapi::kCreateQueueGroup, &bad) == -EINVAL);
    CHECK(fake->close_node(fd) == 0 && fake->close_node(fd2) == 0);
    CHECK(fake->counts().groups == 1);  // the client's group
    CHECK(c.value()->destroy_group(g.value()).ok());
    CHECK(!c.value()->destroy_group(g.value()).ok());  // already gone
}

TEST(snvme_mapping_rules_of_the_driver) {
    auto fake = make_fake(small_fake());
    CHECK(fake != nullptr);
    const int fd = fake->open_node("/dev/ssnvme0");
    AlignedBuf buf(4096, 64 << 10);
    std::vector<std::uint64_t> bus(16);
    uapi::MapRequest r{};
    r.vaddr = reinterpret_cast<std::uint64_t>(buf.p);
    r.n_pages = 16;
    r.ioaddrs = reinterpret_cast<std::uint64_t>(bus.data());
    r.legacy_queue = r.legacy_is_cq = -1;
    r.kind = uapi::kMapRingSq;
    CHECK(fake->ioctl_node(fd, uapi::kMapHostMemory, &r) == -EINVAL);  // a ring needs a group
    r.group_id = 77;
    CHECK(fake->ioctl_node(fd, uapi::kMapHostMemory, &r) == -ENOENT);  // not a group of this file
    r.group_id = 0;
    r.kind = 9;
    CHECK(fake->ioctl_node(fd, uapi::kMapHostMemory, &r) == -EINVAL);  // unknown kind
    r.kind = uapi::kMapData;
    r.mbz[1] = 1;
    CHECK(fake->ioctl_node(fd, uapi::kMapHostMemory, &r) == -EINVAL);  // reserved bytes
    r.mbz[1] = 0;
    r.vaddr += 512;
    CHECK(fake->ioctl_node(fd, uapi::kMapHostMemory, &r) == -EINVAL);  // not page-aligned
    r.vaddr -= 512;
    CHECK(fake->ioctl_node(fd, uapi::kMapHostMemory, &r) == 0);
    for (int i = 0; i < 16; ++i) CHECK(bus[i] == r.vaddr + i * 4096ull);  // the fake's IOMMU is the identity
    CHECK(fake->counts().data_maps == 1);
    std::uint64_t va = r.vaddr;
    CHECK(fake->ioctl_node(fd, uapi::kUnmapDeviceMemory, &va) == -ENOENT);  // mapped as host memory
    CHECK(fake->ioctl_node(fd, uapi::kUnmapHostMemory, &va) == 0);
    CHECK(fake->ioctl_node(fd, uapi::kUnmapHostMemory, &va) == -ENOENT);
    CHECK(fake->ioctl_node(fd, 0xdeadu, &va) == -ENOTTY);
    CHECK(fake->close_node(fd) == 0);
    CHECK(nothing_held(*fake));
}

TEST(snvme_client_maps_whole_pages_and_reports_bus_addresses) {
    auto fake = make_fake(small_fake());
    CHECK(fake != nullptr);
    auto c = SnvmeClient::attach("/dev/ssnvme0", *fake, false);
    CHECK(c.ok());
    AlignedBuf buf(4096, 5 * 4096);
    // [buf + 100, buf + 100 + 3 * 4096 + 1) touches pages 0..3
    auto m = c.value()->map(buf.c() + 100, 3 * 4096 + 1, SnvmeMemory::HOST, uapi::kMapData, 0);
    CHECK(m.ok());
    CHECK(m.value().va == reinterpret_cast<std::uint64_t>(buf.p) && m.value().bus.size() == 4);
    CHECK(m.value().page_bytes == 4096 && m.value().covers(buf.c() + 100, 3 * 4096 + 1));
    CHECK(m.value().bus_at(buf.c() + 4096 + 7) == reinterpret_cast<std::uint64_t>(buf.c()) + 4096 + 7);
    CHECK(m.value().bus_at(buf.c() + 4 * 4096) == 0);  // outside the mapping
    CHECK(fake->counts().data_maps == 1);
    CHECK(c.value()->unmap(m.value()).ok());
    CHECK(!c.value()->unmap(m.value()).ok());
    // ring kinds need a group of this file
    auto r = c.value()->map(buf.p, 4096, SnvmeMemory::HOST, uapi::kMapRingCq, 5);
    CHECK(!r.ok() && r.status().code() == StatusCode::INVALID_ARGUMENT);
    // a driver error comes back with its errno
    fake->fail_next(uapi::kMapHostMemory, ENOMEM);
    auto e = c.value()->map(buf.p, 4096, SnvmeMemory::HOST, uapi::kMapData, 0);
    CHECK(!e.ok() && e.status().code() == StatusCode::RESOURCE_EXHAUSTED);
}

TEST(snvme_add_queues_needs_rings_mapped_with_the_matching_kind) {
    auto fake = make_fake(small_fake(8, 64));
    CHECK(fake != nullptr);
    auto c = SnvmeClient::attach("/dev/ssnvme0", *fake, false);
    CHECK(c.ok());
    auto& cl = *c.value();
    auto g = cl.create_group();
    CHECK(g.ok());
    AlignedBuf sq(4096, 4096), cq(4096, 4096);
    const std::vector<uapi::QueueRings> rings{{reinterpret_cast<std::uint64_t>(sq.p), reinterpret_cast<std::uint64_t>(cq.p)}};
    // nothing mapped yet
    auto q0 = cl.add_queues(g.value(), rings);
    CHECK(!q0.ok() && q0.status().code() == StatusCode::INVALID_ARGUMENT);
    // mapped with swapped kinds
    CHECK(cl.map(sq.p, 4096, SnvmeMemory::HOST, uapi::kMapRingCq, g.value()).ok());
    CHECK(cl.map(cq.p, 4096, SnvmeMemory::HOST, uapi::kMapRingSq, g.value()).ok());
    auto q1 = cl.add_queues(g.value(), rings);
    CHECK(!q1.ok());
    CHECK(fake->counts().queues == 0 && fake->counts().ring_maps == 2);
    // a group of another file is not ours
    auto q2 = cl.add_queues(g.value() + 1, rings);
    CHECK(!q2.ok());
    // an empty or oversized batch
    CHECK(!cl.add_queues(g.value(), {}).ok());
    CHECK(!cl.add_queues(g.value(), std::vector<uapi::QueueRings>(33, rings[0])).ok());
    CHECK(cl.destroy_group(g.value()).ok());
    CHECK(fake->counts().ring_maps == 0 && fake->counts().groups == 0);
}

TEST(snvme_queue_pairs_get_distinct_qids_and_nvme_doorbell_offsets) {
    auto fake = make_fake(small_fake(8, 64));
    CHECK(fake != nullptr);
    auto c = SnvmeClient::attach("/dev/ssnvme0", *fake, false);
    CHECK(c.ok());
    auto& cl = *c.value();
    auto g = cl.create_group();
    CHECK(g.ok());
    AlignedBuf rings(4096, 6 * 4096);
    std::vector<uapi::QueueRings> rs;
    for (int q = 0; q < 3; ++q) {
        char* sq = rings.c() + q * 2 * 4096;
        char* cq = sq + 4096;
        CHECK(cl.map(sq, 4096, SnvmeMemory::HOST, uapi::kMapRingSq, g.value()).ok());
        CHECK(cl.map(cq, 4096, SnvmeMemory::HOST, uapi::kMapRingCq, g.value()).ok());
        rs.push_back({reinterpret_cast<std::uint64_t>(sq), reinterpret_cast<std::uint64_t>(cq)});
    }
    auto qs = cl.add_queues(g.value(), rs);
    CHECK(qs.ok() && qs.value().size() == 3);
    std::set<std::uint32_t> ids;
    for (const auto& q : qs.value()) {
        ids.insert(q.qid);
        CHECK(q.sq_tail_offset == 0x1000 + 8 * q.qid && q.cq_head_offset == q.sq_tail_offset + 4);
    }
    CHECK(ids.size() == 3 && fake->live_qids().size() == 3 && fake->counts().queues == 3);
    // the pool runs dry: 8 QIDs, 3 taken, 6 more asked
    AlignedBuf more(4096, 12 * 4096);
    std::vector<uapi::QueueRings> rs2;
    for (int q = 0; q < 6; ++q) {
        char* sq = more.c() + q * 2 * 4096;
        CHECK(cl.map(sq, 4096, SnvmeMemory::HOST, uapi::kMapRingSq, g.value()).ok());
        CHECK(cl.map(sq + 4096, 4096, SnvmeMemory::HOST, uapi::kMapRingCq, g.value()).ok());
        rs2.push_back({reinterpret_cast<std::uint64_t>(sq), reinterpret_cast<std::uint64_t>(sq + 4096)});
    }
    auto full = cl.add_queues(g.value(), rs2);
    CHECK(!full.ok() && full.status().code() == StatusCode::RESOURCE_EXHAUSTED);
    CHECK(fake->counts().queues == 3);  // nothing half-created
    // destroying the group deletes the queue pairs and returns the QIDs
    CHECK(cl.destroy_group(g.value()).ok());
    CHECK(fake->live_qids().empty() && fake->counts().ring_maps == 0);
}

TEST(snvme_close_releases_what_a_file_still_holds) {
    auto fake = make_fake(small_fake(8, 64));
    CHECK(fake != nullptr);
    const int fd = fake->open_node("/dev/ssnvme0");
    uapi::QueueGroup q{};
    CHECK(fake->ioctl_node(fd, uapi::kCreateQueueGroup, &q) == 0);
    AlignedBuf rings(4096, 3 * 4096);
    std::vector<std::uint64_t> bus(1);
    auto map = [&](char* p, std::uint8_t kind, std::uint32_t group) {
        uapi::MapRequest r{};
        r.vaddr = reinterpret_cast<std::uint64_t>(p);
        r.n_pages = 1;
        r.ioaddrs = reinterpret_cast<std::uint64_t>(bus.data());
        r.legacy_queue = r.legacy_is_cq = -1;
        r.group_id = group;
        r.kind = kind;
        return fake->ioctl_node(fd, uapi::kMapHostMemory, &r);
    };
    CHECK(map(rings.c(), uapi::kMapRingSq, q.group_id) == 0);
    CHECK(map(rings.c() + 4096, uapi::kMapRingCq, q.group_id) == 0);
    CHECK(map(rings.c() + 8192, uapi::kMapData, 0) == 0);
    auto add = std::make_unique<uapi::AddUserQueues>();
    std::memset(add.get(), 0, sizeof(*add));
    add->group_id = q.group_id;
    add->nr_pairs = 1;
    add->rings[0] = {reinterpret_cast<std::uint64_t>(rings.c()), reinterpret_cast<std::uint64_t>(rings.c() + 4096)};
    CHECK(fake->ioctl_node(fd, uapi::kAddUserQueue, add.get()) == 0);
    CHECK(add->out[0].qid == 1);
    const auto held = fake->counts();
    CHECK(held.groups == 1 && held.queues == 1 && held.ring_maps == 2 && held.data_maps == 1);
    CHECK(fake->close_node(fd) == 0);  // the process "died": the close cascade
    CHECK(nothing_held(*fake) && fake->live_qids().empty());
    CHECK(fake->close_node(fd) == -EBADF);
}

TEST(snvme_controller_spans_groups_and_serves_commands_from_the_host) {
    // 40 queue pairs over groups of at most 32: two open files
    auto fake = make_fake(small_fake(48, 64));
    CHECK(fake != nullptr);
    char path[] = "/tmp/tutti_snvme_XXXXXX";
    const int fd = mkstemp(path);
    CHECK(fd >= 0);
    std::vector<unsigned char> pattern(1 << 20);
    for (std::size_t i = 0; i < pattern.size(); ++i) pattern[i] = static_cast<unsigned char>(i * 131 + 7);
    CHECK(write(fd, pattern.data(), pattern.size()) == static_cast<ssize_t>(pattern.size()));
    close(fd);
    {
        SnvmeControllerConfig cc;
        cc.node = "/dev/ssnvme0";
        cc.num_io_queues = 40;
        auto ctl = SnvmeController::create(cc, fake);
        CHECK(ctl.ok());
        auto& c = *ctl.value();
        CHECK(c.groups() == 2 && fake->counts().queues == 40 && fake->counts().files == 2);
        CHECK(c.info().kind == "snvme" && c.info().queue_depth == 64 && c.info().num_io_queues == 40);
        CHECK(c.info().mdts_bytes == (1u << 20));
        std::set<std::uint32_t> qids;
        for (std::uint32_t i = 0; i < 40; ++i) {
            const auto v = c.host_queue(i);
            CHECK(v.sq && v.cq && v.depth == 64 && v.flags == 0);  // fake registers: not MMIO
            qids.insert(v.qid);
        }
        CHECK(qids.size() == 40);
        // the namespace holds the file; a data buffer mapped through the driver
        CHECK(c.emulated_drive() == fake->emulated_drive());
        CHECK(fake->emulated_drive()->attach_file(path, {{0, pattern.size(), 0}}).ok());
        AlignedBuf buf(4096, 64 << 10);
        auto m = c.map_dma(buf.p, 64 << 10);
        CHECK(m.ok() && m.value().page_bytes == 4096 && m.value().bus.size() == 16);
        AlignedBuf list(4096, 4096);
        auto lm = c.map_dma(list.p, 4096);
        CHECK(lm.ok());
        auto* l = static_cast<std::uint64_t*>(list.p);
        for (int k = 1; k < 16; ++k) l[k - 1] = m.value().bus[k];
        // READ 64 KiB at LBA 256 through queue 37 (second group), PRP list
        HostSubmitter hs{c.host_queue(37)};
        nvme::Sqe e{};
        nvme::build_rw_sqe(e, nvme::kOpRead, 5, 1, 256, 128, m.value().bus[0], lm.value().bus[0]);
        CHECK(hs.run(e) == 0);
        CHECK(std::memcmp(buf.p, pattern.data() + 256 * 512, 64 << 10) == 0);
        // WRITE one page through queue 0, read it back through queue 39
        std::memset(buf.p, 0x5A, 4096);
        HostSubmitter h0{c.host_queue(0)};
        nvme::build_rw_sqe(e, nvme::kOpWrite, 6, 1, 8, 8, m.value().bus[0], 0);
        CHECK(h0.run(e) == 0);
        std::memset(buf.p, 0, 4096);
        HostSubmitter h39{c.host_queue(39)};
        nvme::build_rw_sqe(e, nvme::kOpRead, 7, 1, 8, 8, m.value().bus[0], 0);
        CHECK(h39.run(e) == 0);
        CHECK(static_cast<unsigned char*>(buf.p)[100] == 0x5A);
        // a queue reset is a group-wide operation on this driver
        CHECK(c.reset_queue(3).code() == StatusCode::UNSUPPORTED);
        CHECK(c.unmap_dma(m.value()).ok() && c.unmap_dma(lm.value()).ok());
        fake->emulated_drive()->stop();
    }
    CHECK(nothing_held(*fake));
    unlink(path);
}

TEST(snvme_controller_bring_up_failure_releases_everything) {
    auto fake = make_fake(small_fake(48, 64));
    CHECK(fake != nullptr);
    SnvmeControllerConfig cc;
    cc.node = "/dev/ssnvme0";
    cc.num_io_queues = 40;
    {
        auto ctl = SnvmeController::create(cc, fake);
        CHECK(ctl.ok());
    }
    CHECK(nothing_held(*fake));
    // queue creation fails in the driver: what was created so far is released
    fake->fail_next(uapi::kAddUserQueue, ENOSPC, 1);
    auto bad = SnvmeController::create(cc, fake);
    CHECK(!bad.ok() && bad.status().code() == StatusCode::RESOURCE_EXHAUSTED);
    CHECK(nothing_held(*fake));
    // more queue pairs than the driver's QID pool
    cc.num_io_queues = 49;
    auto big = SnvmeController::create(cc, fake);
    CHECK(!big.ok() && big.status().code() == StatusCode::RESOURCE_EXHAUSTED);
    CHECK(nothing_held(*fake));
}

TEST(snvme_provider_is_reported_missing_on_a_machine_without_the_driver) {
    // The production system interface against a node that does not exist here.
    SnvmeControllerConfig cc;
    cc.node = "/dev/ssnvme_absent_for_test";
    cc.num_io_queues = 1;
    auto ctl = SnvmeController::create(cc);
    CHECK(!ctl.ok() && ctl.status().code() == StatusCode::NOT_FOUND);
}

}  // namespace native_tests
}  // namespace tutti

namespace tutti {
namespace native_tests {

TEST(snvme_owner_binds_creates_the_node_and_waits_for_the_scan) {
    auto cfg = small_fake();
    cfg.owner_mode = true;
    cfg.probe_polls = 3;
    auto fake = make_fake(cfg);
    CHECK(fake != nullptr);
    // before the owner: no node to attach to
    CHECK(!SnvmeClient::attach("/dev/ssnvme0", *fake, false).ok());
    {
        auto o = nvme::SnvmeOwner::bring_up("/dev/snvm_control", "0000:1b:00.0", 16, *fake);
        CHECK(o.ok());
        CHECK(o.value()->node() == "/dev/ssnvme0" && o.value()->minor() == 0);
        CHECK(o.value()->info().disk_name == "fake0n1" && o.value()->block_device() == "/dev/fake0n1");
        const auto c = fake->counts();
        CHECK(c.node_created && c.bound && c.kernel_ioq_cap == 16);
        // a client attaches to the node the owner made
        auto cl = SnvmeClient::attach(o.value()->node(), *fake, false);
        CHECK(cl.ok());
    }
    const auto c = fake->counts();
    CHECK(!c.node_created && !c.bound && c.files == 0);  // unbound and removed
}

TEST(snvme_owner_rejects_bad_addresses_and_undoes_a_failed_bind) {
    auto cfg = small_fake();
    cfg.owner_mode = true;
    auto fake = make_fake(cfg);
    CHECK(fake != nullptr);
    CHECK(!nvme::parse_pci_address("1b:00.0").ok());
    CHECK(!nvme::parse_pci_address("0000:1b:00.9").ok());
    auto a = nvme::parse_pci_address("0000:1b:00.1");
    CHECK(a.ok() && a.value().bus == 0x1b && a.value().function == 1);
    // another function than the driver knows
    auto wrong = nvme::SnvmeOwner::bring_up("/dev/snvm_control", "0000:1b:00.1", 0, *fake);
    CHECK(!wrong.ok() && wrong.status().code() == StatusCode::NOT_FOUND);
    // the bind fails: the node created before it is removed again
    fake->fail_next(uapi::kDeviceBind, EIO);
    auto failed = nvme::SnvmeOwner::bring_up("/dev/snvm_control", "0000:1b:00.0", 0, *fake);
    CHECK(!failed.ok());
    CHECK(!fake->counts().node_created && fake->counts().files == 0);
    // no control node at all
    auto none = nvme::SnvmeOwner::bring_up("/dev/snvm_absent", "0000:1b:00.0", 0, *fake);
    CHECK(!none.ok() && none.status().code() == StatusCode::NOT_FOUND);
}

TEST(snvme_owner_times_out_when_the_scan_never_names_the_disk) {
    auto cfg = small_fake();
    cfg.owner_mode = true;
    cfg.probe_polls = 1000000;
    auto fake = make_fake(cfg);
    CHECK(fake != nullptr);
    auto o = nvme::SnvmeOwner::bring_up("/dev/snvm_control", "0000:1b:00.0", 0, *fake, /*probe_wait_ms=*/50);
    CHECK(!o.ok() && o.status().code() == StatusCode::TIMEOUT);
    CHECK(!fake->counts().bound && !fake->counts().node_created);
}

}  // namespace native_tests
}  // namespace tutti
