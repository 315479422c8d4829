#pragma once
// A stand-in for the snvme kernel driver, for machines without one (CPU test
// hosts, GPU boxes without bindable drives).
//
// It answers the per-controller node's ioctls with the driver's rules, the
// ones its clients depend on:
//   * GET_DEV_INFO with the ABI handshake (version and capabilities settable,
//     to exercise a client against an older or a partial driver);
//   * one queue group per open file, at most `max_queues_per_group` queues;
//   * ring mappings need the kind tag and a group of the same file; data
//     mappings belong to the file; pages of 4 KiB (host) or 64 KiB (GPU);
//   * ADD_USER_QUEUE only over rings mapped with the matching kind in the
//     group; QIDs from a pool; every queue has the controller's depth;
//   * DESTROY_QUEUE_GROUP deletes the group's queues and ring mappings;
//     closing a file releases everything it still holds.
// Its hardware is an EmulatedNvmeController with driver-created queues: a
// queue pair exists on it from ADD_USER_QUEUE to DESTROY_QUEUE_GROUP (or
// close), its doorbells are the emulated register file, and a mapping is a
// DMA window of the emulated drive (bus address == virtual address). The
// emulated drive reads rings with host threads, so rings must be host memory.
//
// Seams: fail_next() makes the next N calls of one ioctl fail with an errno;
// counts() reports what is still held (files, groups, queues, mappings).

#include <cstdint>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../nvme/snvme_client.h"

namespace tutti {
namespace testing {

struct FakeSnvmeConfig {
    std::string node = "/dev/ssnvme0";
    nvme::EmulatedControllerConfig drive;  // driver_created_queues is forced on
    std::uint32_t abi_version = snvme::uapi::kAbiVersion;
    std::uint32_t capabilities = snvme::uapi::kClientCaps | snvme::uapi::kCapRawAdmin | snvme::uapi::kCapKernelIoqCap;
    std::uint32_t first_user_qid = 1;
    std::uint32_t max_queues_per_group = snvme::uapi::kMaxQueuesPerGroup;
    // Owner side: the control node binds `pci` and creates `node` (minor
    // `minor`). With owner_mode the node exists only after CHRDEV_CREATE and
    // the disk is named only after DEVICE_BIND plus `probe_polls` device-info
    // queries (the namespace scan); without it the controller is already up.
    std::string control_node = "/dev/snvm_control";
    std::string pci = "0000:1b:00.0";
    int minor = 0;
    bool owner_mode = false;
    std::uint32_t probe_polls = 2;
};

class FakeSnvmeDriver final : public nvme::SnvmeSys {
public:
    static Result<std::unique_ptr<FakeSnvmeDriver>> create(const FakeSnvmeConfig& cfg);
    ~FakeSnvmeDriver() override;

    int open_node(const std::string& path) override;
    int close_node(int fd) override;
    int ioctl_node(int fd, unsigned long request, void* arg) override;
    void* map_registers(int fd, std::size_t bytes) override;
    void unmap_registers(void* p, std::size_t bytes) override;
    Result<void*> register_registers(void* p, std::size_t bytes) override;
    void unregister_registers(void* p) override;
    bool registers_are_mmio() const override { return false; }
    nvme::EmulatedNvmeController* emulated_drive() override { return drive_.get(); }

    // The next `count` calls of `request` fail with -errno_value.
    void fail_next(unsigned long request, int errno_value, std::uint32_t count = 1);

    struct Counts {
        std::uint32_t files = 0, groups = 0, queues = 0, ring_maps = 0, data_maps = 0, bar_maps = 0, registered = 0;
        bool node_created = false, bound = false;
        std::uint32_t kernel_ioq_cap = 0;
    };
    Counts counts() const;
    std::vector<std::uint32_t> live_qids() const;

private:
    explicit FakeSnvmeDriver(const FakeSnvmeConfig& cfg) : cfg_(cfg) {}
    struct Mapping {
        std::uint64_t va = 0, bytes = 0;
        std::uint8_t kind = 0;
        bool device = false;
    };
    struct Group {
        std::uint32_t id = 0;
        std::vector<Mapping> rings;
        std::vector<std::uint32_t> qids;
    };
    struct File {
        bool control = false;
        std::vector<Group> groups;
        std::vector<Mapping> data;
    };
    int control_ioctl(unsigned long request, void* arg);
    bool node_created_ = true, bound_ = true;
    std::uint32_t probe_polls_left_ = 0, kernel_ioq_cap_ = 0;
    int get_info(void* arg);
    int create_group(File& f, void* arg);
    int destroy_group(File& f, std::uint32_t id);
    int map(File& f, void* arg, bool device);
    int unmap(File& f, std::uint64_t va, bool device);
    int add_queues(File& f, void* arg);
    void release_file(File& f);
    static const Mapping* find_ring(const Group& g, std::uint64_t va, std::uint8_t kind);

    FakeSnvmeConfig cfg_;
    std::unique_ptr<nvme::EmulatedNvmeController> drive_;
    mutable std::mutex mu_;
    int next_fd_ = 3;
    std::uint32_t next_group_ = 1;
    std::map<int, File> files_;
    std::vector<bool> qid_used_;  // index: qid
    std::uint32_t bar_maps_ = 0, registered_ = 0;
    std::map<unsigned long, std::pair<int, std::uint32_t>> fail_;
};

}  // namespace testing
}  // namespace tutti
