#pragma once
// Host side of a real NVMe provider: a user-space client of the snvme
// queue-leasing driver and the NvmeController built on it.
//
// The client opens a controller's node, checks the driver's ABI handshake,
// maps the controller's BAR0 (its doorbells) and registers it with CUDA as
// I/O memory, creates a queue group, DMA-maps ring and data buffers (the
// driver pins them and returns one bus address per page) and has the driver
// create I/O queue pairs over the rings. Closing the node releases all of it;
// the client also releases what it created, in reverse order.
//
// SnvmeController turns one controller into the NvmeController the GPU data
// path consumes: `num_io_queues` queue pairs (one queue group per open file,
// at most kMaxQueuesPerGroup queues per group), rings in page-locked host
// memory or in GPU memory, doorbells in BAR0 written with .mmio stores by the
// io kernel (QueuePairView::flags), data buffers mapped per page.
//
// Every OS and CUDA call goes through SnvmeSys, so a fake driver can stand in
// for the kernel module (testing/fake_snvme.h) on machines without one.
//
// Parity: the reference's libnvm client attach and BAR0 registration
// (csrc/device_manager/nvme/libnvm/src/linux/device.cpp:737,791) and its
// queue-group bring-up (csrc/data_paths/local_nvme/io/nvme_queue_group.cu:131-217).

#include <cstdint>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include <tutti/spi/snvme_uapi.h>
#include <tutti/status.h>

#include "controller.h"
#include "host_memory.h"

namespace tutti {
namespace nvme {

// The OS and CUDA calls of the client.
class SnvmeSys {
public:
    virtual ~SnvmeSys() = default;
    virtual int open_node(const std::string& path) = 0;  // file descriptor, or -errno
    virtual int close_node(int fd) = 0;
    virtual int ioctl_node(int fd, unsigned long request, void* arg) = 0;  // 0, or -errno
    // Maps `bytes` of the controller's BAR0 (nullptr on failure).
    virtual void* map_registers(int fd, std::size_t bytes) = 0;
    virtual void unmap_registers(void* p, std::size_t bytes) = 0;
    // Makes mapped registers reachable from GPU kernels; returns their device address.
    virtual Result<void*> register_registers(void* p, std::size_t bytes) = 0;
    virtual void unregister_registers(void* p) = 0;
    // True when the registers are device MMIO (kernels use .mmio stores on them).
    virtual bool registers_are_mmio() const = 0;
    // The emulated drive behind a fake driver (nullptr for real hardware).
    virtual EmulatedNvmeController* emulated_drive() { return nullptr; }
};

// open(2)/ioctl(2)/mmap(2) on the driver's nodes; BAR0 registered with
// cudaHostRegister(IoMemory | Mapped).
SnvmeSys& linux_snvme_sys();

struct SnvmeDeviceInfo {
    std::string disk_name;
    std::uint32_t abi_version = 0;
    std::uint32_t capabilities = 0;
    std::uint32_t lba_bytes = 512;
    std::uint64_t max_transfer_bytes = 0;
    std::uint32_t queue_depth = 0;       // CAP.MQES + 1
    std::uint32_t doorbell_stride = 4;   // bytes between doorbells (4 << CAP.DSTRD)
    std::uint32_t first_user_qid = 0;
    std::uint32_t last_user_qid = 0;
    std::uint32_t max_queues_per_group = 0;
    std::uint64_t bar0_bytes = 0;
    bool sgl = false;
};

// Where a mapped buffer lives (selects the map ioctl and its page size).
enum class SnvmeMemory : int { HOST = 0, DEVICE = 1 };

struct SnvmeQueue {
    std::uint32_t qid;
    std::uint32_t sq_tail_offset;  // BAR0 byte offsets
    std::uint32_t cq_head_offset;
};

class SnvmeClient {
public:
    // `for_gpu`: register BAR0 with CUDA (kernels ring the doorbells).
    static Result<std::unique_ptr<SnvmeClient>> attach(const std::string& node, SnvmeSys& sys, bool for_gpu);
    ~SnvmeClient();
    SnvmeClient(const SnvmeClient&) = delete;
    SnvmeClient& operator=(const SnvmeClient&) = delete;

    const SnvmeDeviceInfo& info() const { return info_; }
    bool mmio_doorbells() const { return sys_->registers_are_mmio(); }

    // One queue group per open file; returns its id and the driver's queue cap.
    Result<std::uint32_t> create_group(std::uint32_t* max_queues = nullptr);
    // Deletes the group's queue pairs and releases its ring mappings.
    Status destroy_group(std::uint32_t group);
    // Pins [p, p+bytes) for the controller. Ring kinds need a group; data
    // mappings belong to the open file.
    Result<DmaMapping> map(void* p, std::uint64_t bytes, SnvmeMemory where, std::uint8_t kind, std::uint32_t group);
    Status unmap(const DmaMapping& m);
    // Creates one I/O queue pair per entry over rings mapped in `group`.
    Result<std::vector<SnvmeQueue>> add_queues(std::uint32_t group, const std::vector<snvme::uapi::QueueRings>& rings);

    std::uint32_t* doorbell_host(std::uint32_t offset) const;
    std::uint32_t* doorbell_device(std::uint32_t offset) const;  // nullptr unless registered for the GPU

private:
    SnvmeClient() = default;
    Status ioctl(unsigned long request, void* arg, const char* what);

    struct Mapped {
        std::uint64_t va;
        SnvmeMemory where;
        std::uint32_t group;  // 0: a data mapping of the file
    };
    SnvmeSys* sys_ = nullptr;
    int fd_ = -1;
    std::string node_;
    SnvmeDeviceInfo info_;
    void* bar_ = nullptr;
    void* bar_device_ = nullptr;
    std::vector<std::uint32_t> groups_;
    std::vector<Mapped> maps_;
};

// "dddd:bb:ss.f" (hexadecimal fields) as the driver's PCI address.
Result<snvme::uapi::PciAddress> parse_pci_address(const std::string& text);

// Owner side: binds a controller to the snvme driver and creates its node,
// which clients then attach to. Bring-up: open the control node,
// CHRDEV_CREATE (the driver returns the node's minor), open the node, an
// optional kernel I/O-queue cap (before the bind), DEVICE_BIND, then
// GET_DEV_INFO until the namespace scan has named the disk (bounded). Any
// failure undoes what was done. Destruction unbinds and removes the node.
// Parity: the reference's nvm_controller_init_common
// (csrc/device_manager/nvme/libnvm/src/linux/device.cpp:512-700).
class SnvmeOwner {
public:
    static Result<std::unique_ptr<SnvmeOwner>> bring_up(const std::string& control_node, const std::string& pci,
                                                        std::uint32_t kernel_ioq_cap, SnvmeSys& sys,
                                                        std::uint32_t probe_wait_ms = 10000);
    ~SnvmeOwner();
    SnvmeOwner(const SnvmeOwner&) = delete;
    SnvmeOwner& operator=(const SnvmeOwner&) = delete;

    const std::string& node() const { return node_; }
    int minor() const { return minor_; }
    const SnvmeDeviceInfo& info() const { return info_; }
    std::string block_device() const { return info_.disk_name.empty() ? "" : "/dev/" + info_.disk_name; }

private:
    SnvmeOwner() = default;
    SnvmeSys* sys_ = nullptr;
    int control_fd_ = -1, dev_fd_ = -1;
    snvme::uapi::PciAddress pci_{};
    bool created_ = false, bound_ = false;
    int minor_ = -1;
    std::string node_;
    SnvmeDeviceInfo info_;
};

struct SnvmeControllerConfig {
    std::string node;                   // the controller's snvme node
    std::uint32_t num_io_queues = 64;
    // Queue depth: the driver creates user queues with the controller's
    // depth (DevInfo::queue_depth); the rings are sized for that.
    bool rings_in_gpu_memory = false;   // rings in HBM (the drive DMAs CQEs into HBM)
    std::uint32_t nsid = 1;
    std::uint64_t namespace_bytes = 0;  // 0: unknown
    std::uint32_t max_command_bytes = 1u << 20;  // largest command issued (<= MDTS)
    int cuda_device = -1;               // -1: current device
};

class SnvmeController final : public NvmeController {
public:
    static Result<std::unique_ptr<SnvmeController>> create(const SnvmeControllerConfig& cfg,
                                                           SnvmeSys& sys = linux_snvme_sys());
    // The same, keeping `sys` (e.g. a fake driver) alive as long as the controller.
    static Result<std::unique_ptr<SnvmeController>> create(const SnvmeControllerConfig& cfg,
                                                           std::shared_ptr<SnvmeSys> sys);
    ~SnvmeController() override;

    const ControllerInfo& info() const override { return info_; }
    QueuePairView device_queue(std::uint32_t i) const override;
    QueuePairView host_queue(std::uint32_t i) const override;
    Result<DmaMapping> map_dma(void* ptr, std::uint64_t bytes) override;
    Status unmap_dma(const DmaMapping& m) override;
    // The driver deletes and creates queue pairs per group only; a queue that
    // timed out cannot be reset alone, and its lease is retired.
    Status reset_queue(std::uint32_t i) override;
    // The counters of the drive behind a fake driver; a real drive reports none here.
    ControllerStats stats() const override {
        EmulatedNvmeController* d = sys_->emulated_drive();
        return d ? d->stats() : ControllerStats{};
    }
    EmulatedNvmeController* emulated_drive() override { return sys_->emulated_drive(); }

    std::uint32_t groups() const { return static_cast<std::uint32_t>(clients_.size()); }

private:
    SnvmeController() = default;
    Status bring_up(const SnvmeControllerConfig& cfg);

    std::shared_ptr<SnvmeSys> sys_owner_;  // declared first: released after everything below
    SnvmeSys* sys_ = nullptr;
    ControllerInfo info_;
    int cuda_device_ = -1;
    std::vector<std::unique_ptr<SnvmeClient>> clients_;  // one open file (and queue group) each
    std::vector<std::uint32_t> group_of_client_;
    HostMappedBuffer host_rings_;
    void* device_rings_raw_ = nullptr;
    std::vector<QueuePairView> device_views_, host_views_;
    std::mutex map_mu_;
};

}  // namespace nvme
}  // namespace tutti
