#pragma once
// The character-device interface of the snvme queue-leasing kernel driver, as
// its user-space clients see it (ABI version 2).
//
// The driver binds an NVMe controller away from the stock nvme driver and lets
// processes lease I/O queue pairs whose rings live in their own memory (host or
// GPU). Two device nodes:
//   * the control node (owner only): bind/unbind a PCI function, create/remove
//     the per-controller node;
//   * the per-controller node: device info (with the ABI handshake), one queue
//     group per open file, user queue pairs inside that group, DMA mappings of
//     ring and data buffers. Closing the file releases everything it created.
//
// Every structure below crosses the user/kernel boundary, so its size and field
// offsets are the driver's, fixed by static_asserts; the ioctl numbers encode
// the structure sizes. Only fixed-width fields (LP64 only).
//
// Interface parity: kernel_modules/snvme/include/uapi/tutti_snvme.h of the
// reference (the same numbers and layouts; this header is written for C++
// clients of that driver).

#include <cstddef>
#include <cstdint>

#include <sys/ioctl.h>

namespace tutti {
namespace snvme {
namespace uapi {

constexpr std::uint32_t kAbiVersion = 2;

// Capability bits reported in DevInfo::capabilities.
constexpr std::uint32_t kCapQueueGroups = 1u << 0;   // CREATE/DESTROY_QUEUE_GROUP
constexpr std::uint32_t kCapUserQueues = 1u << 1;    // ADD_USER_QUEUE
constexpr std::uint32_t kCapRawAdmin = 1u << 2;      // RAW_ADMIN_CMD
constexpr std::uint32_t kCapKernelIoqCap = 1u << 3;  // SET_KERNEL_IOQ_CAP
constexpr std::uint32_t kCapMapKindTag = 1u << 4;    // MapRequest::kind is honoured
// What a queue-leasing client needs from the driver.
constexpr std::uint32_t kClientCaps = kCapQueueGroups | kCapUserQueues | kCapMapKindTag;

constexpr unsigned kDevIoctlType = 0x80;   // per-controller node
constexpr unsigned kCtrlIoctlType = 0x90;  // control node
constexpr std::uint32_t kMaxGroupsPerFile = 1;
constexpr std::uint32_t kMaxQueuesPerGroup = 32;
constexpr std::uint32_t kMaxOwnerPartitions = 8;
constexpr std::size_t kDiskNameBytes = 32;

// Page granularity of the map ioctls: host memory is pinned in CPU pages,
// GPU memory in the GPU's 64 KiB pages.
constexpr std::uint64_t kHostMapPage = 4096;
constexpr std::uint64_t kDeviceMapPage = 64 * 1024;

enum MapKind : std::uint8_t {
    kMapUnspecified = 0,  // pre-tag clients
    kMapRingSq = 1,       // an I/O submission ring (group-scoped)
    kMapRingCq = 2,       // an I/O completion ring (group-scoped)
    kMapData = 3,         // a PRP/SGL data buffer (file-scoped)
};

// MAP_*_MEMORY argument. The driver pins n_pages pages from vaddr and writes
// one bus address per page into the user array at `ioaddrs`.
struct MapRequest {
    std::uint64_t vaddr;
    std::uint64_t n_pages;
    std::uint64_t ioaddrs;      // user address of std::uint64_t[n_pages]
    std::int32_t legacy_queue;  // -1 (queue-group clients)
    std::int32_t legacy_is_cq;  // -1 (queue-group clients)
    std::uint32_t group_id;     // required for ring kinds
    std::uint8_t kind;          // MapKind
    std::uint8_t mbz[3];
};
static_assert(sizeof(MapRequest) == 40, "MapRequest size");
static_assert(offsetof(MapRequest, n_pages) == 8, "MapRequest.n_pages");
static_assert(offsetof(MapRequest, ioaddrs) == 16, "MapRequest.ioaddrs");
static_assert(offsetof(MapRequest, legacy_queue) == 24, "MapRequest.legacy_queue");
static_assert(offsetof(MapRequest, group_id) == 32, "MapRequest.group_id");
static_assert(offsetof(MapRequest, kind) == 36, "MapRequest.kind");

// GET_DEV_INFO result.
struct DevInfo {
    std::uint32_t legacy_user_queues;
    std::uint32_t first_user_qid;      // lowest QID handed to user queues
    std::uint8_t doorbell_stride_log;  // CAP.DSTRD
    std::uint8_t pad0[7];
    std::uint64_t max_transfer_bytes;  // MDTS in bytes
    std::uint64_t lba_bytes;           // namespace logical block size
    char disk_name[kDiskNameBytes];
    std::uint16_t queue_depth;         // CAP.MQES + 1 (clamped by the driver)
    std::uint16_t mbz0;
    std::uint32_t bar0_bytes;
    std::uint32_t last_user_qid;       // highest QID handed to user queues
    std::uint32_t max_queues_per_group;
    std::uint32_t sgl_support;         // Identify Controller SGLS
    std::uint32_t abi_version;         // 0: a driver older than the handshake
    std::uint32_t capabilities;
    std::uint32_t mbz1[3];
};
static_assert(sizeof(DevInfo) == 104, "DevInfo size");
static_assert(offsetof(DevInfo, first_user_qid) == 4, "DevInfo.first_user_qid");
static_assert(offsetof(DevInfo, doorbell_stride_log) == 8, "DevInfo.doorbell_stride_log");
static_assert(offsetof(DevInfo, max_transfer_bytes) == 16, "DevInfo.max_transfer_bytes");
static_assert(offsetof(DevInfo, lba_bytes) == 24, "DevInfo.lba_bytes");
static_assert(offsetof(DevInfo, disk_name) == 32, "DevInfo.disk_name");
static_assert(offsetof(DevInfo, queue_depth) == 64, "DevInfo.queue_depth");
static_assert(offsetof(DevInfo, bar0_bytes) == 68, "DevInfo.bar0_bytes");
static_assert(offsetof(DevInfo, last_user_qid) == 72, "DevInfo.last_user_qid");
static_assert(offsetof(DevInfo, max_queues_per_group) == 76, "DevInfo.max_queues_per_group");
static_assert(offsetof(DevInfo, sgl_support) == 80, "DevInfo.sgl_support");
static_assert(offsetof(DevInfo, abi_version) == 84, "DevInfo.abi_version");
static_assert(offsetof(DevInfo, capabilities) == 88, "DevInfo.capabilities");

// Owner-side queue budget (SET_IOQ_NUM).
struct OwnerPartition {
    std::uint32_t owner_id;
    std::uint32_t count;
    std::int32_t numa_node;
    std::uint32_t mbz;
};
static_assert(sizeof(OwnerPartition) == 16, "OwnerPartition size");

struct QueueBudget {
    std::uint32_t user_queues;
    std::uint32_t flags;  // bit 0: queues on host memory
    std::uint32_t kernel_queue_cap;
    std::uint32_t write_queues;
    std::uint32_t poll_queues;
    std::uint32_t partitions;
    std::uint32_t mbz[2];
    OwnerPartition partition[kMaxOwnerPartitions];
};
static_assert(sizeof(QueueBudget) == 160, "QueueBudget size");
static_assert(offsetof(QueueBudget, kernel_queue_cap) == 8, "QueueBudget.kernel_queue_cap");
static_assert(offsetof(QueueBudget, partitions) == 20, "QueueBudget.partitions");
static_assert(offsetof(QueueBudget, partition) == 32, "QueueBudget.partition");

// PCI function for the control node's bind/unbind/create/remove.
struct PciAddress {
    std::int32_t domain;
    std::int32_t bus;
    std::int32_t slot;
    std::int32_t function;
};
static_assert(sizeof(PciAddress) == 16, "PciAddress size");

// RAW_ADMIN_CMD: one admin SQE in, the CQE's result out.
struct RawAdmin {
    std::uint8_t sqe[64];
    std::uint32_t result_dw0;
    std::uint32_t result_dw1;
    std::uint16_t status;  // CQE DW3[31:17]
    std::uint16_t mbz0;
    std::uint32_t mbz1[4];
};
static_assert(sizeof(RawAdmin) == 92, "RawAdmin size");
static_assert(offsetof(RawAdmin, result_dw0) == 64, "RawAdmin.result_dw0");
static_assert(offsetof(RawAdmin, status) == 72, "RawAdmin.status");

// CREATE_QUEUE_GROUP: the driver fills group_id and max_queues.
struct QueueGroup {
    std::uint32_t group_id;
    std::uint32_t flags;  // MBZ
    std::uint32_t max_queues;
    std::uint32_t mbz[5];
};
static_assert(sizeof(QueueGroup) == 32, "QueueGroup size");
static_assert(offsetof(QueueGroup, max_queues) == 8, "QueueGroup.max_queues");

struct QueueRings {
    std::uint64_t sq_vaddr;  // mapped before as kMapRingSq in the group
    std::uint64_t cq_vaddr;  // mapped before as kMapRingCq in the group
};
static_assert(sizeof(QueueRings) == 16, "QueueRings size");

struct QueueDoorbells {
    std::uint32_t sq_tail_offset;  // byte offset of the SQ tail doorbell in BAR0
    std::uint32_t cq_head_offset;  // byte offset of the CQ head doorbell in BAR0
    std::uint32_t qid;
    std::uint32_t mbz;
};
static_assert(sizeof(QueueDoorbells) == 16, "QueueDoorbells size");

// ADD_USER_QUEUE: creates nr_pairs I/O queue pairs (CQ, then SQ) on the
// controller over the given rings.
struct AddUserQueues {
    std::uint32_t group_id;
    std::uint32_t nr_pairs;  // 1..kMaxQueuesPerGroup
    std::uint32_t flags;     // MBZ
    std::uint32_t mbz[5];
    QueueRings rings[kMaxQueuesPerGroup];
    QueueDoorbells out[kMaxQueuesPerGroup];
};
static_assert(sizeof(AddUserQueues) == 1056, "AddUserQueues size");
static_assert(offsetof(AddUserQueues, nr_pairs) == 4, "AddUserQueues.nr_pairs");
static_assert(offsetof(AddUserQueues, rings) == 32, "AddUserQueues.rings");
static_assert(offsetof(AddUserQueues, out) == 544, "AddUserQueues.out");

// Per-controller node.
constexpr unsigned long kMapHostMemory = _IOW(kDevIoctlType, 1, MapRequest);
constexpr unsigned long kMapDeviceMemory = _IOW(kDevIoctlType, 2, MapRequest);
constexpr unsigned long kMapDeviceQueueMemory = _IOW(kDevIoctlType, 3, MapRequest);
constexpr unsigned long kUnmapHostMemory = _IOW(kDevIoctlType, 4, std::uint64_t);
constexpr unsigned long kUnmapDeviceMemory = _IOW(kDevIoctlType, 5, std::uint64_t);
constexpr unsigned long kUnmapDeviceQueueMemory = _IOW(kDevIoctlType, 6, std::uint64_t);
constexpr unsigned long kSetIoqNum = _IOW(kDevIoctlType, 7, QueueBudget);
constexpr unsigned long kSetShareReg = _IOW(kDevIoctlType, 8, DevInfo);
constexpr unsigned long kGetDevInfo = _IOR(kDevIoctlType, 9, DevInfo);
constexpr unsigned long kClearIoqNum = _IOW(kDevIoctlType, 10, DevInfo);
constexpr unsigned long kRawAdminCmd = _IOWR(kDevIoctlType, 11, RawAdmin);
constexpr unsigned long kCreateQueueGroup = _IOWR(kDevIoctlType, 12, QueueGroup);
constexpr unsigned long kDestroyQueueGroup = _IOW(kDevIoctlType, 13, std::uint32_t);
constexpr unsigned long kAddUserQueue = _IOWR(kDevIoctlType, 14, AddUserQueues);
constexpr unsigned long kSetKernelIoqCap = _IOW(kDevIoctlType, 15, std::uint32_t);

// Control node.
constexpr unsigned long kDeviceBind = _IOW(kCtrlIoctlType, 1, PciAddress);
constexpr unsigned long kDeviceUnbind = _IOW(kCtrlIoctlType, 2, PciAddress);
constexpr unsigned long kChrdevCreate = _IOWR(kCtrlIoctlType, 3, PciAddress);
constexpr unsigned long kChrdevRemove = _IOW(kCtrlIoctlType, 4, PciAddress);

}  // namespace uapi
}  // namespace snvme
}  // namespace tutti
