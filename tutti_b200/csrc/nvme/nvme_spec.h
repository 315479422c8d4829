#pragma once
// NVMe submission/completion entry formats, written from the NVMe Base
// Specification (command dword layout, CQE status field, PRP rules). Shared by
// host code (emulated controller, host submitter, tests) and device code (the
// GPU io kernel), so it is plain C++ with __host__ __device__ helpers.

#include <cstdint>

#if defined(__CUDACC__)
#define TUTTI_HD __host__ __device__ __forceinline__
#else
#define TUTTI_HD inline
#endif

namespace tutti {
namespace nvme {

// I/O command set opcodes used here.
constexpr std::uint8_t kOpFlush = 0x00;
constexpr std::uint8_t kOpWrite = 0x01;
constexpr std::uint8_t kOpRead = 0x02;

// Generic command status values (status code type 0).
constexpr std::uint16_t kScSuccess = 0x00;
constexpr std::uint16_t kScInvalidOpcode = 0x01;
constexpr std::uint16_t kScInvalidField = 0x02;
constexpr std::uint16_t kScDataTransferError = 0x04;
constexpr std::uint16_t kScInternalError = 0x06;
constexpr std::uint16_t kScInvalidNamespace = 0x0B;
constexpr std::uint16_t kScLbaOutOfRange = 0x80;
// Media error type (SCT 2): unrecovered read error.
constexpr std::uint16_t kSctMedia = 0x2;
constexpr std::uint16_t kScUnrecoveredRead = 0x81;

constexpr std::uint32_t kMemoryPageBytes = 4096;  // CC.MPS = 0

// 64-byte submission queue entry.
struct alignas(64) Sqe {
    std::uint32_t cdw0;   // [7:0] opcode, [9:8] fuse, [15:14] psdt, [31:16] cid
    std::uint32_t nsid;
    std::uint32_t cdw2;
    std::uint32_t cdw3;
    std::uint64_t mptr;
    std::uint64_t prp1;
    std::uint64_t prp2;
    std::uint32_t cdw10;  // SLBA[31:0]
    std::uint32_t cdw11;  // SLBA[63:32]
    std::uint32_t cdw12;  // [15:0] NLB (0-based)
    std::uint32_t cdw13;
    std::uint32_t cdw14;
    std::uint32_t cdw15;
};
static_assert(sizeof(Sqe) == 64, "SQE is 64 bytes");

// 16-byte completion queue entry.
struct alignas(16) Cqe {
    std::uint32_t dw0;
    std::uint32_t dw1;
    std::uint32_t dw2;  // [15:0] SQ head pointer, [31:16] SQ identifier
    std::uint32_t dw3;  // [15:0] CID, [16] phase, [31:17] status field
};
static_assert(sizeof(Cqe) == 16, "CQE is 16 bytes");

TUTTI_HD std::uint8_t sqe_opcode(const Sqe& s) { return static_cast<std::uint8_t>(s.cdw0 & 0xFFu); }
TUTTI_HD std::uint16_t sqe_cid(const Sqe& s) { return static_cast<std::uint16_t>(s.cdw0 >> 16); }
TUTTI_HD std::uint64_t sqe_slba(const Sqe& s) {
    return (static_cast<std::uint64_t>(s.cdw11) << 32) | s.cdw10;
}
TUTTI_HD std::uint32_t sqe_nlb(const Sqe& s) { return (s.cdw12 & 0xFFFFu) + 1u; }

TUTTI_HD void build_rw_sqe(Sqe& s, std::uint8_t opcode, std::uint16_t cid, std::uint32_t nsid,
                           std::uint64_t slba, std::uint32_t nblocks, std::uint64_t prp1,
                           std::uint64_t prp2) {
    s.cdw0 = static_cast<std::uint32_t>(opcode) | (static_cast<std::uint32_t>(cid) << 16);
    s.nsid = nsid;
    s.cdw2 = 0;
    s.cdw3 = 0;
    s.mptr = 0;
    s.prp1 = prp1;
    s.prp2 = prp2;
    s.cdw10 = static_cast<std::uint32_t>(slba);
    s.cdw11 = static_cast<std::uint32_t>(slba >> 32);
    s.cdw12 = (nblocks - 1u) & 0xFFFFu;
    s.cdw13 = 0;
    s.cdw14 = 0;
    s.cdw15 = 0;
}

// Status field (SF) = dw3[31:17]: [0] ... here sf bits: SC [7:0], SCT [10:8], CRD, M, DNR.
TUTTI_HD std::uint16_t cqe_cid(std::uint32_t dw3) { return static_cast<std::uint16_t>(dw3 & 0xFFFFu); }
TUTTI_HD std::uint32_t cqe_phase(std::uint32_t dw3) { return (dw3 >> 16) & 1u; }
TUTTI_HD std::uint32_t cqe_status(std::uint32_t dw3) { return dw3 >> 17; }  // 0 == success
TUTTI_HD std::uint32_t make_status(std::uint16_t sct, std::uint16_t sc) {
    return (static_cast<std::uint32_t>(sct & 0x7u) << 8) | (sc & 0xFFu);
}
TUTTI_HD std::uint32_t make_cqe_dw3(std::uint16_t cid, std::uint32_t phase, std::uint32_t status) {
    return static_cast<std::uint32_t>(cid) | ((phase & 1u) << 16) | (status << 17);
}

// Number of PRP-list entries a transfer of `bytes` starting at page offset
// `first_page_offset` needs beyond PRP1 (0: PRP2 unused; 1: PRP2 is a page).
TUTTI_HD std::uint32_t prp_extra_pages(std::uint64_t first_page_offset, std::uint64_t bytes) {
    std::uint64_t first = kMemoryPageBytes - first_page_offset;
    if (bytes <= first) return 0;
    return static_cast<std::uint32_t>((bytes - first + kMemoryPageBytes - 1) / kMemoryPageBytes);
}

// Controller register file as seen by a submitter: doorbells with CAP.DSTRD = 0
// start at 0x1000; SQ y tail at 0x1000 + 8y, CQ y head at 0x1000 + 8y + 4.
constexpr std::uint32_t kDoorbellBase = 0x1000;
TUTTI_HD std::uint32_t sq_doorbell_offset(std::uint32_t qid) { return kDoorbellBase + 8u * qid; }
TUTTI_HD std::uint32_t cq_doorbell_offset(std::uint32_t qid) { return kDoorbellBase + 8u * qid + 4u; }

}  // namespace nvme
}  // namespace tutti
