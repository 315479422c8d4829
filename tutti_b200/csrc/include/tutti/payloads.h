#pragma once
// Resolver <-> DataPath private payload for file-backed NVMe targets.
//
// A file resolves to an ordered list of extents mapping the file's logical
// bytes to byte offsets on a namespace of one controller (for a RAID0 member,
// the member's controller). The DataPath turns namespace bytes into LBAs at
// submit time. Parity: reference payloads/ext4_local_nvme/payload.h:76-141
// (extents, namespace identity, RAID0 layout, recommended DataPath key).

#include <cstdint>
#include <string>
#include <vector>

namespace tutti {

constexpr char kFileExtentPayloadType[] = "tutti.file-extents";
constexpr std::uint32_t kFileExtentPayloadVersion = 1;

struct FileExtent {
    std::uint64_t logical;   // byte offset in the file
    std::uint64_t physical;  // byte offset on the device (namespace) `device`
    std::uint64_t length;    // bytes
    std::uint32_t device;    // index into the DataPath's device table
    std::uint32_t flags;
};

struct FileExtentPayload {
    std::string path;
    std::uint64_t file_size = 0;
    std::uint64_t st_dev = 0;
    std::uint64_t st_ino = 0;
    // Identity of the backing namespace (PCI BDF + nsid on real hardware; the
    // emulated controller name otherwise).
    std::string controller;
    std::uint32_t nsid = 1;
    std::uint32_t block_bytes = 512;
    // How the extents were obtained: "fiemap" (physical blocks of the block
    // device) or "synthetic" (a private namespace range assigned per file for
    // emulated controllers on filesystems without FIEMAP).
    std::string mapping;
    std::vector<FileExtent> extents;  // sorted by logical, non-overlapping
};

}  // namespace tutti
