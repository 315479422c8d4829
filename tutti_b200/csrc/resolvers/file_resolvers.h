#pragma once
// File resolvers: URI ("file:///abs/path" or "/abs/path") -> FileExtentPayload.
//
//  * LocalFileResolver   one mount bound to one device. Extents come from
//    FS_IOC_FIEMAP with FIEMAP_FLAG_SYNC (reference
//    csrc/resolvers/local_file/resolver.h:147-440: O_DIRECT open, fsync, reject
//    unwritten/delalloc/unknown/encoded/shared extents, merge adjacent extents,
//    cap the extent count, verify the backing device), or, where the
//    filesystem has no FIEMAP (tmpfs) or the binding asks for it, from a
//    synthetic per-file namespace range that an emulated controller backs with
//    the file itself.
//  * MultiMountResolver  longest-prefix dispatch over several mounts
//    (reference multi_mount_resolver.h:35).
//  * Raid0Resolver       an md RAID0 mount: FIEMAP offsets on the md device are
//    translated to member-device offsets with the geometry probed from
//    /sys/block/<md>/md (reference raid0_resolver.h:20-87, common/md_raid0.h).

#include <cstdint>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include <tutti/payloads.h>
#include <tutti/spi/resolver.h>

namespace tutti {

struct MountBinding {
    std::string mount_path;               // absolute directory prefix
    std::uint32_t device_index = 0;       // DataPath device-table row
    std::string controller;               // backing controller identity
    std::uint32_t nsid = 1;
    std::uint32_t block_bytes = 512;
    std::uint64_t namespace_base_bytes = 0;  // partition start within the namespace
    std::uint64_t expected_st_dev = 0;    // 0: not checked
    std::string mapping = "auto";         // "fiemap" | "synthetic" | "auto"
    std::string datapath_key = "nvme-gpu";
    // The device-side file handle is a binary-searched extent array of any
    // length, so the cap only guards against pathological fragmentation (the
    // reference's fixed-size handle capped it at 124).
    std::uint32_t max_extents = 65536;
};

// Raw FIEMAP walk (exposed for tests and the RAID0 resolver).
struct RawExtent {
    std::uint64_t logical, physical, length;
    std::uint32_t flags;
};
Result<std::vector<RawExtent>> fiemap_extents(int fd, std::uint64_t size, bool sync);

// Flags that make an extent unusable for direct device IO.
bool fiemap_extent_rejected(std::uint32_t flags);

std::string uri_to_path(std::string_view uri);

class LocalFileResolver : public StorageTargetResolver {
public:
    explicit LocalFileResolver(MountBinding binding);
    Result<ResolvedTarget> resolve(std::string_view uri, const ResolveOptions& options) override;
    const MountBinding& binding() const { return binding_; }

    // Builds the payload without wrapping it (RAID0 reuses it).
    Result<std::shared_ptr<FileExtentPayload>> build_payload(const std::string& path);

private:
    MountBinding binding_;
};

class MultiMountResolver : public StorageTargetResolver {
public:
    Status add(std::unique_ptr<StorageTargetResolver> resolver, std::string mount_path);
    Result<ResolvedTarget> resolve(std::string_view uri, const ResolveOptions& options) override;
    std::size_t size() const { return mounts_.size(); }

private:
    std::vector<std::pair<std::string, std::unique_ptr<StorageTargetResolver>>> mounts_;
};

struct Raid0Member {
    std::uint32_t device_index = 0;
    std::uint64_t data_offset_bytes = 0;  // member offset of md byte 0 of this member
    std::string name;
};

struct Raid0Geometry {
    std::uint64_t chunk_bytes = 0;
    std::vector<Raid0Member> members;  // in raid slot order
};

// Probes <sysfs_root>/block/<md>/md: level must be raid0; chunk_size; raid_disks;
// rd<N>/{slot,offset} -> members in slot order. `sysfs_root` is "/sys" normally.
Result<Raid0Geometry> probe_md_raid0(const std::string& sysfs_root, const std::string& md_name);
// The md array (e.g. "md0") whose block device holds `path`'s filesystem:
// st_dev -> <sysfs_root>/dev/block/MAJ:MIN -> that device's name, which must
// have an md/ directory. Lets a raid0 resolver find its array from the mount.
Result<std::string> find_md_array(const std::string& sysfs_root, const std::string& path);

// md byte offset -> (member index, member byte offset).
struct Raid0Location {
    std::uint32_t member;
    std::uint64_t offset;
    std::uint64_t contiguous;  // bytes until the chunk boundary
};
Raid0Location raid0_map(const Raid0Geometry& g, std::uint64_t md_offset);

class Raid0Resolver : public StorageTargetResolver {
public:
    Raid0Resolver(MountBinding md_binding, Raid0Geometry geometry,
                  std::vector<std::string> member_controllers);
    Result<ResolvedTarget> resolve(std::string_view uri, const ResolveOptions& options) override;

private:
    LocalFileResolver base_;
    Raid0Geometry geo_;
    std::vector<std::string> member_controllers_;
};

}  // namespace tutti
