#pragma once
// Host administration of the device-manager daemon: file systems on the
// drives, md RAID0 arrays over them, and per-accelerator views of the mounts.
//
//   * MountManager::mount: mounts a drive's block device (ext4 or XFS, read
//     from the superblock) at its mount path, or adopts a mount that is
//     already there when it is the same device and file system. Only mounts
//     the daemon made itself are unmounted at shutdown.
//   * MountManager::unmount_all: unmounts in reverse order; a busy mount
//     (EBUSY) is retried `retry_max` times `retry_interval_ms` apart, and each
//     time the processes holding it (open files, mapped files, working or
//     root directories under it) are reported. A second stop request ends
//     the retries and leaves the busy mounts in place.
//   * MountManager::assemble_raid0: brings up an existing md RAID0 array over
//     the member drives (mdadm --assemble), or adopts the one udev already
//     assembled from exactly those members; an inactive partial assembly is
//     stopped and assembled again. It never creates an array (that erases
//     the members) and stops, at shutdown, only arrays it assembled itself.
//   * build_view_root: the directory an accelerator's processes open the
//     drives through: one link per drive it may use, to the drive's mount.
//
// Every OS call goes through HostSys, so the tests run it against a fake
// host (mountinfo text, sysfs entries, block-device bytes, a command log).
// Parity: reference nvmeservice/src/mount_manager.h:79 (MountManager:
// mount_one, adopt, unmount_all with EBUSY holder reports and force exit,
// assemble_raid0, stop_arrays) and the accelerator view roots of its config.

#include <atomic>
#include <cstdint>
#include <string>
#include <vector>

#include <tutti/status.h>

namespace tutti {
namespace daemon {

class HostSys {
public:
    virtual ~HostSys() = default;
    virtual bool read_text(const std::string& path, std::string* out) = 0;
    // Reads `n` bytes at `off` of a file or block device; bytes read or -errno.
    virtual long read_at(const std::string& path, std::uint64_t off, void* buf, std::size_t n) = 0;
    virtual int mount(const std::string& source, const std::string& target, const std::string& fs_type) = 0;
    virtual int unmount(const std::string& target) = 0;  // 0 or -errno
    virtual int make_dirs(const std::string& path) = 0;  // 0 or -errno
    virtual int run(const std::vector<std::string>& argv) = 0;  // exit status (-1: could not run)
    virtual std::vector<std::string> list_dir(const std::string& path) = 0;
    virtual bool read_link(const std::string& path, std::string* out) = 0;
    virtual int make_symlink(const std::string& target, const std::string& link) = 0;
    virtual int remove_file(const std::string& path) = 0;
    // st_rdev of a block device node.
    virtual bool device_numbers(const std::string& path, unsigned* major, unsigned* minor) = 0;
    virtual void sleep_ms(std::uint32_t ms) = 0;
};

HostSys& linux_host_sys();

// One line of /proc/self/mountinfo.
struct MountEntry {
    std::string mount_point;
    std::string fs_type;
    std::string source;
    unsigned major = 0, minor = 0;
};
std::vector<MountEntry> parse_mountinfo(const std::string& text);

// "ext4" (the ext2/3/4 superblock magic; the ext4 driver mounts all three),
// "xfs", or "" when neither superblock is found.
std::string detect_filesystem(HostSys& sys, const std::string& block_device);

struct MountHolder {
    std::int64_t pid = 0;
    std::string comm;
    std::string how;     // "fd", "map", "cwd", "root", "exe"
    std::string detail;  // the path found under the mount
};

struct MountOutcome {
    bool mounted_by_daemon = false;
    bool already_mounted = false;
    std::string fs_type;
    std::string error;  // non-empty: not mounted
};

class MountManager {
public:
    explicit MountManager(HostSys& sys, std::uint32_t retry_interval_ms = 1000, std::uint32_t retry_max = 30)
        : sys_(sys), retry_interval_ms_(retry_interval_ms), retry_max_(retry_max) {}

    MountOutcome mount(const std::string& block_device, const std::string& mount_path);
    // Unmounts the daemon's own mounts; returns how many are still mounted
    // (busy), with one line per report in *report.
    int unmount_all(std::vector<std::string>* report = nullptr);
    std::vector<MountHolder> holders(const std::string& mount_path);
    bool lookup(const std::string& mount_path, MountEntry* out);

    // Returns the array's device node (/dev/mdN).
    Result<std::string> assemble_raid0(const std::string& name, const std::vector<std::string>& members);
    int stop_arrays();  // arrays this manager assembled; returns how many failed to stop

    void request_force_exit() { force_exit_.store(true); }
    bool force_exit_requested() const { return force_exit_.load(); }
    std::vector<std::string> owned_mounts() const;

private:
    std::string md_holder(const std::string& member);
    HostSys& sys_;
    std::uint32_t retry_interval_ms_, retry_max_;
    struct Owned {
        std::string device, path;
    };
    std::vector<Owned> owned_;
    std::vector<std::string> arrays_;
    std::atomic<bool> force_exit_{false};
};

// Makes `view_root` hold exactly one link per (name, target) pair, replacing
// links of those names; other entries of the directory are left alone.
Status build_view_root(HostSys& sys, const std::string& view_root,
                       const std::vector<std::pair<std::string, std::string>>& links);

}  // namespace daemon
}  // namespace tutti
