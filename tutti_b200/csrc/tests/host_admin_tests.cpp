// Tests of the daemon's host administration (mounts, md RAID0 arrays,
// accelerator view roots) against a fake host: mountinfo text, sysfs
// entries, block-device bytes and a log of the commands run.
//
// Parity: reference tests/device_manager/nvmeservice/nvmeservice_phase3_contract_test.cpp
// (mount adoption and ownership, EBUSY retries with holder reports, RAID0
// assembly and adoption).

#include <cerrno>
#include <map>

#include "harness.h"

#include "../daemon/host_admin.h"

namespace tutti {
namespace native_tests {

using daemon::HostSys;
using daemon::MountManager;

namespace {

struct FakeHost final : HostSys {
    std::map<std::string, std::string> files;                  // path -> text or bytes
    std::map<std::string, std::string> links;                  // path -> target
    std::map<std::string, std::vector<std::string>> dirs;     // path -> entries
    std::map<std::string, std::pair<unsigned, unsigned>> blk;  // device node -> major:minor
    struct Mounted {
        std::string source, target, fs;
        unsigned major, minor;
    };
    std::vector<Mounted> mounts;
    std::map<std::string, int> busy;  // target -> EBUSY answers left
    std::vector<std::string> made_dirs;
    std::vector<std::vector<std::string>> ran;
    std::map<std::string, int> run_status;  // argv[0] + " " + argv[1] -> exit status
    std::function<void(const std::vector<std::string>&)> on_run;
    int sleeps = 0;
    std::function<void()> on_sleep;

    bool read_text(const std::string& path, std::string* out) override {
        if (path == "/proc/self/mountinfo") {
            std::string t;
            int id = 20;
            for (const auto& m : mounts) {
                std::string mp;
                for (char c : m.target) mp += c == ' ' ? std::string("\\040") : std::string(1, c);
                t += std::to_string(id++) + " 1 " + std::to_string(m.major) + ":" + std::to_string(m.minor) + " / " + mp +
                     " rw,relatime shared:1 - " + m.fs + " " + m.source + " rw\n";
            }
            *out = t;
            return true;
        }
        auto it = files.find(path);
        if (it == files.end()) return false;
        *out = it->second;
        return true;
    }
    long read_at(const std::string& path, std::uint64_t off, void* buf, std::size_t n) override {
        auto it = files.find(path);
        if (it == files.end()) return -ENOENT;
        if (off >= it->second.size()) return 0;
        const std::size_t k = std::min<std::size_t>(n, it->second.size() - off);
        std::memcpy(buf, it->second.data() + off, k);
        return static_cast<long>(k);
    }
    int mount(const std::string& source, const std::string& target, const std::string& fs) override {
        auto b = blk.find(source);
        if (b == blk.end()) return -ENODEV;
        mounts.push_back({source, target, fs, b->second.first, b->second.second});
        return 0;
    }
    int unmount(const std::string& target) override {
        if (busy[target] > 0) {
            --busy[target];
            return -EBUSY;
        }
        for (auto it = mounts.rbegin(); it != mounts.rend(); ++it)
            if (it->target == target) {
                mounts.erase(std::next(it).base());
                return 0;
            }
        return -EINVAL;
    }
    int make_dirs(const std::string& path) override {
        made_dirs.push_back(path);
        return 0;
    }
    int run(const std::vector<std::string>& argv) override {
        ran.push_back(argv);
        if (on_run) on_run(argv);
        auto it = run_status.find(argv[0] + (argv.size() > 1 ? " " + argv[1] : ""));
        return it == run_status.end() ? 0 : it->second;
    }
    std::vector<std::string> list_dir(const std::string& path) override {
        auto it = dirs.find(path);
        return it == dirs.end() ? std::vector<std::string>{} : it->second;
    }
    bool read_link(const std::string& path, std::string* out) override {
        auto it = links.find(path);
        if (it == links.end()) return false;
        *out = it->second;
        return true;
    }
    int make_symlink(const std::string& target, const std::string& link) override {
        if (links.count(link)) return -EEXIST;
        links[link] = target;
        return 0;
    }
    int remove_file(const std::string& path) override { return links.erase(path) ? 0 : -ENOENT; }
    bool device_numbers(const std::string& path, unsigned* ma, unsigned* mi) override {
        auto b = blk.find(path);
        if (b == blk.end()) return false;
        *ma = b->second.first;
        *mi = b->second.second;
        return true;
    }
    void sleep_ms(std::uint32_t) override {
        ++sleeps;
        if (on_sleep) on_sleep();
    }

    void ext4_disk(const std::string& dev, unsigned ma, unsigned mi) {
        std::string sb(2048, '\0');
        sb[1024 + 0x38] = '\x53';
        sb[1024 + 0x39] = '\xEF';
        files[dev] = sb;
        blk[dev] = {ma, mi};
    }
    void xfs_disk(const std::string& dev, unsigned ma, unsigned mi) {
        std::string sb(2048, '\0');
        sb.replace(0, 4, "XFSB");
        files[dev] = sb;
        blk[dev] = {ma, mi};
    }
    bool was_run(const std::string& a0, const std::string& a1) const {
        for (const auto& r : ran)
            if (r.size() > 1 && r[0] == a0 && r[1] == a1) return true;
        return false;
    }
};

}  // namespace

TEST(host_mountinfo_parser_reads_devices_types_and_escaped_paths) {
    const std::string text =
        "36 35 98:0 /mnt1 /mnt/parent rw,noatime master:1 - ext3 /dev/root rw,errors=continue\n"
        "40 36 259:3 / /mnt/kv\\040store rw,relatime shared:7 shared:9 - xfs /dev/nvme1n1 rw,attr2\n"
        "41 36 0:52 / /proc rw - proc proc rw\n"
        "garbage line\n";
    const auto e = daemon::parse_mountinfo(text);
    CHECK(e.size() == 3);
    CHECK(e[0].major == 98 && e[0].minor == 0 && e[0].fs_type == "ext3" && e[0].source == "/dev/root");
    CHECK(e[1].mount_point == "/mnt/kv store" && e[1].fs_type == "xfs" && e[1].major == 259 && e[1].minor == 3);
    CHECK(e[2].mount_point == "/proc" && e[2].fs_type == "proc");
}

TEST(host_filesystem_is_read_from_the_superblock) {
    FakeHost h;
    h.ext4_disk("/dev/a", 259, 1);
    h.xfs_disk("/dev/b", 259, 2);
    h.files["/dev/c"] = std::string(4096, '\0');
    CHECK(daemon::detect_filesystem(h, "/dev/a") == "ext4");
    CHECK(daemon::detect_filesystem(h, "/dev/b") == "xfs");
    CHECK(daemon::detect_filesystem(h, "/dev/c").empty());
    CHECK(daemon::detect_filesystem(h, "/dev/missing").empty());
}

TEST(host_mount_owns_what_it_mounts_and_adopts_what_it_finds) {
    FakeHost h;
    h.ext4_disk("/dev/nvme0n1", 259, 0);
    h.xfs_disk("/dev/nvme1n1", 259, 1);
    h.ext4_disk("/dev/nvme2n1", 259, 2);
    h.mounts.push_back({"/dev/nvme1n1", "/mnt/nvme1", "xfs", 259, 1});  // up before the daemon
    MountManager m(h, 10, 3);
    auto a = m.mount("/dev/nvme0n1", "/mnt/nvme0");
    CHECK(a.error.empty() && a.mounted_by_daemon && a.fs_type == "ext4");
    CHECK(!h.made_dirs.empty() && h.made_dirs.back() == "/mnt/nvme0");
    auto b = m.mount("/dev/nvme1n1", "/mnt/nvme1");
    CHECK(b.error.empty() && b.already_mounted && !b.mounted_by_daemon);
    // the path holds another device: refused, nothing changed
    auto c = m.mount("/dev/nvme2n1", "/mnt/nvme1");
    CHECK(!c.error.empty() && c.error.find("already a mount") != std::string::npos);
    // a device without a file system
    h.files["/dev/nvme3n1"] = std::string(4096, '\0');
    h.blk["/dev/nvme3n1"] = {259, 3};
    CHECK(!m.mount("/dev/nvme3n1", "/mnt/nvme3").error.empty());
    CHECK(m.owned_mounts() == std::vector<std::string>{"/mnt/nvme0"});
    // shutdown unmounts only its own mount
    CHECK(m.unmount_all() == 0);
    CHECK(h.mounts.size() == 1 && h.mounts[0].target == "/mnt/nvme1");
}

TEST(host_busy_unmount_is_retried_and_reports_its_holders) {
    FakeHost h;
    h.ext4_disk("/dev/nvme0n1", 259, 0);
    MountManager m(h, 5, 4);
    CHECK(m.mount("/dev/nvme0n1", "/mnt/kv").mounted_by_daemon);
    h.busy["/mnt/kv"] = 2;  // busy twice, then free
    h.dirs["/proc"] = {"1", "4242", "self", "77"};
    h.files["/proc/4242/comm"] = "vllm-worker\n";
    h.dirs["/proc/4242/fd"] = {"0", "7"};
    h.links["/proc/4242/fd/7"] = "/mnt/kv/r0/segments/3.seg";
    h.links["/proc/4242/cwd"] = "/mnt/kv/r0";
    h.files["/proc/77/comm"] = "bash";
    h.files["/proc/77/maps"] = "7f00-7f10 r--p 00000000 103:02 12 /mnt/kv/lib.so\n7f10-7f20 r--p 0 0:0 0 /usr/lib/x.so\n";
    h.links["/proc/77/root"] = "/";
    std::vector<std::string> report;
    CHECK(m.unmount_all(&report) == 0);
    CHECK(h.sleeps == 2 && h.mounts.empty());
    bool fd = false, cwd = false, map = false;
    for (const auto& l : report) {
        fd |= l.find("pid 4242 (vllm-worker): fd fd 7 /mnt/kv/r0/segments/3.seg") != std::string::npos;
        cwd |= l.find("pid 4242 (vllm-worker): cwd /mnt/kv/r0") != std::string::npos;
        map |= l.find("pid 77 (bash): map /mnt/kv/lib.so") != std::string::npos;
    }
    CHECK(fd && cwd && map);
}

TEST(host_unmount_gives_up_after_its_retries_or_a_second_stop) {
    FakeHost h;
    h.ext4_disk("/dev/nvme0n1", 259, 0);
    h.ext4_disk("/dev/nvme1n1", 259, 1);
    MountManager m(h, 5, 3);
    CHECK(m.mount("/dev/nvme0n1", "/mnt/a").mounted_by_daemon);
    CHECK(m.mount("/dev/nvme1n1", "/mnt/b").mounted_by_daemon);
    h.busy["/mnt/a"] = 100;
    h.busy["/mnt/b"] = 100;
    CHECK(m.unmount_all() == 2);  // 4 attempts each, 3 sleeps each
    CHECK(h.sleeps == 6 && h.mounts.size() == 2);
    // a second stop request during the retries ends them at once
    h.sleeps = 0;
    h.on_sleep = [&] { m.request_force_exit(); };
    CHECK(m.unmount_all() == 2);
    CHECK(h.sleeps == 1);
    // once free, the next call unmounts both
    h.busy.clear();
    CHECK(m.unmount_all() == 0 && h.mounts.empty());
}

TEST(host_raid0_is_assembled_from_its_members_or_adopted) {
    FakeHost h;
    // mdadm --assemble makes md127 the holder of both members
    h.on_run = [&](const std::vector<std::string>& a) {
        if (a.size() > 2 && a[0] == "mdadm" && a[1] == "--assemble") {
            h.dirs["/sys/class/block/nvme0n1/holders"] = {"md127"};
            h.dirs["/sys/class/block/nvme1n1/holders"] = {"md127"};
            h.files["/sys/block/md127/md/level"] = "raid0\n";
            h.files["/sys/block/md127/md/raid_disks"] = "2\n";
            h.files["/sys/block/md127/md/array_state"] = "clean\n";
        }
    };
    MountManager m(h);
    auto dev = m.assemble_raid0("kv", {"/dev/nvme0n1", "/dev/nvme1n1"});
    CHECK(dev.ok() && dev.value() == "/dev/md127");
    CHECK(h.was_run("mdadm", "--assemble") && h.was_run("udevadm", "settle"));
    bool named = false;
    for (const auto& r : h.ran) named |= r.size() > 2 && r[1] == "--assemble" && r[2] == "/dev/md/kv";
    CHECK(named);
    CHECK(m.stop_arrays() == 0 && h.was_run("mdadm", "--stop"));
    // already assembled by udev: adopted, and not stopped at shutdown
    FakeHost h2 = FakeHost();
    h2.dirs["/sys/class/block/nvme0n1/holders"] = {"md5"};
    h2.dirs["/sys/class/block/nvme1n1/holders"] = {"md5"};
    h2.files["/sys/block/md5/md/level"] = "raid0";
    h2.files["/sys/block/md5/md/raid_disks"] = "2";
    h2.files["/sys/block/md5/md/array_state"] = "clean";
    MountManager m2(h2);
    auto d2 = m2.assemble_raid0("kv", {"/dev/nvme0n1", "/dev/nvme1n1"});
    CHECK(d2.ok() && d2.value() == "/dev/md5" && !h2.was_run("mdadm", "--assemble"));
    CHECK(m2.stop_arrays() == 0 && !h2.was_run("mdadm", "--stop"));
}

TEST(host_raid0_refuses_mixed_members_other_levels_and_failed_assembly) {
    FakeHost h;
    h.dirs["/sys/class/block/nvme0n1/holders"] = {"md1"};
    h.dirs["/sys/class/block/nvme1n1/holders"] = {"md2"};
    MountManager m(h);
    auto mixed = m.assemble_raid0("kv", {"/dev/nvme0n1", "/dev/nvme1n1"});
    CHECK(!mixed.ok() && mixed.status().message().find("different md arrays") != std::string::npos);
    CHECK(!m.assemble_raid0("kv", {"/dev/nvme0n1"}).ok());  // one member
    // an inactive partial assembly is stopped, then the assembly fails
    FakeHost h2;
    h2.dirs["/sys/class/block/nvme0n1/holders"] = {"md9"};
    h2.dirs["/sys/class/block/nvme1n1/holders"] = {"md9"};
    h2.files["/sys/block/md9/md/array_state"] = "inactive\n";
    h2.on_run = [&](const std::vector<std::string>& a) {
        if (a.size() > 1 && a[1] == "--stop") {
            h2.dirs.erase("/sys/class/block/nvme0n1/holders");
            h2.dirs.erase("/sys/class/block/nvme1n1/holders");
        }
    };
    h2.run_status["mdadm --assemble"] = 1;
    MountManager m2(h2);
    auto failed = m2.assemble_raid0("kv", {"/dev/nvme0n1", "/dev/nvme1n1"});
    CHECK(!failed.ok() && failed.status().message().find("never here") != std::string::npos);
    CHECK(h2.was_run("mdadm", "--stop"));
    // a raid1 array over the members is not accepted
    FakeHost h3;
    h3.dirs["/sys/class/block/nvme0n1/holders"] = {"md3"};
    h3.dirs["/sys/class/block/nvme1n1/holders"] = {"md3"};
    h3.files["/sys/block/md3/md/level"] = "raid1";
    h3.files["/sys/block/md3/md/raid_disks"] = "2";
    MountManager m3(h3);
    CHECK(!m3.assemble_raid0("kv", {"/dev/nvme0n1", "/dev/nvme1n1"}).ok());
}

TEST(host_view_root_links_each_allowed_drive_and_keeps_other_entries) {
    FakeHost h;
    h.links["/run/tutti/gpu0/nvme1"] = "/old/place";  // stale
    h.links["/run/tutti/gpu0/notes"] = "/elsewhere";  // not ours
    CHECK(daemon::build_view_root(h, "/run/tutti/gpu0", {{"nvme0", "/mnt/nvme0"}, {"nvme1", "/mnt/nvme1"}}).ok());
    CHECK(h.links["/run/tutti/gpu0/nvme0"] == "/mnt/nvme0");
    CHECK(h.links["/run/tutti/gpu0/nvme1"] == "/mnt/nvme1");
    CHECK(h.links["/run/tutti/gpu0/notes"] == "/elsewhere");
    CHECK(!daemon::build_view_root(h, "/run/tutti/gpu0", {{"../x", "/mnt"}}).ok());
    CHECK(!daemon::build_view_root(h, "", {}).ok());
}

}  // namespace native_tests
}  // namespace tutti
