#include "host_admin.h"

#include <dirent.h>
#include <fcntl.h>
#include <spawn.h>
#include <sys/mount.h>
#include <sys/stat.h>
#include <sys/sysmacros.h>
#include <sys/wait.h>
#include <unistd.h>

#include <algorithm>
#include <cctype>
#include <cerrno>
#include <chrono>
#include <cstring>
#include <fstream>
#include <sstream>
#include <thread>

extern char** environ;

namespace tutti {
namespace daemon {

namespace {

class LinuxHostSys final : public HostSys {
public:
    bool read_text(const std::string& path, std::string* out) override {
        std::ifstream f(path);
        if (!f) return false;
        std::stringstream ss;
        ss << f.rdbuf();
        *out = ss.str();
        return true;
    }
    long read_at(const std::string& path, std::uint64_t off, void* buf, std::size_t n) override {
        const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
        if (fd < 0) return -errno;
        const ssize_t r = ::pread(fd, buf, n, static_cast<off_t>(off));
        const long out = r < 0 ? -errno : static_cast<long>(r);
        ::close(fd);
        return out;
    }
    int mount(const std::string& source, const std::string& target, const std::string& fs_type) override {
        return ::mount(source.c_str(), target.c_str(), fs_type.c_str(), 0, nullptr) == 0 ? 0 : -errno;
    }
    int unmount(const std::string& target) override { return ::umount2(target.c_str(), 0) == 0 ? 0 : -errno; }
    int make_dirs(const std::string& path) override {
        std::string cur;
        std::stringstream ss(path);
        std::string part;
        if (!path.empty() && path[0] == '/') cur = "/";
        while (std::getline(ss, part, '/')) {
            if (part.empty()) continue;
            cur += (cur.empty() || cur.back() == '/' ? "" : "/") + part;
            if (::mkdir(cur.c_str(), 0755) != 0 && errno != EEXIST) return -errno;
        }
        return 0;
    }
    int run(const std::vector<std::string>& argv) override {
        if (argv.empty()) return -1;
        std::vector<char*> args;
        for (const auto& a : argv) args.push_back(const_cast<char*>(a.c_str()));
        args.push_back(nullptr);
        pid_t pid = 0;
        if (posix_spawnp(&pid, args[0], nullptr, nullptr, args.data(), environ) != 0) return -1;
        int status = 0;
        while (::waitpid(pid, &status, 0) < 0) {
            if (errno != EINTR) return -1;
        }
        return WIFEXITED(status) ? WEXITSTATUS(status) : -1;
    }
    std::vector<std::string> list_dir(const std::string& path) override {
        std::vector<std::string> out;
        DIR* d = ::opendir(path.c_str());
        if (!d) return out;
        while (dirent* e = ::readdir(d)) {
            if (std::strcmp(e->d_name, ".") && std::strcmp(e->d_name, "..")) out.emplace_back(e->d_name);
        }
        ::closedir(d);
        return out;
    }
    bool read_link(const std::string& path, std::string* out) override {
        char buf[4096];
        const ssize_t n = ::readlink(path.c_str(), buf, sizeof(buf) - 1);
        if (n < 0) return false;
        out->assign(buf, static_cast<std::size_t>(n));
        return true;
    }
    int make_symlink(const std::string& target, const std::string& link) override {
        return ::symlink(target.c_str(), link.c_str()) == 0 ? 0 : -errno;
    }
    int remove_file(const std::string& path) override { return ::unlink(path.c_str()) == 0 ? 0 : -errno; }
    bool device_numbers(const std::string& path, unsigned* major, unsigned* minor) override {
        struct stat st {};
        if (::stat(path.c_str(), &st) != 0 || !S_ISBLK(st.st_mode)) return false;
        *major = ::major(st.st_rdev);
        *minor = ::minor(st.st_rdev);
        return true;
    }
    void sleep_ms(std::uint32_t ms) override { std::this_thread::sleep_for(std::chrono::milliseconds(ms)); }
};

std::string trim(const std::string& s) {
    std::size_t a = 0, b = s.size();
    while (a < b && std::isspace(static_cast<unsigned char>(s[a]))) ++a;
    while (b > a && std::isspace(static_cast<unsigned char>(s[b - 1]))) --b;
    return s.substr(a, b - a);
}

// Mount points in mountinfo escape space, tab, newline and backslash as \ooo.
std::string unescape_octal(const std::string& s) {
    std::string out;
    for (std::size_t i = 0; i < s.size(); ++i) {
        if (s[i] == '\\' && i + 3 < s.size() && std::isdigit(static_cast<unsigned char>(s[i + 1])) &&
            std::isdigit(static_cast<unsigned char>(s[i + 2])) && std::isdigit(static_cast<unsigned char>(s[i + 3]))) {
            out.push_back(static_cast<char>((s[i + 1] - '0') * 64 + (s[i + 2] - '0') * 8 + (s[i + 3] - '0')));
            i += 3;
        } else {
            out.push_back(s[i]);
        }
    }
    return out;
}

std::string base_name(const std::string& p) {
    const auto k = p.find_last_of('/');
    return k == std::string::npos ? p : p.substr(k + 1);
}

bool under(const std::string& path, const std::string& mount_path) {
    if (path == mount_path) return true;
    const std::string prefix = mount_path.back() == '/' ? mount_path : mount_path + "/";
    return path.compare(0, prefix.size(), prefix) == 0;
}

bool all_digits(const std::string& s) {
    return !s.empty() && std::all_of(s.begin(), s.end(), [](char c) { return c >= '0' && c <= '9'; });
}

}  // namespace

HostSys& linux_host_sys() {
    static LinuxHostSys sys;
    return sys;
}

std::vector<MountEntry> parse_mountinfo(const std::string& text) {
    // "<id> <parent> <major>:<minor> <root> <mount point> <options> [optional...] - <fs> <source> <super options>"
    std::vector<MountEntry> out;
    std::istringstream lines(text);
    std::string line;
    while (std::getline(lines, line)) {
        std::istringstream f(line);
        std::vector<std::string> tok;
        std::string t;
        while (f >> t) tok.push_back(t);
        auto sep = std::find(tok.begin(), tok.end(), "-");
        if (tok.size() < 7 || sep == tok.end() || sep - tok.begin() < 6 || tok.end() - sep < 3) continue;
        MountEntry e;
        const std::string& dev = tok[2];
        const auto colon = dev.find(':');
        if (colon == std::string::npos) continue;
        e.major = static_cast<unsigned>(std::strtoul(dev.substr(0, colon).c_str(), nullptr, 10));
        e.minor = static_cast<unsigned>(std::strtoul(dev.substr(colon + 1).c_str(), nullptr, 10));
        e.mount_point = unescape_octal(tok[4]);
        e.fs_type = *(sep + 1);
        e.source = unescape_octal(*(sep + 2));
        out.push_back(std::move(e));
    }
    return out;
}

std::string detect_filesystem(HostSys& sys, const std::string& block_device) {
    unsigned char head[2048];
    const long n = sys.read_at(block_device, 0, head, sizeof(head));
    if (n < 4) return "";
    if (std::memcmp(head, "XFSB", 4) == 0) return "xfs";  // XFS superblock at byte 0 (big-endian magic)
    // ext2/3/4: superblock at byte 1024, s_magic (little-endian 0xEF53) at offset 0x38 in it
    if (n >= 1024 + 0x3A && head[1024 + 0x38] == 0x53 && head[1024 + 0x39] == 0xEF) return "ext4";
    return "";
}

bool MountManager::lookup(const std::string& mount_path, MountEntry* out) {
    std::string text;
    if (!sys_.read_text("/proc/self/mountinfo", &text)) return false;
    const auto entries = parse_mountinfo(text);
    // the last entry for a path is the one visible (mounts stack)
    for (auto it = entries.rbegin(); it != entries.rend(); ++it)
        if (it->mount_point == mount_path) {
            *out = *it;
            return true;
        }
    return false;
}

MountOutcome MountManager::mount(const std::string& block_device, const std::string& mount_path) {
    MountOutcome r;
    MountEntry cur;
    const std::string fs = detect_filesystem(sys_, block_device);
    if (lookup(mount_path, &cur)) {
        unsigned ma = 0, mi = 0;
        const bool same_device = sys_.device_numbers(block_device, &ma, &mi) && ma == cur.major && mi == cur.minor;
        const bool same_fs = fs.empty() || cur.fs_type == fs || (fs == "ext4" && cur.fs_type.rfind("ext", 0) == 0);
        if (!same_device || !same_fs) {
            r.error = mount_path + " is already a mount of " + cur.source + " (" + cur.fs_type + "), not " + block_device;
            return r;
        }
        r.already_mounted = true;  // adopted: never unmounted by the daemon
        r.fs_type = cur.fs_type;
        return r;
    }
    if (fs.empty()) {
        r.error = "no ext4 or XFS superblock on " + block_device;
        return r;
    }
    if (int rc = sys_.make_dirs(mount_path); rc != 0) {
        r.error = "cannot create " + mount_path + ": " + std::strerror(-rc);
        return r;
    }
    if (int rc = sys_.mount(block_device, mount_path, fs); rc != 0) {
        r.error = "mount " + block_device + " on " + mount_path + " (" + fs + "): " + std::strerror(-rc);
        return r;
    }
    r.mounted_by_daemon = true;
    r.fs_type = fs;
    owned_.push_back({block_device, mount_path});
    return r;
}

std::vector<MountHolder> MountManager::holders(const std::string& mount_path) {
    std::vector<MountHolder> out;
    for (const std::string& pid_s : sys_.list_dir("/proc")) {
        if (!all_digits(pid_s)) continue;
        const std::string base = "/proc/" + pid_s;
        std::string comm;
        sys_.read_text(base + "/comm", &comm);
        comm = trim(comm);
        const std::int64_t pid = std::strtoll(pid_s.c_str(), nullptr, 10);
        auto add = [&](const char* how, const std::string& detail) { out.push_back({pid, comm, how, detail}); };
        std::string link;
        for (const char* what : {"cwd", "root", "exe"})
            if (sys_.read_link(base + "/" + what, &link) && under(link, mount_path) &&
                !(std::strcmp(what, "root") == 0 && link == "/"))
                add(what, link);
        for (const std::string& fd : sys_.list_dir(base + "/fd"))
            if (sys_.read_link(base + "/fd/" + fd, &link) && under(link, mount_path)) add("fd", "fd " + fd + " " + link);
        std::string maps;
        if (sys_.read_text(base + "/maps", &maps)) {
            std::istringstream ls(maps);
            std::string line, last;
            while (std::getline(ls, line)) {
                const auto slash = line.find('/');
                if (slash == std::string::npos) continue;
                const std::string path = line.substr(slash);
                if (path != last && under(path, mount_path)) add("map", path);
                last = path;
            }
        }
    }
    return out;
}

int MountManager::unmount_all(std::vector<std::string>* report) {
    int busy = 0;
    for (auto it = owned_.rbegin(); it != owned_.rend();) {
        bool done = false;
        for (std::uint32_t attempt = 0; attempt <= retry_max_; ++attempt) {
            const int rc = sys_.unmount(it->path);
            if (rc == 0) {
                done = true;
                break;
            }
            if (rc != -EBUSY) {
                if (report) report->push_back("umount " + it->path + ": " + std::strerror(-rc));
                break;
            }
            if (report) {
                report->push_back(it->path + " is busy (attempt " + std::to_string(attempt + 1) + ")");
                for (const MountHolder& h : holders(it->path))
                    report->push_back("  held by pid " + std::to_string(h.pid) + " (" + h.comm + "): " + h.how + " " +
                                      h.detail);
            }
            if (force_exit_.load() || attempt == retry_max_) break;
            sys_.sleep_ms(retry_interval_ms_);
            if (force_exit_.load()) break;
        }
        if (done) {
            it = decltype(it)(owned_.erase(std::next(it).base()));
        } else {
            ++busy;
            ++it;
        }
    }
    return busy;
}

std::vector<std::string> MountManager::owned_mounts() const {
    std::vector<std::string> out;
    for (const auto& o : owned_) out.push_back(o.path);
    return out;
}

std::string MountManager::md_holder(const std::string& member) {
    for (const std::string& h : sys_.list_dir("/sys/class/block/" + base_name(member) + "/holders"))
        if (h.rfind("md", 0) == 0) return h;
    return "";
}

Result<std::string> MountManager::assemble_raid0(const std::string& name, const std::vector<std::string>& members) {
    using R = Result<std::string>;
    if (members.size() < 2) return R::Failure({StatusCode::INVALID_ARGUMENT, "raid0 array " + name + " needs two or more members"});
    (void)sys_.run({"udevadm", "settle", "--timeout=10"});  // udev may be assembling it right now
    auto common = [&](std::string* holder) {
        *holder = md_holder(members.front());
        for (const auto& m : members)
            if (md_holder(m) != *holder) return false;
        return true;
    };
    std::string holder;
    if (!common(&holder)) return R::Failure({StatusCode::INVALID_ARGUMENT, "members of " + name + " belong to different md arrays"});
    if (!holder.empty()) {
        std::string state;
        sys_.read_text("/sys/block/" + holder + "/md/array_state", &state);
        if (trim(state) == "inactive") {  // a partial incremental assembly: start over
            (void)sys_.run({"mdadm", "--stop", "/dev/" + holder});
            holder.clear();
        }
    }
    bool assembled = false;
    if (holder.empty()) {
        std::vector<std::string> argv = {"mdadm", "--assemble", "/dev/md/" + name, "--run"};
        argv.insert(argv.end(), members.begin(), members.end());
        const int rc = sys_.run(argv);
        (void)sys_.run({"udevadm", "settle", "--timeout=10"});
        if (rc != 0 || !common(&holder) || holder.empty())
            return R::Failure({StatusCode::NOT_FOUND, "mdadm --assemble of " + name + " failed (status " + std::to_string(rc) +
                                                          "); an array is created once by an operator, never here"});
        assembled = true;
    }
    std::string level, disks;
    sys_.read_text("/sys/block/" + holder + "/md/level", &level);
    sys_.read_text("/sys/block/" + holder + "/md/raid_disks", &disks);
    if (trim(level) != "raid0" || trim(disks) != std::to_string(members.size())) {
        if (assembled) (void)sys_.run({"mdadm", "--stop", "/dev/" + holder});
        return R::Failure({StatusCode::INVALID_ARGUMENT, "/dev/" + holder + " is " + trim(level) + " over " + trim(disks) +
                                                             " disks, not raid0 over these " + std::to_string(members.size())});
    }
    if (assembled) arrays_.push_back("/dev/" + holder);
    return R("/dev/" + holder);
}

int MountManager::stop_arrays() {
    int failed = 0;
    for (auto it = arrays_.rbegin(); it != arrays_.rend(); ++it)
        if (sys_.run({"mdadm", "--stop", *it}) != 0) ++failed;
    arrays_.clear();
    return failed;
}

Status build_view_root(HostSys& sys, const std::string& view_root,
                       const std::vector<std::pair<std::string, std::string>>& links) {
    if (view_root.empty()) return {StatusCode::INVALID_ARGUMENT, "empty view root"};
    if (int rc = sys.make_dirs(view_root); rc != 0)
        return {StatusCode::PERMISSION_DENIED, "cannot create " + view_root + ": " + std::strerror(-rc)};
    for (const auto& kv : links) {
        if (kv.first.empty() || kv.first.find('/') != std::string::npos)
            return {StatusCode::INVALID_ARGUMENT, "bad view entry name '" + kv.first + "'"};
        const std::string link = view_root + "/" + kv.first;
        std::string cur;
        if (sys.read_link(link, &cur)) {
            if (cur == kv.second) continue;
            (void)sys.remove_file(link);
        }
        if (int rc = sys.make_symlink(kv.second, link); rc != 0)
            return {StatusCode::INTERNAL, "cannot link " + link + ": " + std::strerror(-rc)};
    }
    return Status::Ok();
}

}  // namespace daemon
}  // namespace tutti
