#include "file_resolvers.h"

#include <fcntl.h>
#include <linux/fiemap.h>
#include <linux/fs.h>
#include <sys/ioctl.h>
#include <sys/stat.h>
#include <sys/sysmacros.h>
#include <unistd.h>

#include <algorithm>
#include <climits>
#include <cerrno>
#include <cstring>
#include <cstdio>

namespace tutti {

std::string uri_to_path(std::string_view uri) {
    constexpr std::string_view kFile = "file://";
    if (uri.substr(0, kFile.size()) == kFile) uri.remove_prefix(kFile.size());
    return std::string(uri);
}

bool fiemap_extent_rejected(std::uint32_t f) {
    const std::uint32_t bad = FIEMAP_EXTENT_UNKNOWN | FIEMAP_EXTENT_DELALLOC | FIEMAP_EXTENT_ENCODED |
                              FIEMAP_EXTENT_DATA_ENCRYPTED | FIEMAP_EXTENT_NOT_ALIGNED |
                              FIEMAP_EXTENT_DATA_INLINE | FIEMAP_EXTENT_DATA_TAIL |
                              FIEMAP_EXTENT_UNWRITTEN | FIEMAP_EXTENT_SHARED;
    return (f & bad) != 0;
}

Result<std::vector<RawExtent>> fiemap_extents(int fd, std::uint64_t size, bool sync) {
    using R = Result<std::vector<RawExtent>>;
    std::vector<RawExtent> out;
    constexpr std::uint32_t kBatch = 256;
    std::vector<char> buf(sizeof(struct fiemap) + kBatch * sizeof(struct fiemap_extent));
    std::uint64_t start = 0;
    while (start < size) {
        std::memset(buf.data(), 0, buf.size());
        auto* fm = reinterpret_cast<struct fiemap*>(buf.data());
        fm->fm_start = start;
        fm->fm_length = size - start;
        fm->fm_flags = sync ? FIEMAP_FLAG_SYNC : 0;
        fm->fm_extent_count = kBatch;
        if (ioctl(fd, FS_IOC_FIEMAP, fm) != 0)
            return R::Failure({errno == EOPNOTSUPP || errno == ENOTTY ? StatusCode::UNSUPPORTED
                                                                      : StatusCode::INTERNAL,
                               std::string("FIEMAP failed: ") + std::strerror(errno)});
        if (fm->fm_mapped_extents == 0) break;
        bool last = false;
        for (std::uint32_t i = 0; i < fm->fm_mapped_extents; ++i) {
            const auto& e = fm->fm_extents[i];
            out.push_back({e.fe_logical, e.fe_physical, e.fe_length, e.fe_flags});
            start = e.fe_logical + e.fe_length;
            if (e.fe_flags & FIEMAP_EXTENT_LAST) last = true;
        }
        if (last) break;
    }
    return out;
}

namespace {

// Process-wide synthetic namespace ranges, per controller identity.
struct SyntheticSpace {
    std::mutex mu;
    std::map<std::string, std::uint64_t> next;  // controller -> bump pointer
    std::map<std::tuple<std::string, std::uint64_t, std::uint64_t>, std::pair<std::uint64_t, std::uint64_t>>
        files;  // (controller, dev, ino) -> (base, capacity)
};
SyntheticSpace& synthetic_space() {
    static SyntheticSpace s;
    return s;
}

std::uint64_t synthetic_base(const std::string& ctrl, std::uint64_t dev, std::uint64_t ino, std::uint64_t size) {
    auto& s = synthetic_space();
    std::lock_guard<std::mutex> g(s.mu);
    auto key = std::make_tuple(ctrl, dev, ino);
    auto it = s.files.find(key);
    if (it != s.files.end() && it->second.second >= size) return it->second.first;
    const std::uint64_t align = 1ull << 20;
    std::uint64_t cap = std::max<std::uint64_t>(align, (size + align - 1) & ~(align - 1));
    std::uint64_t& bump = s.next[ctrl];
    if (bump == 0) bump = align;  // keep namespace byte 0 unused
    std::uint64_t base = bump;
    bump += cap;
    s.files[key] = {base, cap};
    return base;
}

}  // namespace

LocalFileResolver::LocalFileResolver(MountBinding b) : binding_(std::move(b)) {}

Result<std::shared_ptr<FileExtentPayload>> LocalFileResolver::build_payload(const std::string& path) {
    using R = Result<std::shared_ptr<FileExtentPayload>>;
    int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd < 0) return R::Failure({StatusCode::NOT_FOUND, "cannot open " + path + ": " + std::strerror(errno)});
    struct stat st {};
    if (fstat(fd, &st) != 0 || !S_ISREG(st.st_mode)) {
        ::close(fd);
        return R::Failure({StatusCode::INVALID_ARGUMENT, "not a regular file: " + path});
    }
    if (binding_.expected_st_dev != 0 && static_cast<std::uint64_t>(st.st_dev) != binding_.expected_st_dev) {
        ::close(fd);
        return R::Failure({StatusCode::INVALID_ARGUMENT, "file is not on the bound device: " + path});
    }
    auto p = std::make_shared<FileExtentPayload>();
    p->path = path;
    p->file_size = static_cast<std::uint64_t>(st.st_size);
    p->st_dev = static_cast<std::uint64_t>(st.st_dev);
    p->st_ino = static_cast<std::uint64_t>(st.st_ino);
    p->controller = binding_.controller;
    p->nsid = binding_.nsid;
    p->block_bytes = binding_.block_bytes;

    bool use_fiemap = binding_.mapping != "synthetic";
    if (use_fiemap) {
        ::fsync(fd);
        auto ex = fiemap_extents(fd, p->file_size, true);
        if (!ex.ok()) {
            if (binding_.mapping == "fiemap") {
                ::close(fd);
                return R::Failure(ex.status());
            }
            use_fiemap = false;  // auto: filesystem without FIEMAP
        } else {
            std::vector<FileExtent> merged;
            for (const auto& e : ex.value()) {
                if (fiemap_extent_rejected(e.flags)) {
                    ::close(fd);
                    return R::Failure({StatusCode::UNSUPPORTED,
                                       "extent not usable for device IO (flags " + std::to_string(e.flags) +
                                           ") in " + path});
                }
                if ((e.physical % binding_.block_bytes) || (e.logical % binding_.block_bytes)) {
                    ::close(fd);
                    return R::Failure({StatusCode::UNSUPPORTED, "extent not block aligned in " + path});
                }
                std::uint64_t phys = e.physical + binding_.namespace_base_bytes;
                if (!merged.empty() && merged.back().logical + merged.back().length == e.logical &&
                    merged.back().physical + merged.back().length == phys)
                    merged.back().length += e.length;
                else
                    merged.push_back({e.logical, phys, e.length, binding_.device_index, 0});
            }
            std::uint64_t covered = 0;
            for (auto& m : merged) {
                if (m.logical != covered) {
                    ::close(fd);
                    return R::Failure({StatusCode::UNSUPPORTED, "file has holes: " + path});
                }
                covered += m.length;
            }
            if (covered < p->file_size) {
                ::close(fd);
                return R::Failure({StatusCode::UNSUPPORTED, "file not fully allocated: " + path});
            }
            if (merged.size() > binding_.max_extents) {
                ::close(fd);
                return R::Failure({StatusCode::RESOURCE_EXHAUSTED,
                                   "file has " + std::to_string(merged.size()) + " extents (max " +
                                       std::to_string(binding_.max_extents) + "): " + path});
            }
            p->mapping = "fiemap";
            p->extents = std::move(merged);
        }
    }
    if (!use_fiemap) {
        std::uint64_t base = synthetic_base(binding_.controller, p->st_dev, p->st_ino, p->file_size);
        p->mapping = "synthetic";
        p->extents = {{0, base, p->file_size, binding_.device_index, 0}};
    }
    ::close(fd);
    return p;
}

Result<ResolvedTarget> LocalFileResolver::resolve(std::string_view uri, const ResolveOptions&) {
    std::string path = uri_to_path(uri);
    if (path.empty() || path[0] != '/')
        return Result<ResolvedTarget>::Failure({StatusCode::INVALID_ARGUMENT, "path must be absolute"});
    if (!binding_.mount_path.empty()) {
        // A resolver serves the files of its mount only; compare canonical paths
        // so that ".." or a symlink cannot step outside it.
        char real_file[PATH_MAX], real_mount[PATH_MAX];
        if (!::realpath(path.c_str(), real_file))
            return Result<ResolvedTarget>::Failure({StatusCode::NOT_FOUND, "cannot resolve " + path});
        const std::string mount = ::realpath(binding_.mount_path.c_str(), real_mount) ? std::string(real_mount)
                                                                                      : binding_.mount_path;
        const std::string file(real_file);
        if (file.compare(0, mount.size(), mount) != 0 || (file.size() > mount.size() && mount != "/" &&
                                                          file[mount.size()] != '/'))
            return Result<ResolvedTarget>::Failure(
                {StatusCode::INVALID_ARGUMENT, path + " is outside the mount " + binding_.mount_path});
    }
    auto p = build_payload(path);
    if (!p.ok()) return Result<ResolvedTarget>::Failure(p.status());
    std::uint64_t size = p.value()->file_size;
    return ResolvedTarget::make<FileExtentPayload>("tutti.local-file", kFileExtentPayloadType,
                                                   kFileExtentPayloadVersion, size, binding_.datapath_key,
                                                   std::string(uri), p.value());
}

Status MultiMountResolver::add(std::unique_ptr<StorageTargetResolver> r, std::string mount) {
    if (!r) return {StatusCode::INVALID_ARGUMENT, "null resolver"};
    while (mount.size() > 1 && mount.back() == '/') mount.pop_back();
    for (auto& m : mounts_)
        if (m.first == mount) return {StatusCode::INVALID_ARGUMENT, "duplicate mount " + mount};
    mounts_.emplace_back(std::move(mount), std::move(r));
    std::sort(mounts_.begin(), mounts_.end(),
              [](const auto& a, const auto& b) { return a.first.size() > b.first.size(); });
    return Status::Ok();
}

Result<ResolvedTarget> MultiMountResolver::resolve(std::string_view uri, const ResolveOptions& o) {
    std::string path = uri_to_path(uri);
    for (auto& m : mounts_) {
        const std::string& pre = m.first;
        if (path.compare(0, pre.size(), pre) == 0 && (path.size() == pre.size() || path[pre.size()] == '/'))
            return m.second->resolve(uri, o);
    }
    return Result<ResolvedTarget>::Failure({StatusCode::NOT_FOUND, "no mount covers " + path});
}

namespace {
bool read_sysfs(const std::string& p, std::string& out) {
    std::FILE* f = std::fopen(p.c_str(), "r");
    if (!f) return false;
    char buf[256];
    const bool ok = std::fgets(buf, sizeof(buf), f) != nullptr;
    std::fclose(f);
    if (!ok) return false;
    out = buf;
    while (!out.empty() && (out.back() == '\n' || out.back() == ' ')) out.pop_back();
    return true;
}
}  // namespace

Result<Raid0Geometry> probe_md_raid0(const std::string& sysfs_root, const std::string& md) {
    using R = Result<Raid0Geometry>;
    const std::string base = sysfs_root + "/block/" + md + "/md/";
    std::string level, chunk, disks;
    if (!read_sysfs(base + "level", level)) return R::Failure({StatusCode::NOT_FOUND, "no md level for " + md});
    if (level != "raid0") return R::Failure({StatusCode::UNSUPPORTED, md + " is " + level + ", not raid0"});
    if (!read_sysfs(base + "chunk_size", chunk) || !read_sysfs(base + "raid_disks", disks))
        return R::Failure({StatusCode::NOT_FOUND, "incomplete md sysfs for " + md});
    Raid0Geometry g;
    g.chunk_bytes = std::stoull(chunk);
    std::uint32_t n = static_cast<std::uint32_t>(std::stoul(disks));
    if (g.chunk_bytes == 0 || n == 0) return R::Failure({StatusCode::INVALID_ARGUMENT, "bad md geometry"});
    g.members.resize(n);
    std::vector<bool> seen(n, false);
    for (std::uint32_t i = 0; i < n; ++i) {
        std::string slot, off;
        const std::string rd = base + "rd" + std::to_string(i) + "/";
        if (!read_sysfs(rd + "slot", slot) || !read_sysfs(rd + "offset", off))
            return R::Failure({StatusCode::NOT_FOUND, "missing md member rd" + std::to_string(i)});
        std::uint32_t s = static_cast<std::uint32_t>(std::stoul(slot));
        if (s >= n || seen[s]) return R::Failure({StatusCode::INVALID_ARGUMENT, "bad md slot"});
        seen[s] = true;
        g.members[s].data_offset_bytes = std::stoull(off) * 512ull;  // sectors
        g.members[s].device_index = s;
        g.members[s].name = "rd" + std::to_string(i);
    }
    return g;
}

Result<std::string> find_md_array(const std::string& sysfs_root, const std::string& path) {
    using R = Result<std::string>;
    struct stat st {};
    if (::stat(path.c_str(), &st) != 0) return R::Failure({StatusCode::NOT_FOUND, "stat " + path + " failed"});
    const std::string link = sysfs_root + "/dev/block/" + std::to_string(major(st.st_dev)) + ":" +
                             std::to_string(minor(st.st_dev));
    char buf[4096];
    const ssize_t n = ::readlink(link.c_str(), buf, sizeof(buf) - 1);
    if (n <= 0) return R::Failure({StatusCode::NOT_FOUND, "no block device entry " + link + " for " + path});
    std::string target(buf, static_cast<std::size_t>(n));
    const std::string name = target.substr(target.find_last_of('/') + 1);
    struct stat md {};
    if (::stat((sysfs_root + "/block/" + name + "/md").c_str(), &md) != 0)
        return R::Failure({StatusCode::NOT_FOUND, path + " is on " + name + ", not on an md array"});
    return name;
}

Raid0Location raid0_map(const Raid0Geometry& g, std::uint64_t md_offset) {
    const std::uint64_t n = g.members.size();
    const std::uint64_t chunk = md_offset / g.chunk_bytes;
    const std::uint64_t within = md_offset % g.chunk_bytes;
    Raid0Location loc;
    loc.member = static_cast<std::uint32_t>(chunk % n);
    loc.offset = g.members[loc.member].data_offset_bytes + (chunk / n) * g.chunk_bytes + within;
    loc.contiguous = g.chunk_bytes - within;
    return loc;
}

Raid0Resolver::Raid0Resolver(MountBinding md, Raid0Geometry geo, std::vector<std::string> ctrls)
    : base_([&] {
          md.mapping = "fiemap";
          return md;
      }()),
      geo_(std::move(geo)),
      member_controllers_(std::move(ctrls)) {}

Result<ResolvedTarget> Raid0Resolver::resolve(std::string_view uri, const ResolveOptions&) {
    using R = Result<ResolvedTarget>;
    auto p = base_.build_payload(uri_to_path(uri));
    if (!p.ok()) return R::Failure(p.status());
    auto out = std::make_shared<FileExtentPayload>(*p.value());
    out->extents.clear();
    for (const auto& e : p.value()->extents) {
        std::uint64_t lo = e.logical, ph = e.physical - base_.binding().namespace_base_bytes, left = e.length;
        while (left > 0) {
            Raid0Location loc = raid0_map(geo_, ph);
            std::uint64_t n = std::min(left, loc.contiguous);
            out->extents.push_back({lo, loc.offset, n, geo_.members[loc.member].device_index, 0});
            lo += n;
            ph += n;
            left -= n;
        }
    }
    out->controller = "raid0";
    out->mapping = "fiemap-raid0";
    std::uint64_t size = out->file_size;
    return ResolvedTarget::make<FileExtentPayload>("tutti.raid0-file", kFileExtentPayloadType,
                                                   kFileExtentPayloadVersion, size,
                                                   base_.binding().datapath_key, std::string(uri), out);
}

}  // namespace tutti
