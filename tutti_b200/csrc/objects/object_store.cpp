#include "object_store.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/file.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstring>
#include <cstdio>
#include <map>
#include <set>

#include "digest.h"

namespace tutti {

namespace {
constexpr std::uint64_t kHeaderBytes = 4096;
constexpr char kObjMagic[8] = {'T', 'U', 'T', 'T', 'I', 'O', 'B', 'J'};
constexpr char kIdxMagic[8] = {'T', 'U', 'T', 'T', 'I', 'I', 'D', 'X'};
constexpr char kResMagic[8] = {'T', 'U', 'T', 'T', 'I', 'R', 'E', 'S'};
constexpr std::uint32_t kVersion = 1;

std::string join(const std::string& a, const std::string& b) {
    if (a.empty()) return b;
    return a.back() == '/' ? a + b : a + "/" + b;
}

Status errno_status(const std::string& what) {
    return {StatusCode::INTERNAL, what + ": " + std::strerror(errno)};
}

Status mkdirs(const std::string& path) {
    std::string cur;
    std::size_t i = 0;
    if (!path.empty() && path[0] == '/') cur = "/";
    while (i < path.size()) {
        std::size_t j = path.find('/', i);
        if (j == std::string::npos) j = path.size();
        const std::string part = path.substr(i, j - i);
        i = j + 1;
        if (part.empty()) continue;
        cur = join(cur, part);
        if (::mkdir(cur.c_str(), 0755) != 0 && errno != EEXIST) return errno_status("mkdir " + cur);
    }
    return Status::Ok();
}

template <typename T>
void put(std::uint8_t* b, std::size_t off, T v) {
    std::memcpy(b + off, &v, sizeof(T));  // little-endian hosts only (x86-64, aarch64)
}
template <typename T>
T get(const std::uint8_t* b, std::size_t off) {
    T v;
    std::memcpy(&v, b + off, sizeof(T));
    return v;
}

bool pread_full(int fd, void* buf, std::size_t n, std::uint64_t off) {
    std::size_t done = 0;
    while (done < n) {
        ssize_t r = ::pread(fd, static_cast<char*>(buf) + done, n - done, off + done);
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) return false;
        done += static_cast<std::size_t>(r);
    }
    return true;
}
bool pwrite_full(int fd, const void* buf, std::size_t n, std::uint64_t off) {
    std::size_t done = 0;
    while (done < n) {
        ssize_t r = ::pwrite(fd, static_cast<const char*>(buf) + done, n - done, off + done);
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) return false;
        done += static_cast<std::size_t>(r);
    }
    return true;
}
}  // namespace

std::uint64_t ObjectKey::identity() const noexcept { return object_identity(bytes.data(), bytes.size()); }
std::uint32_t ObjectKey::key_crc32() const noexcept { return crc32c(bytes.data(), bytes.size()); }

SegmentFileObjectStore::SegmentFileObjectStore() = default;
SegmentFileObjectStore::~SegmentFileObjectStore() { close(); }

std::uint64_t SegmentFileObjectStore::header_offset_for_slot(std::uint64_t slot) const {
    const std::uint64_t n = cfg_.devices.size();
    return ((slot / n) % cfg_.segment_file_slots) * slot_bytes_;
}
std::uint64_t SegmentFileObjectStore::payload_offset_for_slot(std::uint64_t slot) const {
    return header_offset_for_slot(slot) + cfg_.segment_header_bytes;
}
std::string SegmentFileObjectStore::slot_path(std::uint64_t slot) const {
    const std::uint64_t n = cfg_.devices.size();
    const std::uint64_t dev = slot % n;
    const std::uint64_t file_id = (slot / n) / cfg_.segment_file_slots;
    return join(join(cfg_.devices[dev].mount_path, "r" + std::to_string(cfg_.rank_id) + "/segments"),
                std::to_string(file_id) + ".seg");
}
std::string SegmentFileObjectStore::slot_uri(std::uint64_t slot) const {
    if (slot >= ready_.load()) return "";
    return "file://" + slot_path(slot);
}

int SegmentFileObjectStore::fd_for_slot(std::uint64_t slot, bool /*write*/) const {
    const std::string p = slot_path(slot);
    std::lock_guard<std::mutex> g(fd_mu_);
    auto it = fds_.find(p);
    if (it != fds_.end()) return it->second;
    // One cached descriptor per segment file, writable unless the store is read-only.
    int fd = ::open(p.c_str(), (cfg_.read_only ? O_RDONLY : O_RDWR) | O_CLOEXEC);
    if (fd >= 0) fds_[p] = fd;
    return fd;
}

Status SegmentFileObjectStore::check_writable(const char* op) const {
    if (!open_) return {StatusCode::NOT_READY, std::string(op) + ": store is not open"};
    if (cfg_.read_only) return {StatusCode::UNSUPPORTED, std::string(op) + ": store is read-only"};
    return Status::Ok();
}

Status SegmentFileObjectStore::save_namespace_meta() {
    char buf[512];
    const int n = std::snprintf(
        buf, sizeof(buf),
        "tutti-namespace v1\nsegment_bytes %llu\nsegment_count %u\nsegment_file_slots %llu\n"
        "segment_header_bytes %llu\ndevices %zu\nrank_count %u\nfingerprint %llu\n",
        static_cast<unsigned long long>(cfg_.layout.segment_bytes), cfg_.layout.segment_count,
        static_cast<unsigned long long>(cfg_.segment_file_slots),
        static_cast<unsigned long long>(cfg_.segment_header_bytes), cfg_.devices.size(), cfg_.rank_count,
        static_cast<unsigned long long>(fingerprint_digest_));
    const std::string path = join(join(cfg_.uri, "meta"), "namespace");
    // Every rank of a namespace writes the same meta file: a private temporary
    // name per rank and process keeps concurrent opens from racing on it.
    const std::string tmp = path + ".tmp." + std::to_string(cfg_.rank_id) + "." + std::to_string(::getpid());
    int fd = ::open(tmp.c_str(), O_WRONLY | O_CREAT | O_TRUNC | O_CLOEXEC, 0644);
    if (fd < 0) return errno_status("write " + tmp);
    const bool ok = pwrite_full(fd, buf, static_cast<std::size_t>(n), 0) && ::fsync(fd) == 0;
    ::close(fd);
    if (!ok) return errno_status("write " + tmp);
    if (::rename(tmp.c_str(), path.c_str()) != 0) return errno_status("rename namespace meta");
    return Status::Ok();
}

Status SegmentFileObjectStore::check_namespace_meta(bool* exists) {
    const std::string path = join(join(cfg_.uri, "meta"), "namespace");
    std::FILE* f = std::fopen(path.c_str(), "r");
    *exists = f != nullptr;
    if (!f) return Status::Ok();
    std::map<std::string, std::string> kv;
    char line[256];
    while (std::fgets(line, sizeof(line), f)) {
        char k[128], v[128];
        if (std::sscanf(line, "%127s %127s", k, v) == 2) kv[k] = v;
    }
    std::fclose(f);
    auto want = [&](const char* key, std::uint64_t val) {
        return kv.count(key) && kv[key] == std::to_string(val);
    };
    if (!want("segment_bytes", cfg_.layout.segment_bytes) || !want("segment_count", cfg_.layout.segment_count) ||
        !want("segment_file_slots", cfg_.segment_file_slots) ||
        !want("segment_header_bytes", cfg_.segment_header_bytes) || !want("devices", cfg_.devices.size()) ||
        !want("fingerprint", fingerprint_digest_))
        return {StatusCode::INVALID_ARGUMENT, "namespace fingerprint or layout mismatch at " + cfg_.uri};
    return Status::Ok();
}

Status SegmentFileObjectStore::adopt_namespace_meta() {
    const std::string path = join(join(cfg_.uri, "meta"), "namespace");
    std::FILE* f = std::fopen(path.c_str(), "r");
    if (!f) return {StatusCode::NOT_FOUND, "no namespace at " + cfg_.uri};
    std::map<std::string, std::string> kv;
    char line[256];
    while (std::fgets(line, sizeof(line), f)) {
        char k[128], v[128];
        if (std::sscanf(line, "%127s %127s", k, v) == 2) kv[k] = v;
    }
    std::fclose(f);
    for (const char* key : {"segment_bytes", "segment_count", "segment_file_slots", "segment_header_bytes", "devices",
                            "rank_count", "fingerprint"})
        if (!kv.count(key)) return {StatusCode::DATA_LOSS, std::string("namespace meta lacks ") + key};
    cfg_.layout.segment_bytes = std::stoull(kv["segment_bytes"]);
    cfg_.layout.segment_count = static_cast<std::uint32_t>(std::stoul(kv["segment_count"]));
    cfg_.segment_file_slots = std::stoull(kv["segment_file_slots"]);
    cfg_.segment_header_bytes = std::stoull(kv["segment_header_bytes"]);
    cfg_.rank_count = static_cast<std::uint32_t>(std::stoul(kv["rank_count"]));
    if (std::stoull(kv["devices"]) != cfg_.devices.size())
        return {StatusCode::INVALID_ARGUMENT, "namespace has " + kv["devices"] + " devices, view names " +
                                                  std::to_string(cfg_.devices.size())};
    adopted_fingerprint_ = std::stoull(kv["fingerprint"]);
    // capacity: every complete file group on media
    const std::uint64_t group = cfg_.segment_file_slots * cfg_.devices.size();
    const std::uint64_t file_b = cfg_.segment_file_slots * (cfg_.segment_header_bytes + cfg_.layout.payload_bytes());
    std::uint64_t groups = 0;
    for (;; ++groups) {
        bool all = true;
        for (std::uint64_t d = 0; d < cfg_.devices.size() && all; ++d) {
            // file g of every device holds file group g
            const std::string p = join(join(cfg_.devices[d].mount_path, "r" + std::to_string(cfg_.rank_id) + "/segments"),
                                       std::to_string(groups) + ".seg");
            struct stat st {};
            if (::stat(p.c_str(), &st) != 0 || static_cast<std::uint64_t>(st.st_size) < file_b) all = false;
        }
        if (!all) break;
    }
    cfg_.capacity_slots = std::max<std::uint64_t>(groups, 1) * group;
    return Status::Ok();
}

Status SegmentFileObjectStore::open(const StoreConfig& config) {
    std::lock_guard<std::mutex> g(mu_);
    if (open_) return {StatusCode::INVALID_ARGUMENT, "already open"};
    cfg_ = config;
    if (cfg_.uri.empty()) return {StatusCode::INVALID_ARGUMENT, "uri required"};
    adopted_fingerprint_ = 0;
    if (cfg_.adopt_namespace_meta) {
        if (!cfg_.read_only) return {StatusCode::INVALID_ARGUMENT, "adopt_namespace_meta needs a read-only view"};
        if (cfg_.devices.empty()) {
            StoreDevice d;
            d.mount_path = cfg_.uri;
            cfg_.devices.push_back(d);
        }
        TUTTI_RETURN_IF_ERROR(adopt_namespace_meta());
    }
    if (cfg_.layout.segment_bytes == 0 || cfg_.layout.segment_count == 0)
        return {StatusCode::INVALID_ARGUMENT, "layout must be non-empty"};
    if (cfg_.layout.segment_bytes % 4096) return {StatusCode::INVALID_ARGUMENT, "segment_bytes must be 4096-aligned"};
    if (cfg_.segment_file_slots == 0) return {StatusCode::INVALID_ARGUMENT, "segment_file_slots must be positive"};
    if (cfg_.segment_header_bytes < kHeaderBytes || cfg_.segment_header_bytes % 4096)
        return {StatusCode::INVALID_ARGUMENT, "segment_header_bytes must be >= 4096 and 4096-aligned"};
    if (cfg_.devices.empty()) {
        StoreDevice d;
        d.mount_path = cfg_.uri;
        cfg_.devices.push_back(d);
    }
    for (auto& d : cfg_.devices)
        if (d.mount_path.empty()) return {StatusCode::INVALID_ARGUMENT, "device needs a mount_path"};
    if (cfg_.rank_count == 0 || cfg_.rank_id >= cfg_.rank_count)
        return {StatusCode::INVALID_ARGUMENT, "rank_id must be < rank_count"};
    slot_bytes_ = cfg_.segment_header_bytes + cfg_.layout.payload_bytes();
    if (cfg_.capacity_slots)
        total_slots_ = cfg_.capacity_slots;
    else if (cfg_.capacity_bytes)
        total_slots_ = cfg_.capacity_bytes / slot_bytes_;
    else
        total_slots_ = cfg_.segment_file_slots * cfg_.devices.size();
    if (total_slots_ == 0) return {StatusCode::INVALID_ARGUMENT, "capacity too small to hold a single object"};
    group_slots_ = cfg_.segment_file_slots * cfg_.devices.size();
    fingerprint_digest_ = cfg_.adopt_namespace_meta
                              ? adopted_fingerprint_
                              : object_identity(cfg_.namespace_fingerprint.data(), cfg_.namespace_fingerprint.size());
    bool exists = false;
    TUTTI_RETURN_IF_ERROR(check_namespace_meta(&exists));
    if (!cfg_.read_only) {
        TUTTI_RETURN_IF_ERROR(mkdirs(join(cfg_.uri, "meta")));
        for (auto& d : cfg_.devices)
            TUTTI_RETURN_IF_ERROR(mkdirs(join(d.mount_path, "r" + std::to_string(cfg_.rank_id) + "/segments")));
        if (!exists) TUTTI_RETURN_IF_ERROR(save_namespace_meta());
    } else if (!exists) {
        return {StatusCode::NOT_FOUND, "read-only open of a namespace that does not exist: " + cfg_.uri};
    }
    slots_.assign(total_slots_, Slot{});
    by_key_.clear();
    // Adopt every complete file group already on media.
    std::uint64_t ready = 0;
    for (std::uint64_t grp = 0; grp * group_slots_ < total_slots_; ++grp) {
        bool all = true;
        for (std::uint64_t d = 0; d < cfg_.devices.size(); ++d)
            if (!segment_file_ready(slot_path(grp * group_slots_ + d))) all = false;
        if (!all) break;
        ready = std::min(total_slots_, (grp + 1) * group_slots_);
    }
    ready_.store(ready);
    open_ = true;
    if (!cfg_.read_only && ready == 0) {
        Status s = materialize_group(0);
        if (!s.ok()) {
            open_ = false;
            return s;
        }
        ready_.store(std::min(total_slots_, group_slots_));
    }
    precreate_target_ = ready_.load();
    Status b = open_bitmap();
    (void)b;  // an unusable bitmap only disables the cross-rank shortcut
    return Status::Ok();
}

namespace {
// The `.ready` marker of a segment file: its size and the (st_dev, st_ino) it
// was written for, so a replacement file of the same name and size is never
// taken for a prepared one.
std::string ready_marker_text(std::uint64_t bytes, const struct stat& st) {
    return "tutti-ready v1 " + std::to_string(bytes) + " " + std::to_string(static_cast<std::uint64_t>(st.st_dev)) +
           " " + std::to_string(static_cast<std::uint64_t>(st.st_ino)) + "\n";
}

// Holds `<mount>/.tutti_segment_precreate.lock` exclusively: ranks that share a
// mount create their segment files one at a time, which keeps each file's
// extents long (concurrent zero-fills interleave their blocks).
class MountCreateLock {
public:
    explicit MountCreateLock(const std::string& mount) {
        const std::string p = mount + "/.tutti_segment_precreate.lock";
        fd_ = ::open(p.c_str(), O_RDWR | O_CREAT | O_CLOEXEC, 0644);
        if (fd_ >= 0) {
            while (::flock(fd_, LOCK_EX) != 0 && errno == EINTR) {
            }
        }
    }
    ~MountCreateLock() {
        if (fd_ >= 0) ::close(fd_);  // closing releases the lock
    }
    MountCreateLock(const MountCreateLock&) = delete;
    MountCreateLock& operator=(const MountCreateLock&) = delete;

private:
    int fd_ = -1;
};
}  // namespace

bool SegmentFileObjectStore::segment_file_ready(const std::string& path) const {
    struct stat st {};
    if (::stat(path.c_str(), &st) != 0 || static_cast<std::uint64_t>(st.st_size) < file_bytes()) return false;
    std::FILE* f = std::fopen((path + ".ready").c_str(), "r");
    if (!f) return false;
    char line[160] = {0};
    const bool got = std::fgets(line, sizeof(line), f) != nullptr;
    std::fclose(f);
    return got && ready_marker_text(file_bytes(), st) == line;
}

Status SegmentFileObjectStore::materialize_group(std::uint64_t grp) {
    const std::uint64_t fb = file_bytes();
    for (std::uint64_t d = 0; d < cfg_.devices.size(); ++d) {
        const std::string p = slot_path(grp * group_slots_ + d);
        if (segment_file_ready(p)) continue;  // prepared by an earlier open
        const std::string tmp = p + ".tmp";
        MountCreateLock serial(cfg_.devices[d].mount_path);
        int fd = ::open(tmp.c_str(), O_RDWR | O_CREAT | O_TRUNC | O_CLOEXEC, 0644);
        if (fd < 0) return errno_status("create " + tmp);
        if (cfg_.materialize == "fallocate") {
            if (::posix_fallocate(fd, 0, static_cast<off_t>(fb)) != 0) {
                ::close(fd);
                return errno_status("fallocate " + tmp);
            }
        } else {
            // Real zeros: FIEMAP must report written (not unwritten/delalloc) extents.
            std::vector<char> zero(4u << 20, 0);
            for (std::uint64_t o = 0; o < fb; o += zero.size()) {
                std::size_t n = static_cast<std::size_t>(std::min<std::uint64_t>(zero.size(), fb - o));
                if (!pwrite_full(fd, zero.data(), n, o)) {
                    ::close(fd);
                    return errno_status("zero-fill " + tmp);
                }
            }
        }
        if (::fsync(fd) != 0) {
            ::close(fd);
            return errno_status("fsync " + tmp);
        }
        ::close(fd);
        if (::rename(tmp.c_str(), p.c_str()) != 0) return errno_status("publish " + p);
        // The marker goes last (written, synced, renamed into place): a crash
        // before it leaves a file that the next open prepares again.
        struct stat st {};
        if (::stat(p.c_str(), &st) != 0) return errno_status("stat " + p);
        const std::string mk = ready_marker_text(fb, st), mtmp = p + ".ready.tmp";
        int mfd = ::open(mtmp.c_str(), O_WRONLY | O_CREAT | O_TRUNC | O_CLOEXEC, 0644);
        if (mfd < 0) return errno_status("create " + mtmp);
        const bool ok = pwrite_full(mfd, mk.data(), mk.size(), 0) && ::fsync(mfd) == 0;
        ::close(mfd);
        if (!ok) return errno_status("write " + mtmp);
        if (::rename(mtmp.c_str(), (p + ".ready").c_str()) != 0) return errno_status("publish " + p + ".ready");
    }
    return Status::Ok();
}

Result<std::uint64_t> SegmentFileObjectStore::precreate_step(std::uint64_t headroom) {
    using R = Result<std::uint64_t>;
    {
        std::lock_guard<std::mutex> g(mu_);
        TUTTI_RETURN_IF_ERROR_R(R, check_writable("precreate_step"));
    }
    const std::uint64_t ready = ready_.load();
    if (ready >= total_slots_) return std::uint64_t{0};
    {
        std::lock_guard<std::mutex> g(mu_);
        if (frontier_ + headroom < ready) return std::uint64_t{0};
    }
    bool expected = false;
    if (!precreating_.compare_exchange_strong(expected, true)) return std::uint64_t{0};
    const std::uint64_t grp = ready / group_slots_;
    precreate_target_ = std::min(total_slots_, (grp + 1) * group_slots_);
    Status s = materialize_group(grp);  // no store lock during file IO
    if (!s.ok()) {
        precreating_.store(false);
        return R::Failure(s);
    }
    const std::uint64_t now = std::min(total_slots_, (grp + 1) * group_slots_);
    ready_.store(now);
    precreating_.store(false);
    return now - ready;
}

std::uint64_t SegmentFileObjectStore::precreated_slots() const { return ready_.load(); }
std::uint64_t SegmentFileObjectStore::precreate_target() const { return precreate_target_; }
std::uint64_t SegmentFileObjectStore::ready_slots() const { return ready_.load(); }

std::uint64_t SegmentFileObjectStore::slot_generation(std::uint64_t slot) const {
    std::lock_guard<std::mutex> g(mu_);
    return slot < slots_.size() ? slots_[slot].generation : 0;
}

Status SegmentFileObjectStore::close() {
    {
        std::lock_guard<std::mutex> g(mu_);
        if (!open_) return Status::Ok();
    }
    if (!cfg_.read_only) checkpoint();
    std::lock_guard<std::mutex> g(mu_);
    {
        std::lock_guard<std::mutex> f(fd_mu_);
        for (auto& kv : fds_) ::close(kv.second);
        fds_.clear();
    }
    if (bitmap_) {
        ::msync(bitmap_, bitmap_bytes_, MS_SYNC);
        ::munmap(bitmap_, bitmap_bytes_);
        bitmap_ = nullptr;
    }
    for (auto& pb : peer_bitmaps_) ::munmap(const_cast<std::uint8_t*>(pb.first), pb.second);
    peer_bitmaps_.clear();
    slots_.clear();
    by_key_.clear();
    open_ = false;
    return Status::Ok();
}

Status SegmentFileObjectStore::open_bitmap() {
    bitmaps_usable_ = false;
    if (cfg_.rank_count <= 1) return Status::Ok();
    const std::string dir = join(cfg_.uri, "residency");
    if (!cfg_.read_only) TUTTI_RETURN_IF_ERROR(mkdirs(dir));
    bitmap_bytes_ = kHeaderBytes + (total_slots_ + 7) / 8;
    auto path_for = [&](std::uint32_t r) { return join(dir, "r" + std::to_string(r) + ".bitmap"); };
    if (!cfg_.read_only) {
        int fd = ::open(path_for(cfg_.rank_id).c_str(), O_RDWR | O_CREAT | O_CLOEXEC, 0644);
        if (fd < 0) return errno_status("open bitmap");
        if (::ftruncate(fd, static_cast<off_t>(bitmap_bytes_)) != 0) {
            ::close(fd);
            return errno_status("size bitmap");
        }
        void* m = ::mmap(nullptr, bitmap_bytes_, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
        ::close(fd);
        if (m == MAP_FAILED) return errno_status("mmap bitmap");
        bitmap_ = static_cast<std::uint8_t*>(m);
        // Rebuilt from verified state by recover(); start from all-clear.
        std::memset(bitmap_, 0, bitmap_bytes_);
        std::memcpy(bitmap_, kResMagic, 8);
        put<std::uint32_t>(bitmap_, 8, kVersion);
        put<std::uint32_t>(bitmap_, 12, cfg_.rank_id);
        put<std::uint32_t>(bitmap_, 16, cfg_.rank_count);
        put<std::uint64_t>(bitmap_, 20, total_slots_);
        put<std::uint64_t>(bitmap_, 28, fingerprint_digest_);
    }
    bool all_ok = true;
    for (std::uint32_t r = 0; r < cfg_.rank_count; ++r) {
        if (r == cfg_.rank_id && bitmap_) continue;
        int fd = ::open(path_for(r).c_str(), O_RDONLY | O_CLOEXEC);
        if (fd < 0) {
            all_ok = false;
            continue;
        }
        struct stat st {};
        if (::fstat(fd, &st) != 0 || static_cast<std::size_t>(st.st_size) != bitmap_bytes_) {
            ::close(fd);
            all_ok = false;
            continue;
        }
        void* m = ::mmap(nullptr, bitmap_bytes_, PROT_READ, MAP_SHARED, fd, 0);
        ::close(fd);
        if (m == MAP_FAILED) {
            all_ok = false;
            continue;
        }
        peer_bitmaps_.push_back({static_cast<const std::uint8_t*>(m), bitmap_bytes_});
    }
    bitmaps_usable_ = all_ok;
    return Status::Ok();
}

void SegmentFileObjectStore::set_bit(std::uint64_t slot, bool v) {
    if (!bitmap_) return;
    std::uint8_t* b = bitmap_ + kHeaderBytes + slot / 8;
    const std::uint8_t m = static_cast<std::uint8_t>(1u << (slot % 8));
    if (v)
        *b |= m;
    else
        *b &= static_cast<std::uint8_t>(~m);
}

bool SegmentFileObjectStore::contains(const ObjectKey& k) const {
    std::lock_guard<std::mutex> g(mu_);
    std::string key(k.bytes.begin(), k.bytes.end());
    auto it = by_key_.find(key);
    return it != by_key_.end() && slots_[it->second].state == SlotState::COMMITTED;
}

std::uint64_t SegmentFileObjectStore::contains_prefix(const ObjectKey* keys, std::size_t n) const {
    std::lock_guard<std::mutex> g(mu_);
    std::uint64_t i = 0;
    for (; i < n; ++i) {
        std::string key(keys[i].bytes.begin(), keys[i].bytes.end());
        auto it = by_key_.find(key);
        if (it == by_key_.end() || slots_[it->second].state != SlotState::COMMITTED) break;
    }
    return i;
}

std::uint64_t SegmentFileObjectStore::contains_prefix_all_ranks(const ObjectKey* keys, std::size_t n) const {
    const std::uint64_t mine = contains_prefix(keys, n);
    if (cfg_.rank_count <= 1 || !bitmaps_usable_) return mine;
    std::lock_guard<std::mutex> g(mu_);
    std::uint64_t i = 0;
    for (; i < mine; ++i) {
        std::string key(keys[i].bytes.begin(), keys[i].bytes.end());
        const std::uint64_t s = by_key_.at(key);
        bool all = true;
        for (auto& pb : peer_bitmaps_) {
            if (get<std::uint64_t>(pb.first, 20) != total_slots_ || get<std::uint64_t>(pb.first, 28) != fingerprint_digest_ ||
                std::memcmp(pb.first, kResMagic, 8) != 0)
                return mine;  // degenerate to this rank's own answer
            if (!(pb.first[kHeaderBytes + s / 8] & (1u << (s % 8)))) {
                all = false;
                break;
            }
        }
        if (!all) break;
    }
    return i;
}

Result<ObjectPlacement> SegmentFileObjectStore::lookup(const ObjectKey& k) const {
    std::lock_guard<std::mutex> g(mu_);
    std::string key(k.bytes.begin(), k.bytes.end());
    auto it = by_key_.find(key);
    if (it == by_key_.end() || slots_[it->second].state != SlotState::COMMITTED)
        return Result<ObjectPlacement>::Failure({StatusCode::NOT_FOUND, "object not committed"});
    const std::uint64_t s = it->second;
    return ObjectPlacement{"file://" + slot_path(s), payload_offset_for_slot(s), cfg_.layout.payload_bytes(), s,
                           slots_[s].generation};
}

StoreUsage SegmentFileObjectStore::usage() const {
    std::lock_guard<std::mutex> g(mu_);
    StoreUsage u;
    std::uint64_t committed = 0, reserved = 0;
    u.per_device_bytes.assign(cfg_.devices.size(), 0);
    for (std::uint64_t s = 0; s < slots_.size(); ++s) {
        if (slots_[s].state == SlotState::COMMITTED) ++committed;
        if (slots_[s].state == SlotState::RESERVED) ++reserved;
        if (slots_[s].state != SlotState::FREE) u.per_device_bytes[s % cfg_.devices.size()] += slot_bytes_;
    }
    u.capacity_bytes = total_slots_ * slot_bytes_;
    u.committed_bytes = committed * slot_bytes_;
    u.reserved_bytes = reserved * slot_bytes_;
    u.usable_bytes = (total_slots_ - committed - reserved) * slot_bytes_;
    return u;
}

Result<ReserveOutcome> SegmentFileObjectStore::reserve(const ObjectKey* keys, std::size_t n) {
    using R = Result<ReserveOutcome>;
    std::lock_guard<std::mutex> g(mu_);
    TUTTI_RETURN_IF_ERROR_R(R, check_writable("reserve"));
    ReserveOutcome out;
    const std::uint64_t ready = ready_.load();
    for (std::size_t i = 0; i < n; ++i) {
        std::string key(keys[i].bytes.begin(), keys[i].bytes.end());
        if (key.empty() || key.size() > kHeaderBytes - 64) {
            ++out.rejected_count;
            continue;
        }
        auto it = by_key_.find(key);
        if (it != by_key_.end()) {
            const std::uint64_t s = it->second;
            out.accepted.push_back({"file://" + slot_path(s), payload_offset_for_slot(s), cfg_.layout.payload_bytes(),
                                    s, slots_[s].generation});
            out.accepted_keys.push_back(keys[i]);
            continue;
        }
        // Lowest free ready slot at or after the frontier (wraps once).
        std::uint64_t found = UINT64_MAX;
        for (std::uint64_t k = 0; k < ready; ++k) {
            const std::uint64_t s = (frontier_ + k) % ready;
            if (slots_[s].state == SlotState::FREE) {
                found = s;
                break;
            }
        }
        if (found == UINT64_MAX) {
            ++out.rejected_count;
            continue;
        }
        frontier_ = found + 1;
        Slot& sl = slots_[found];
        sl.state = SlotState::RESERVED;
        sl.generation += 1;
        sl.key = key;
        by_key_[key] = found;
        out.accepted.push_back({"file://" + slot_path(found), payload_offset_for_slot(found),
                                cfg_.layout.payload_bytes(), found, sl.generation});
        out.accepted_keys.push_back(keys[i]);
    }
    return out;
}

Status SegmentFileObjectStore::write_header(std::uint64_t slot, const Slot& s, bool valid) {
    alignas(4096) static thread_local std::uint8_t h[kHeaderBytes];
    std::memset(h, 0, sizeof(h));
    if (valid) {
        std::memcpy(h, kObjMagic, 8);
        put<std::uint32_t>(h, 8, kVersion);
        put<std::uint64_t>(h, 16, object_identity(s.key.data(), s.key.size()));
        put<std::uint64_t>(h, 24, cfg_.layout.payload_bytes());
        put<std::uint64_t>(h, 32, s.generation);
        put<std::uint32_t>(h, 40, static_cast<std::uint32_t>(s.key.size()));
        put<std::uint32_t>(h, 44, crc32c(s.key.data(), s.key.size()));
        put<std::uint64_t>(h, 48, s.commit_seq);
        put<std::uint32_t>(h, 56, crc32c(h, 56));
        std::memcpy(h + 64, s.key.data(), s.key.size());
    }
    int fd = fd_for_slot(slot, true);
    if (fd < 0) return errno_status("open segment for header");
    if (!pwrite_full(fd, h, kHeaderBytes, header_offset_for_slot(slot))) return errno_status("write header");
    return Status::Ok();
}

bool SegmentFileObjectStore::read_header(std::uint64_t slot, std::string* key, std::uint64_t* gen,
                                         std::uint64_t* seq) const {
    std::uint8_t h[kHeaderBytes];
    int fd = fd_for_slot(slot, false);
    if (fd < 0 || !pread_full(fd, h, kHeaderBytes, header_offset_for_slot(slot))) return false;
    if (std::memcmp(h, kObjMagic, 8) != 0) return false;
    if (get<std::uint32_t>(h, 8) != kVersion) return false;
    if (get<std::uint32_t>(h, 56) != crc32c(h, 56)) return false;
    if (get<std::uint64_t>(h, 24) != cfg_.layout.payload_bytes()) return false;
    const std::uint32_t klen = get<std::uint32_t>(h, 40);
    if (klen == 0 || klen > kHeaderBytes - 64) return false;
    std::string k(reinterpret_cast<const char*>(h + 64), klen);
    if (crc32c(k.data(), k.size()) != get<std::uint32_t>(h, 44)) return false;
    if (object_identity(k.data(), k.size()) != get<std::uint64_t>(h, 16)) return false;
    *key = std::move(k);
    *gen = get<std::uint64_t>(h, 32);
    *seq = get<std::uint64_t>(h, 48);
    return true;
}

Status SegmentFileObjectStore::commit(const ObjectKey* keys, std::size_t n) {
    std::lock_guard<std::mutex> g(mu_);
    TUTTI_RETURN_IF_ERROR(check_writable("commit"));
    std::vector<std::uint64_t> todo;
    for (std::size_t i = 0; i < n; ++i) {
        std::string key(keys[i].bytes.begin(), keys[i].bytes.end());
        auto it = by_key_.find(key);
        if (it == by_key_.end()) return {StatusCode::NOT_FOUND, "commit of a key that was not reserved"};
        if (slots_[it->second].state == SlotState::RESERVED) todo.push_back(it->second);
    }
    // 1) payload durable: one fdatasync per segment file touched
    std::set<int> fds;
    for (auto s : todo) fds.insert(fd_for_slot(s, true));
    for (int fd : fds)
        if (fd >= 0 && ::fdatasync(fd) != 0) return errno_status("fdatasync payload");
    // 2) headers, then their fdatasync
    for (auto s : todo) {
        slots_[s].commit_seq = ++commit_seq_;
        TUTTI_RETURN_IF_ERROR(write_header(s, slots_[s], true));
    }
    for (int fd : fds)
        if (fd >= 0 && ::fdatasync(fd) != 0) return errno_status("fdatasync header");
    for (auto s : todo) {
        slots_[s].state = SlotState::COMMITTED;
        set_bit(s, true);
    }
    return Status::Ok();
}

Status SegmentFileObjectStore::abort(const ObjectKey* keys, std::size_t n) {
    std::lock_guard<std::mutex> g(mu_);
    TUTTI_RETURN_IF_ERROR(check_writable("abort"));
    for (std::size_t i = 0; i < n; ++i) {
        std::string key(keys[i].bytes.begin(), keys[i].bytes.end());
        auto it = by_key_.find(key);
        if (it == by_key_.end() || slots_[it->second].state != SlotState::RESERVED) continue;
        slots_[it->second].state = SlotState::FREE;
        slots_[it->second].key.clear();
        by_key_.erase(it);
    }
    return Status::Ok();
}

Result<std::uint64_t> SegmentFileObjectStore::release(const ObjectKey* keys, std::size_t n) {
    using R = Result<std::uint64_t>;
    std::lock_guard<std::mutex> g(mu_);
    TUTTI_RETURN_IF_ERROR_R(R, check_writable("release"));
    std::uint64_t released = 0;
    for (std::size_t i = 0; i < n; ++i) {
        std::string key(keys[i].bytes.begin(), keys[i].bytes.end());
        auto it = by_key_.find(key);
        if (it == by_key_.end()) continue;
        Slot& s = slots_[it->second];
        if (s.state != SlotState::COMMITTED || s.pins > 0) continue;
        TUTTI_RETURN_IF_ERROR_R(R, write_header(it->second, s, false));  // invalidate before reuse
        set_bit(it->second, false);
        s.state = SlotState::FREE;
        s.key.clear();
        by_key_.erase(it);
        ++released;
    }
    return released;
}

Status SegmentFileObjectStore::pin(const ObjectKey* keys, std::size_t n) {
    std::lock_guard<std::mutex> g(mu_);
    for (std::size_t i = 0; i < n; ++i) {
        auto it = by_key_.find(std::string(keys[i].bytes.begin(), keys[i].bytes.end()));
        if (it == by_key_.end()) return {StatusCode::NOT_FOUND, "pin of an unknown key"};
        slots_[it->second].pins += 1;
    }
    return Status::Ok();
}

Status SegmentFileObjectStore::unpin(const ObjectKey* keys, std::size_t n) {
    std::lock_guard<std::mutex> g(mu_);
    for (std::size_t i = 0; i < n; ++i) {
        auto it = by_key_.find(std::string(keys[i].bytes.begin(), keys[i].bytes.end()));
        if (it == by_key_.end()) return {StatusCode::NOT_FOUND, "unpin of an unknown key"};
        if (slots_[it->second].pins == 0) return {StatusCode::INVALID_ARGUMENT, "unpin below zero"};
        slots_[it->second].pins -= 1;
    }
    return Status::Ok();
}

Status SegmentFileObjectStore::checkpoint() {
    std::lock_guard<std::mutex> g(mu_);
    TUTTI_RETURN_IF_ERROR(check_writable("checkpoint"));
    std::vector<std::uint8_t> body;
    std::uint64_t count = 0;
    body.resize(8);
    for (std::uint64_t s = 0; s < slots_.size(); ++s) {
        const Slot& sl = slots_[s];
        if (sl.state != SlotState::COMMITTED) continue;
        ++count;
        const std::size_t o = body.size();
        body.resize(o + 36 + sl.key.size());
        put<std::uint32_t>(body.data(), o, static_cast<std::uint32_t>(sl.key.size()));
        put<std::uint64_t>(body.data(), o + 4, s);
        put<std::uint64_t>(body.data(), o + 12, cfg_.layout.payload_bytes());
        put<std::uint64_t>(body.data(), o + 20, sl.generation);
        put<std::uint64_t>(body.data(), o + 28, sl.commit_seq);
        std::memcpy(body.data() + o + 36, sl.key.data(), sl.key.size());
    }
    put<std::uint64_t>(body.data(), 0, count);
    const std::uint64_t need = (kHeaderBytes + body.size() + 4095) / 4096 * 4096;
    // Container capacity fixed by the slot count (worst case: 64-byte keys).
    const std::uint64_t cap = (kHeaderBytes + 8 + total_slots_ * (36 + 64) + 4095) / 4096 * 4096;
    if (need > cap) return {StatusCode::RESOURCE_EXHAUSTED, "checkpoint image exceeds its container"};
    std::vector<std::uint8_t> img(need, 0);
    std::memcpy(img.data(), kIdxMagic, 8);
    const std::uint64_t seq = ++ckpt_seq_;
    put<std::uint32_t>(img.data(), 8, kVersion);
    put<std::uint64_t>(img.data(), 12, seq);
    put<std::uint64_t>(img.data(), 20, static_cast<std::uint64_t>(body.size()));
    put<std::uint32_t>(img.data(), 28, crc32c(body.data(), body.size()));
    std::memcpy(img.data() + kHeaderBytes, body.data(), body.size());
    const std::string path = join(join(cfg_.uri, "meta"), "checkpoint.bin");
    int fd = ::open(path.c_str(), O_RDWR | O_CREAT | O_CLOEXEC, 0644);
    if (fd < 0) return errno_status("open checkpoint");
    // Never overwrite the container holding the newest state: alternate by seq.
    const std::uint64_t container = seq % 2;
    bool ok = pwrite_full(fd, img.data(), img.size(), container * cap) && ::fdatasync(fd) == 0;
    ::close(fd);
    if (!ok) return errno_status("write checkpoint");
    if (bitmap_) ::msync(bitmap_, bitmap_bytes_, MS_ASYNC);
    return Status::Ok();
}

Result<std::vector<ObjectKey>> SegmentFileObjectStore::recover() {
    using R = Result<std::vector<ObjectKey>>;
    std::lock_guard<std::mutex> g(mu_);
    if (!open_) return R::Failure({StatusCode::NOT_READY, "store is not open"});
    std::set<std::uint64_t> candidates;
    // Checkpoint: newest container that verifies.
    const std::uint64_t cap = (kHeaderBytes + 8 + total_slots_ * (36 + 64) + 4095) / 4096 * 4096;
    const std::string path = join(join(cfg_.uri, "meta"), "checkpoint.bin");
    int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd >= 0) {
        std::uint64_t best_seq = 0;
        std::vector<std::uint8_t> best;
        for (std::uint64_t c = 0; c < 2; ++c) {
            std::uint8_t h[kHeaderBytes];
            if (!pread_full(fd, h, kHeaderBytes, c * cap) || std::memcmp(h, kIdxMagic, 8) != 0) continue;
            const std::uint64_t seq = get<std::uint64_t>(h, 12), bb = get<std::uint64_t>(h, 20);
            if (bb > cap - kHeaderBytes || bb < 8) continue;
            std::vector<std::uint8_t> body(bb);
            if (!pread_full(fd, body.data(), bb, c * cap + kHeaderBytes)) continue;
            if (crc32c(body.data(), body.size()) != get<std::uint32_t>(h, 28)) continue;
            if (seq > best_seq) {
                best_seq = seq;
                best = std::move(body);
            }
        }
        ::close(fd);
        ckpt_seq_ = best_seq;
        if (!best.empty()) {
            const std::uint64_t n = get<std::uint64_t>(best.data(), 0);
            std::size_t o = 8;
            for (std::uint64_t i = 0; i < n; ++i) {
                if (o + 36 > best.size()) break;
                const std::uint32_t kl = get<std::uint32_t>(best.data(), o);
                const std::uint64_t s = get<std::uint64_t>(best.data(), o + 4);
                if (o + 36 + kl > best.size()) break;
                if (s < total_slots_) candidates.insert(s);
                o += 36 + kl;
            }
        }
    }
    const std::uint64_t ready = ready_.load();
    if (cfg_.recover_full_scan || candidates.empty()) {
        for (std::uint64_t s = 0; s < ready; ++s) candidates.insert(s);
    }
    std::vector<ObjectKey> out;
    for (auto s : candidates) {
        if (s >= ready) continue;
        std::string key;
        std::uint64_t gen = 0, seq = 0;
        if (!read_header(s, &key, &gen, &seq)) continue;
        auto it = by_key_.find(key);
        if (it != by_key_.end()) {
            // Duplicate key: keep the newer commit.
            if (slots_[it->second].commit_seq >= seq) continue;
            slots_[it->second].state = SlotState::FREE;
            set_bit(it->second, false);
        }
        Slot& sl = slots_[s];
        sl.state = SlotState::COMMITTED;
        sl.generation = gen;
        sl.commit_seq = seq;
        sl.key = key;
        by_key_[key] = s;
        commit_seq_ = std::max(commit_seq_, seq);
        set_bit(s, true);
    }
    for (auto& kv : by_key_) {
        ObjectKey k;
        k.bytes.assign(kv.first.begin(), kv.first.end());
        out.push_back(std::move(k));
    }
    return out;
}

}  // namespace tutti
