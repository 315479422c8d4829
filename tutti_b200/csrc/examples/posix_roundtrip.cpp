// posix_roundtrip: the public C++ API end to end, without a GPU.
//
//   tutti_posix_roundtrip <directory>
//
// Assembles a StorageRuntime from its components (a file resolver for the
// "file" scheme, the host-executed POSIX DataPath), opens a file under
// <directory>, registers host memory, writes a pattern, reads it back into a
// cleared buffer and checks every byte. Prints "OK <bytes>" and exits 0.
// A GPU deployment swaps the DataPath (and its resolver mapping); the calls
// below stay the same.
// Parity: reference examples/tutti_runtime_example (assembly, open, register,
// submit, wait, release through the public API).

#include <fcntl.h>
#include <unistd.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include <tutti/storage_runtime.h>

#include "../datapaths/posix_data_path.h"
#include "../resolvers/file_resolvers.h"

using namespace tutti;

namespace {
int fail(const std::string& what, const Status& s) {
    std::fprintf(stderr, "%s: %s\n", what.c_str(), s.to_string().c_str());
    return 1;
}
}  // namespace

int main(int argc, char** argv) {
    if (argc != 2) {
        std::fprintf(stderr, "usage: %s <directory>\n", argv[0]);
        return 2;
    }
    const std::string dir = argv[1];
    const std::string path = dir + "/object.seg";
    constexpr std::uint64_t kFile = 4u << 20, kIo = 1u << 20;
    {  // the target: a file with real (written) blocks
        std::vector<char> zero(kFile, 0);
        const int fd = ::open(path.c_str(), O_CREAT | O_TRUNC | O_WRONLY, 0644);
        if (fd < 0 || ::pwrite(fd, zero.data(), zero.size(), 0) != static_cast<ssize_t>(zero.size()) || ::fsync(fd))
            return fail("create " + path, {StatusCode::NOT_FOUND, std::strerror(errno)});
        ::close(fd);
    }

    // 1) components: resolver (scheme "file") and DataPath (key "posix")
    OwnedComponents comps;
    MountBinding mb;
    mb.mount_path = dir;
    mb.controller = "posix0";
    mb.mapping = "synthetic";  // host IO needs no physical extents
    mb.datapath_key = "posix";
    auto mm = std::make_unique<MultiMountResolver>();
    Status s = mm->add(std::make_unique<LocalFileResolver>(mb), dir);
    if (!s.ok()) return fail("resolver", s);
    comps.resolvers.push_back({"file", std::move(mm)});
    PosixConfig pc;
    pc.threads = 2;
    pc.direct_io = false;
    comps.data_paths.push_back({"posix", std::make_shared<PosixDataPath>(pc), DataPathConfig{"posix"}});
    RuntimeConfig rc;
    rc.accel_id = 0;
    auto created = StorageRuntime::create_owning(rc, std::move(comps));
    if (!created.ok()) return fail("create runtime", created.status());
    std::unique_ptr<StorageRuntime> rt = std::move(created).value();

    // 2) target and memory
    auto target = rt->open("file://" + path);
    if (!target.ok()) return fail("open", target.status());
    void* buf = nullptr;
    if (posix_memalign(&buf, 4096, kIo) != 0) return fail("alloc", {StatusCode::RESOURCE_EXHAUSTED, "oom"});
    MemoryView v;
    v.address = buf;
    v.size = kIo;
    v.expected_kind = MemoryKind::HOST;
    auto mem = rt->register_memory(v);
    if (!mem.ok()) return fail("register_memory", mem.status());

    // 3) write a pattern at 1 MiB, read it back into a cleared buffer
    auto* bytes = static_cast<unsigned char*>(buf);
    for (std::uint64_t i = 0; i < kIo; ++i) bytes[i] = static_cast<unsigned char>(i * 131 + 7);
    std::vector<unsigned char> want(bytes, bytes + kIo);
    const HostSubmitContext ctx{ExecutionDomain::HOST_EXECUTION, -1, nullptr};
    for (IoDirection dir_ : {IoDirection::WRITE, IoDirection::READ}) {
        if (dir_ == IoDirection::READ) std::memset(buf, 0, kIo);
        IoRequest req{dir_, mem.value(), 0, target.value(), kIo, kIo};
        IoSubmitOutcome o = rt->submit(&req, 1, ctx);
        if (!o.io) return fail("submit", o.status);
        WaitOutcome w = rt->wait(*o.io, 10000);
        if (!w.observation_status.ok()) return fail("wait", w.observation_status);
        if (w.result->state != IoState::COMPLETED) return fail("io", w.result->status);
        s = rt->release_io(*o.io);
        if (!s.ok()) return fail("release_io", s);
    }
    if (std::memcmp(buf, want.data(), kIo) != 0) return fail("verify", {StatusCode::DATA_LOSS, "bytes differ"});

    // 4) teardown in reverse order
    s = rt->unregister_memory(mem.value());
    if (s.ok()) s = rt->close(target.value());
    if (s.ok()) s = rt->shutdown(10000);
    std::free(buf);
    if (!s.ok()) return fail("teardown", s);
    std::printf("OK %llu\n", static_cast<unsigned long long>(kIo));
    return 0;
}
