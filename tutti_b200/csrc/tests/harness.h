#pragma once
// Minimal test harness of the native suites: TEST registers a case, CHECK
// records a failure and returns from the case. `Fixture` is a runtime over
// the mock DataPath kit with one 64 KiB host buffer and one 64 KiB target.

#include <cstdio>
#include <cstring>
#include <functional>
#include <memory>
#include <string>
#include <vector>

#include <tutti/storage_runtime.h>

#include <unistd.h>

#include "../nvme/controller.h"

#include "../testing/mock_data_path.h"

namespace tutti {
namespace native_tests {

using namespace tutti::testing;

struct TestCase {
    const char* name;
    std::function<void()> fn;
};
inline std::vector<TestCase>& registry() {
    static std::vector<TestCase> r;
    return r;
}
struct Reg {
    Reg(const char* n, std::function<void()> f) { registry().push_back({n, std::move(f)}); }
};
inline int g_failures = 0;

#define TEST(name)                   \
    void name();                     \
    static Reg reg_##name(#name, name); \
    void name()
#define CHECK(cond)                                                                   \
    do {                                                                              \
        if (!(cond)) {                                                                \
            std::fprintf(stderr, "  CHECK failed %s:%d: %s\n", __FILE__, __LINE__, #cond); \
            ++g_failures;                                                             \
            return;                                                                   \
        }                                                                             \
    } while (0)

struct Fixture {
    MemResolver resolver;
    MockDataPath dp;
    std::unique_ptr<StorageRuntime> rt;
    std::vector<char> buf = std::vector<char>(1 << 16, 0);
    MemoryHandle mem;
    TargetHandle tgt;
    explicit Fixture(std::uint64_t budget = 64) {
        auto blob = std::make_shared<std::string>(1 << 16, '\0');
        for (std::size_t i = 0; i < blob->size(); ++i) (*blob)[i] = static_cast<char>(i * 7);
        resolver.objects["a"] = blob;
        resolver.objects["b"] = std::make_shared<std::string>(1 << 14, 'b');
        RuntimeConfig c;
        c.accel_id = 0;
        c.max_terminal_results = budget;
        RuntimeComponents comps;
        comps.resolvers.push_back({"mem", &resolver});
        comps.data_paths.push_back({"mock", &dp, DataPathConfig{"mock"}});
        rt = StorageRuntime::create(c, comps).value();
        MemoryView v;
        v.address = buf.data();
        v.size = buf.size();
        v.expected_kind = MemoryKind::HOST;
        mem = rt->register_memory(v).value();
        tgt = rt->open("mem://a").value();
    }
    IoRequest req(std::uint64_t off, std::uint64_t len, IoDirection d = IoDirection::READ) {
        return IoRequest{d, mem, off, tgt, off, len};
    }
    HostSubmitContext ctx() { return HostSubmitContext{ExecutionDomain::HOST_EXECUTION, -1, nullptr}; }
};

// Drives one emulated queue pair from the host: submits one SQE and waits
// (bounded) for its CQE; returns the CQE status field, or -1 on timeout.
struct HostSubmitter {
    nvme::QueuePairView q;
    std::uint32_t tail = 0, head = 0, phase = 1;
    // Submits one SQE and waits (bounded) for its CQE; returns the status field or -1 on timeout.
    int run(const nvme::Sqe& e, int polls = 200000) {
        q.sq[tail] = e;
        tail = (tail + 1) % q.depth;
        __atomic_store_n(q.sq_doorbell, tail, __ATOMIC_RELEASE);
        for (int i = 0; i < polls; ++i) {
            const std::uint32_t dw3 = __atomic_load_n(&q.cq[head].dw3, __ATOMIC_ACQUIRE);
            if (nvme::cqe_phase(dw3) == phase) {
                head = (head + 1) % q.depth;
                if (head == 0) phase ^= 1u;
                __atomic_store_n(q.cq_doorbell, head, __ATOMIC_RELEASE);
                return static_cast<int>(nvme::cqe_status(dw3));
            }
            usleep(10);
        }
        return -1;
    }
    // After the controller reset this queue: start over at slot 0, phase 1.
    void reset() { tail = head = 0, phase = 1; }
};


}  // namespace native_tests
}  // namespace tutti
