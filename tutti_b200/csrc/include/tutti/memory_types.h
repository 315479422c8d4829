#pragma once
// Memory nouns for register_memory(). Parity: reference
// csrc/include/tutti/memory_types.h:39-83 (kinds, ownership, MemoryView fields,
// io_granularity > 0 requests register-time descriptor prebuild).

#include <cstdint>
#include <string>

namespace tutti {

enum class MemoryKind {
    HOST,         // pageable host memory
    PINNED_HOST,  // page-locked host memory
    DEVICE,       // device-local memory (HBM)
    MANAGED,      // unified memory
};

enum class MemoryOwnership {
    RUNTIME_OWNED,
    CALLER_OWNED,
};

struct MemoryView {
    void* address = nullptr;
    std::uint64_t size = 0;
    MemoryKind expected_kind = MemoryKind::DEVICE;
    MemoryOwnership ownership = MemoryOwnership::CALLER_OWNED;
    std::int32_t expected_accel_id = -1;  // < 0: unspecified
    std::string expected_profile;         // empty: unspecified
    // > 0: the DataPath prebuilds per-granule transfer descriptors at register
    // time so submit is a table lookup. 0: descriptors are built per submit.
    std::uint64_t io_granularity = 0;
};

}  // namespace tutti
