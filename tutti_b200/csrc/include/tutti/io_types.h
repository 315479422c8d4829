#pragma once
// Public IO nouns: opaque generation-tagged handles, the six-field IoRequest and
// the host submit context.
//
// Parity: reference csrc/include/tutti/io_types.h:33-105 (handle tags, exactly six
// IoRequest fields, ExecutionDomain, HostSubmitContext with accel_id -1 meaning
// "the runtime's accelerator").

#include <cstdint>
#include <functional>

#include <cuda_runtime_api.h>

namespace tutti {

class StorageRuntime;

namespace detail {

// (runtime_id, slot, generation); generation 0 is the never-minted handle.
// Only StorageRuntime can mint a valid one; the raw triple is exposed read-only
// so bindings can marshal handles across the language boundary.
template <typename Tag>
class OpaqueHandle {
public:
    constexpr OpaqueHandle() noexcept = default;
    constexpr bool valid() const noexcept { return generation_ != 0; }
    constexpr bool operator==(const OpaqueHandle& o) const noexcept {
        return runtime_id_ == o.runtime_id_ && slot_ == o.slot_ &&
               generation_ == o.generation_;
    }
    constexpr bool operator!=(const OpaqueHandle& o) const noexcept { return !(*this == o); }
    constexpr std::uint32_t runtime_id() const noexcept { return runtime_id_; }
    constexpr std::uint32_t slot() const noexcept { return slot_; }
    constexpr std::uint64_t generation() const noexcept { return generation_; }

    // Bindings re-import a handle they exported; validity is still checked by the
    // runtime against its registry (a forged triple is just a stale handle).
    static constexpr OpaqueHandle from_raw(std::uint32_t rid, std::uint32_t slot,
                                           std::uint64_t gen) noexcept {
        return OpaqueHandle(rid, slot, gen);
    }

private:
    friend class ::tutti::StorageRuntime;
    constexpr OpaqueHandle(std::uint32_t rid, std::uint32_t slot, std::uint64_t gen) noexcept
        : runtime_id_(rid), slot_(slot), generation_(gen) {}
    std::uint32_t runtime_id_ = 0;
    std::uint32_t slot_ = 0;
    std::uint64_t generation_ = 0;
};

struct MemoryHandleTag {};
struct TargetHandleTag {};
struct IoHandleTag {};

}  // namespace detail

using MemoryHandle = detail::OpaqueHandle<detail::MemoryHandleTag>;
using TargetHandle = detail::OpaqueHandle<detail::TargetHandleTag>;
using IoHandle = detail::OpaqueHandle<detail::IoHandleTag>;

enum class IoDirection {
    READ,   // target -> memory
    WRITE,  // memory -> target
};

// Byte-range IO intent. Exactly six fields; bounds/alignment are validated by
// the runtime against the DataPath capabilities, never here.
struct IoRequest {
    IoDirection direction;
    MemoryHandle memory;
    std::uint64_t memory_offset;
    TargetHandle target;
    std::uint64_t target_offset;
    std::uint64_t length;
};

enum class ExecutionDomain {
    HOST_EXECUTION,
    DEVICE_EXECUTION,
};

// Stored format of the bytes a submit moves (one per submit). With
// FP8_E4M3_BLOCK128 the memory side holds bf16 and each request is stored as
// [E4M3 values][one fp32 scale per 128 values]: `length` stays the memory
// length (a multiple of 1024), the target range is stored_bytes(length) long
// and starts 16-byte aligned; consecutive requests must tile LBA-aligned runs.
enum class IoTransform : std::uint32_t {
    NONE = 0,
    FP8_E4M3_BLOCK128 = 1,
};

inline std::uint64_t stored_bytes(IoTransform t, std::uint64_t memory_bytes) {
    return t == IoTransform::FP8_E4M3_BLOCK128 ? memory_bytes / 64 * 33 : memory_bytes;
}

struct HostSubmitContext {
    ExecutionDomain execution_domain = ExecutionDomain::DEVICE_EXECUTION;
    std::int32_t accel_id = -1;  // -1: the owning runtime's accelerator
    cudaStream_t stream = nullptr;
    IoTransform transform = IoTransform::NONE;
};

}  // namespace tutti
