#pragma once
// Persisted digests of the storage object layer.
//  * crc32c: CRC-32C (Castagnoli, reflected polynomial 0x82F63B78), the
//    table-driven byte-at-a-time algorithm (Sarwate), as used by iSCSI/ext4.
//  * object_identity: FNV-1a 64 followed by the SplitMix64 finaliser (Steele,
//    Lea, Flood 2014). Both are fixed by the on-disk format shared with the
//    reference store (reference csrc/include/tutti/spi/object_digest.h:50-160),
//    so an object written by either is recognised by the other.

#include <cstddef>
#include <cstdint>

namespace tutti {

namespace detail {
struct Crc32cTable {
    std::uint32_t t[256];
    constexpr Crc32cTable() : t{} {
        for (std::uint32_t i = 0; i < 256; ++i) {
            std::uint32_t c = i;
            for (int k = 0; k < 8; ++k) c = (c & 1u) ? (c >> 1) ^ 0x82F63B78u : (c >> 1);
            t[i] = c;
        }
    }
};
inline constexpr Crc32cTable kCrc32cTable{};
}  // namespace detail

inline std::uint32_t crc32c_update(std::uint32_t state, const void* data, std::size_t n) noexcept {
    const auto* p = static_cast<const std::uint8_t*>(data);
    for (std::size_t i = 0; i < n; ++i) state = detail::kCrc32cTable.t[(state ^ p[i]) & 0xFFu] ^ (state >> 8);
    return state;
}

// CRC-32C of a buffer; 0 for an empty buffer.
inline std::uint32_t crc32c(const void* data, std::size_t n) noexcept {
    if (!data || n == 0) return 0;
    return crc32c_update(0xFFFFFFFFu, data, n) ^ 0xFFFFFFFFu;
}

inline std::uint64_t object_identity(const void* data, std::size_t n) noexcept {
    std::uint64_t h = 0xCBF29CE484222325ull;  // FNV-1a 64 offset basis
    const auto* p = static_cast<const std::uint8_t*>(data);
    for (std::size_t i = 0; p && i < n; ++i) {
        h ^= p[i];
        h *= 0x100000001B3ull;  // FNV-1a 64 prime
    }
    h ^= h >> 30;  // SplitMix64 finaliser
    h *= 0xBF58476D1CE4E5B9ull;
    h ^= h >> 27;
    h *= 0x94D049BB133111EBull;
    h ^= h >> 31;
    return h;
}

}  // namespace tutti
