#pragma once
// Storage object layer: fixed segment files holding fixed-size slots, one
// durable object (a KV chunk with all its layers) per slot.
//
// On-disk format (kept identical to the reference store so either can read a
// namespace the other wrote; reference csrc/include/tutti/spi/storage_object_store.h:280-395,
// csrc/storage_objects/slot_placement_policy.cpp, checkpoint_region.cpp):
//   <mount[d]>/r<rank>/segments/<file_id>.seg   d = slot % N,
//       file_id = (slot / N) / segment_file_slots,
//       slot region at ((slot / N) % segment_file_slots) * slot_bytes,
//       slot_bytes = segment_header_bytes + payload_bytes;
//       object header in the first 4 KiB of the region, payload at +segment_header_bytes.
//   Object header: "TUTTIOBJ" | u32 version @8 | u64 identity @16 |
//       u64 payload_bytes @24 | u64 generation @32 | u32 key_len @40 |
//       u32 key_crc32 @44 | u64 commit_seq @48 | u32 header_crc32 @56 (over [0,56)) |
//       key bytes @64 (this store's addition: lets a full scan rebuild keys).
//   <uri>/meta/checkpoint.bin: two mirrored containers, each a 4 KiB header
//       "TUTTIIDX" | u32 version @8 | u64 seq @12 | u64 body_bytes @20 |
//       u32 body_crc32 @28, then a body of u64 count and entries
//       (u32 key_len, u64 slot, u64 payload_bytes, u64 generation, u64 commit_seq, key).
//   <uri>/residency/r<rank>.bitmap: 4 KiB header "TUTTIRES" | u32 version @8 |
//       u32 rank_id @12 | u32 rank_count @16 | u64 slot_count @20 |
//       u64 fingerprint digest @28, then one bit per slot (mmapped; never authoritative).
//   <uri>/meta/namespace: geometry + fingerprint; a mismatch fails open() closed.
//
// Commit order: payload fdatasync, then header write + fdatasync. A slot whose
// header does not verify is "never written".

#include <atomic>
#include <cstdint>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include <tutti/status.h>

namespace tutti {

struct ObjectKey {
    std::vector<std::uint8_t> bytes;
    std::uint64_t identity() const noexcept;
    std::uint32_t key_crc32() const noexcept;
    bool operator==(const ObjectKey& o) const noexcept { return bytes == o.bytes; }
};

struct ObjectLayout {
    std::uint64_t segment_bytes = 0;
    std::uint32_t segment_count = 0;
    std::uint64_t payload_bytes() const noexcept { return segment_bytes * segment_count; }
};

struct StoreDevice {
    std::string mount_path;
    std::string controller_pci_addr;
    std::uint32_t namespace_id = 0;
    std::uint32_t block_size = 0;
    std::string backing_device_path;
    std::uint64_t namespace_base_bytes = 0;
};

struct StoreConfig {
    std::string uri;
    std::uint64_t capacity_slots = 0;
    std::uint64_t capacity_bytes = 0;
    ObjectLayout layout;
    std::uint64_t segment_file_slots = 0;
    std::uint64_t segment_header_bytes = 0;
    std::vector<std::uint8_t> namespace_fingerprint;
    std::vector<StoreDevice> devices;
    std::uint32_t rank_id = 0;
    std::uint32_t rank_count = 1;
    bool read_only = false;
    std::uint32_t residency_sync_interval_ms = 1000;
    // "zeros" writes real zeros (FIEMAP-verified allocated extents, needed by
    // device IO); "fallocate" reserves blocks (unwritten extents, host IO only).
    std::string materialize = "zeros";
    bool recover_full_scan = false;
    // Read-only views only: take segment geometry, fingerprint and capacity from
    // the namespace's own meta file and media instead of checking them (a
    // scheduler that knows the namespace's location but not the model).
    bool adopt_namespace_meta = false;
};

struct ObjectPlacement {
    std::string uri;
    std::uint64_t offset = 0;
    std::uint64_t payload_bytes = 0;
    std::uint64_t slot = 0;
    std::uint64_t generation = 0;
    bool valid() const noexcept { return !uri.empty(); }
};

struct StoreUsage {
    std::uint64_t capacity_bytes = 0, committed_bytes = 0, reserved_bytes = 0, reclaiming_bytes = 0,
                  usable_bytes = 0;
    std::vector<std::uint64_t> per_device_bytes;
};

struct ReserveOutcome {
    std::vector<ObjectPlacement> accepted;
    std::vector<ObjectKey> accepted_keys;
    std::uint64_t rejected_count = 0;
};

class SegmentFileObjectStore {
public:
    SegmentFileObjectStore();
    ~SegmentFileObjectStore();

    Status open(const StoreConfig& config);
    Status close();

    bool contains(const ObjectKey& key) const;
    std::uint64_t contains_prefix(const ObjectKey* keys, std::size_t count) const;
    std::uint64_t contains_prefix_all_ranks(const ObjectKey* keys, std::size_t count) const;
    Result<ObjectPlacement> lookup(const ObjectKey& key) const;
    StoreUsage usage() const;

    std::uint64_t ready_slots() const;
    std::string slot_uri(std::uint64_t slot) const;
    std::string slot_path(std::uint64_t slot) const;
    // True when `path` has its full size and a `.ready` marker bound to its inode.
    bool segment_file_ready(const std::string& path) const;
    std::uint64_t slot_generation(std::uint64_t slot) const;
    std::uint64_t slot_bytes() const { return slot_bytes_; }
    std::uint64_t total_slots() const { return total_slots_; }

    Result<ReserveOutcome> reserve(const ObjectKey* keys, std::size_t count);
    Status commit(const ObjectKey* keys, std::size_t count);
    Status abort(const ObjectKey* keys, std::size_t count);
    Result<std::uint64_t> release(const ObjectKey* keys, std::size_t count);
    Status pin(const ObjectKey* keys, std::size_t count);
    Status unpin(const ObjectKey* keys, std::size_t count);

    Result<std::vector<ObjectKey>> recover();
    Status checkpoint();

    Result<std::uint64_t> precreate_step(std::uint64_t headroom);
    std::uint64_t precreated_slots() const;
    std::uint64_t precreate_target() const;

    // Placement math (exposed for tests of the on-disk format).
    std::uint64_t header_offset_for_slot(std::uint64_t slot) const;
    std::uint64_t payload_offset_for_slot(std::uint64_t slot) const;
    std::uint64_t file_bytes() const { return slot_bytes_ * cfg_.segment_file_slots; }

private:
    enum class SlotState : std::uint8_t { FREE, RESERVED, COMMITTED };
    struct Slot {
        SlotState state = SlotState::FREE;
        std::uint64_t generation = 0;
        std::uint32_t pins = 0;
        std::string key;  // raw key bytes
        std::uint64_t commit_seq = 0;
    };
    Status check_writable(const char* op) const;
    Status materialize_group(std::uint64_t group);
    Status write_header(std::uint64_t slot, const Slot& s, bool valid);
    bool read_header(std::uint64_t slot, std::string* key, std::uint64_t* gen, std::uint64_t* seq) const;
    int fd_for_slot(std::uint64_t slot, bool write) const;
    Status open_bitmap();
    void set_bit(std::uint64_t slot, bool v);
    Status save_namespace_meta();
    Status check_namespace_meta(bool* exists);
    Status adopt_namespace_meta();

    StoreConfig cfg_;
    bool open_ = false;
    std::uint64_t slot_bytes_ = 0;
    std::uint64_t total_slots_ = 0;
    std::uint64_t group_slots_ = 0;
    std::uint64_t fingerprint_digest_ = 0;
    mutable std::mutex mu_;
    std::vector<Slot> slots_;
    std::unordered_map<std::string, std::uint64_t> by_key_;
    std::atomic<std::uint64_t> ready_{0};
    std::uint64_t frontier_ = 0;  // next slot to try
    std::uint64_t commit_seq_ = 0;
    std::uint64_t ckpt_seq_ = 0;
    std::uint64_t precreate_target_ = 0;
    std::atomic<bool> precreating_{false};
    mutable std::mutex fd_mu_;
    mutable std::map<std::string, int> fds_;
    // residency
    std::uint8_t* bitmap_ = nullptr;
    std::size_t bitmap_bytes_ = 0;
    std::vector<std::pair<const std::uint8_t*, std::size_t>> peer_bitmaps_;
    std::uint64_t adopted_fingerprint_ = 0;
    bool bitmaps_usable_ = false;
};

}  // namespace tutti
