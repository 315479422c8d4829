// Fused GPU NVMe io kernel for sm_100a (warp-specialised).
//
// CTA of 512 threads = 16 warps, one CTA per queue lease:
//   * warp 0, lane 0 - the queue engine. It claims commands from the global
//     work-stealing cursor, resolves each command's logical range against the
//     target's HBM-resident extent table (device, LBA, extent and MDTS splits),
//     writes 64-byte SQEs into the CTA's own SQ on every device it touches,
//     rings each SQ tail doorbell once per round, drains CQEs by phase bit
//     (one CQ head doorbell per device per round) and enforces a
//     %globaltimer deadline per command. It never stalls on data movement.
//   * warps 1..15 - three mover groups of five warps. A group claims a ready
//     slot from a shared-memory queue and moves it: staging -> caller memory
//     for reads (the paged scatter), caller memory -> staging for writes (the
//     paged gather, then the engine submits the write). Groups synchronise on
//     their own named barrier, so three slots move at once while the engine
//     keeps the queues full.
// Staging reads use ld.global.cv (the controller rewrites a slot between
// uses); caller-memory stores use st.global.cs. Every wait is bounded: a
// command past its deadline is reported as a timeout and its slot is
// quarantined until its late completions drain; a launch that ends with
// commands still owned by the controller marks the queue dirty so the host
// resets it before the next launch; mover waits carry an iteration limit.
//
// Parity: reference csrc/data_paths/striped_local_nvme/fused_submit_kernel.cuh:171-218
// (pool of workers, one launch across N drives) fused with the separate
// csrc/kv_transfer/src/mem_kernels.cu:66-130 scatter; status words follow
// submit_one.cuh:117-143 (0 ok, 1 resolve, 2 timeout, 3 NVMe error).

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "io_kernel.h"
#include "primitives.cuh"

namespace tutti {
namespace io {

namespace {

enum SlotStateKind : int { S_FREE = 0, S_SUBMIT, S_INFLIGHT, S_READY, S_GATHER, S_POISON, S_MOVING };

constexpr int kMoverGroups = 3;
// A mover that waits longer than the command deadline plus this margin for
// the engine (which itself stops once nothing has moved for a deadline) gives
// up and flags the launch.
constexpr unsigned long long kMoverGraceNs = 2000000000ull;
constexpr unsigned long long kEngineGraceNs = 500000000ull;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ std::uint32_t ld_acquire_sys(const std::uint32_t* p) {
    std::uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(std::uint32_t* p, std::uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint4 ld_cv_v4(const void* p) {
    uint4 v;
    asm volatile("ld.global.cv.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void st_cs_v4(void* p, uint4 v) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

__device__ __forceinline__ float ld_cv_f32(const void* p) {
    float v;
    asm volatile("ld.global.cv.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}

constexpr float kE4M3Max = 448.0f;

// 16 E4M3 values (one uint4) times `scale` -> 16 bf16 values (two uint4).
__device__ __forceinline__ void fp8x16_dequant(uint4 q, float scale, uint4 out[2]) {
    const std::uint32_t w[4] = {q.x, q.y, q.z, q.w};
    std::uint32_t o[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float f[4];
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const __half_raw h =
                __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>((w[i] >> (8 * b)) & 0xFFu), __NV_E4M3);
            f[b] = __half2float(__half(h)) * scale;
        }
        __nv_bfloat162 lo = __floats2bfloat162_rn(f[0], f[1]), hi = __floats2bfloat162_rn(f[2], f[3]);
        o[2 * i] = *reinterpret_cast<std::uint32_t*>(&lo);
        o[2 * i + 1] = *reinterpret_cast<std::uint32_t*>(&hi);
    }
    out[0] = make_uint4(o[0], o[1], o[2], o[3]);
    out[1] = make_uint4(o[4], o[5], o[6], o[7]);
}

// Moves one fp8-transformed command: warps take pieces; within a piece a lane
// handles 16 consecutive values, so 8 lanes share one 128-value scale group
// (pieces hold a multiple of 512 values, so every lane of the warp takes part
// in every iteration and the shuffles are full-warp).
template <int W>
__device__ void move_slot_fp8(const IoKernelParams& p, const IoCommand& c, char* stage, bool to_memory, int gwarp,
                              int lane) {
    const IoPiece* pcs = p.pieces + c.first_piece;
    const std::uint32_t groups = (to_memory && c.replicas > 1) ? c.replicas : 1u;
    for (std::uint32_t q = gwarp; q < c.n_pieces; q += W) {
        const IoPiece pc = pcs[q];
        const std::uint32_t k = pc.bytes / 33u;  // memory bytes / 64
        const std::uint32_t units = 2u * k;      // 16-value units
        char* vals = stage + pc.off;
        char* scl = vals + 32u * k;
        if (to_memory) {
            for (std::uint32_t u = lane; u < units; u += 32) {
                uint4 o[2];
                fp8x16_dequant(ld_cv_v4(vals + 16u * u), ld_cv_f32(scl + 4u * (u >> 3)), o);
                for (std::uint32_t g = 0; g < groups; ++g) {
                    char* m = reinterpret_cast<char*>(g == 0 ? pc.mem : pcs[g * c.n_pieces + q].mem) + 32u * u;
                    st_cs_v4(m, o[0]);
                    st_cs_v4(m + 16, o[1]);
                }
            }
        } else {
            const char* mem = reinterpret_cast<const char*>(pc.mem);
            for (std::uint32_t u = lane; u < units; u += 32) {
                const uint4 a = *reinterpret_cast<const uint4*>(mem + 32u * u);
                const uint4 b = *reinterpret_cast<const uint4*>(mem + 32u * u + 16);
                const std::uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
                float v[16];
                float amax = 0.f;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
                    v[2 * i] = f.x;
                    v[2 * i + 1] = f.y;
                    amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
                }
#pragma unroll
                for (int o = 1; o < 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
                const float sc = amax > 0.f ? amax / kE4M3Max : 1.f;
                const float inv = 1.f / sc;
                std::uint32_t packed[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    std::uint32_t x = 0;
#pragma unroll
                    for (int b = 0; b < 4; ++b) {
                        const __nv_fp8_storage_t e = __nv_cvt_float_to_fp8(v[4 * i + b] * inv, __NV_SATFINITE, __NV_E4M3);
                        x |= static_cast<std::uint32_t>(e) << (8 * b);
                    }
                    packed[i] = x;
                }
                *reinterpret_cast<uint4*>(vals + 16u * u) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
                if ((lane & 7) == 0) *reinterpret_cast<float*>(scl + 4u * (u >> 3)) = sc;
            }
        }
    }
}

// Non-aligned named barrier (threads of a warp may arrive after diverging);
// callers reconverge with __syncwarp() first.
__device__ __forceinline__ void named_barrier(int id, int threads) {
    asm volatile("barrier.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Extent containing `pos` (binary search); -1 if none.
__device__ int find_extent(const DevTarget& t, std::uint64_t pos) {
    int lo = 0, hi = static_cast<int>(t.n_extents) - 1;
    while (lo <= hi) {
        const int mid = (lo + hi) >> 1;
        const DevExtent& e = t.extents[mid];
        if (pos < e.logical)
            hi = mid - 1;
        else if (pos >= e.logical + e.length)
            lo = mid + 1;
        else
            return mid;
    }
    return -1;
}

struct SubCmd {
    std::uint64_t lba;
    std::uint32_t device;
    std::uint32_t off;
    std::uint32_t bytes;
};

__device__ int resolve_cmd(const IoKernelParams& p, const IoCommand& c, SubCmd* out, std::uint32_t* err) {
    if (c.target == 0xFFFFFFFFu) {
        *err = kCmdResolve;
        return 0;
    }
    const DevTarget t = p.targets[c.target];
    if (t.extents == nullptr || c.bytes == 0 || c.bytes > p.slot_bytes || c.logical + c.bytes > t.size) {
        *err = kCmdResolve;
        return 0;
    }
    std::uint64_t pos = c.logical;
    std::uint32_t rem = c.bytes, off = 0;
    int n = 0;
    while (rem > 0) {
        const int ei = find_extent(t, pos);
        if (ei < 0 || n == kMaxSub) {
            *err = kCmdResolve;
            return 0;
        }
        const DevExtent e = t.extents[ei];
        if (e.device >= p.n_devices) {
            *err = kCmdBadDevice;
            return 0;
        }
        const DevDevice& d = p.devices[e.device];
        const std::uint64_t in_ext = e.logical + e.length - pos;
        std::uint32_t len = rem;
        if (in_ext < len) len = static_cast<std::uint32_t>(in_ext);
        if (d.mdts_bytes < len) len = d.mdts_bytes;
        const std::uint64_t phys = e.physical + (pos - e.logical);
        const std::uint64_t lba_mask = (1ull << d.lba_shift) - 1;
        if ((phys & lba_mask) || (len & lba_mask)) {
            *err = kCmdResolve;
            return 0;
        }
        out[n] = SubCmd{phys >> d.lba_shift, e.device, off, len};
        ++n;
        pos += len;
        off += len;
        rem -= len;
    }
    return n;
}

// One mover group moves one slot: warps take 4 KiB chunks of the command.
template <int W>
__device__ void move_slot(const IoKernelParams& p, const IoCommand& c, char* stage, bool to_memory, int gwarp,
                          int lane) {
    if (c.transform == kXformFp8Block128) {
        move_slot_fp8<W>(p, c, stage, to_memory, gwarp, lane);
        return;
    }
    const IoPiece* pcs = p.pieces + c.first_piece;
    const std::uint32_t nchunks = (c.bytes + 4095u) >> 12;
    for (std::uint32_t ch = gwarp; ch < nchunks; ch += W) {
        const std::uint32_t co = ch << 12;
        const std::uint32_t ce = min(co + 4096u, c.bytes);
        int lo = 0, hi = static_cast<int>(c.n_pieces) - 1, pi = 0;
        while (lo <= hi) {
            const int mid = (lo + hi) >> 1;
            if (pcs[mid].off <= co) {
                pi = mid;
                lo = mid + 1;
            } else {
                hi = mid - 1;
            }
        }
        const IoPiece first = pcs[pi];
        const std::uint32_t groups = (to_memory && c.replicas > 1) ? c.replicas : 1u;
        if (first.off <= co && first.off + first.bytes >= ce) {
            char* mem = reinterpret_cast<char*>(first.mem) + (co - first.off);
            const std::uint32_t units = (ce - co) >> 4;
            uint4 v[8];
            if (to_memory) {
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const std::uint32_t u = lane + 32 * k;
                    if (u < units) v[k] = ld_cv_v4(stage + co + (u << 4));
                }
                for (std::uint32_t g = 0; g < groups; ++g) {
                    char* gm = g == 0 ? mem
                                      : reinterpret_cast<char*>(pcs[g * c.n_pieces + pi].mem) + (co - first.off);
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const std::uint32_t u = lane + 32 * k;
                        if (u < units) st_cs_v4(gm + (u << 4), v[k]);
                    }
                }
            } else {
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const std::uint32_t u = lane + 32 * k;
                    if (u < units) v[k] = *reinterpret_cast<const uint4*>(mem + (u << 4));
                }
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const std::uint32_t u = lane + 32 * k;
                    if (u < units) *reinterpret_cast<uint4*>(stage + co + (u << 4)) = v[k];
                }
            }
        } else {
            for (int q = pi; q < static_cast<int>(c.n_pieces) && pcs[q].off < ce; ++q) {
                const IoPiece pc = pcs[q];
                const std::uint32_t a = max(co, pc.off), b = min(ce, pc.off + pc.bytes);
                for (std::uint32_t o = a + (lane << 4); o < b; o += 512) {
                    if (to_memory) {
                        const uint4 v = ld_cv_v4(stage + o);
                        for (std::uint32_t g = 0; g < groups; ++g)
                            st_cs_v4(reinterpret_cast<char*>(pcs[g * c.n_pieces + q].mem) + (o - pc.off), v);
                    } else {
                        *reinterpret_cast<uint4*>(stage + o) =
                            *reinterpret_cast<const uint4*>(reinterpret_cast<char*>(pc.mem) + (o - pc.off));
                    }
                }
            }
        }
    }
}

// Bulk-copy mover (HBM staging): lane 0 of the group's warp streams the slot
// through a ring of kBulkStages shared-memory chunks: cp.async.bulk
// global->shared completing on the stage's mbarrier, then one
// cp.async.bulk shared->global per destination (replica groups store the
// same chunk to every rank's pool). `phase_bits` carries the mbarrier phases
// from slot to slot. Every wait is bounded by a %globaltimer deadline; on
// expiry the function drains its own copies in flight and returns false.
__device__ bool move_slot_bulk(const IoKernelParams& p, const IoCommand& c, char* stage, bool to_memory,
                               unsigned char* ring, std::uint64_t* bars, std::uint32_t& phase_bits) {
    const IoPiece* pcs = p.pieces + c.first_piece;
    const std::uint32_t groups = (to_memory && c.replicas > 1) ? c.replicas : 1u;
    const unsigned long long deadline = dev::globaltimer_ns() + p.timeout_ns + kMoverGraceNs;
    // chunk cursor over (piece, offset within piece)
    std::uint32_t load_q = 0, load_off = 0;
    std::uint32_t q_of[kBulkStages], off_of[kBulkStages], bytes_of[kBulkStages];
    auto next_chunk = [&](std::uint32_t& q, std::uint32_t& off, std::uint32_t& bytes) -> bool {
        while (load_q < c.n_pieces) {
            const std::uint32_t pb = pcs[load_q].bytes;
            if (load_off < pb) {
                q = load_q;
                off = load_off;
                bytes = min(kBulkChunk, pb - load_off);
                load_off += bytes;
                return true;
            }
            ++load_q;
            load_off = 0;
        }
        return false;
    };
    auto issue_load = [&](std::uint32_t st, std::uint32_t q, std::uint32_t off, std::uint32_t bytes) {
        const IoPiece& pc = pcs[q];
        const char* src = to_memory ? stage + pc.off + off : reinterpret_cast<const char*>(pc.mem) + off;
        dev::mbar_arrive_expect_tx(&bars[st], bytes);
        dev::bulk_g2s(ring + st * kBulkChunk, src, bytes, &bars[st]);
        q_of[st] = q;
        off_of[st] = off;
        bytes_of[st] = bytes;
    };
    std::uint32_t in_flight = 0, head = 0, tail = 0;
    while (in_flight < kBulkStages) {
        std::uint32_t q, off, bytes;
        if (!next_chunk(q, off, bytes)) break;
        issue_load(tail, q, off, bytes);
        tail = (tail + 1) % kBulkStages;
        ++in_flight;
    }
    bool ok = true;
    while (in_flight > 0) {
        const std::uint32_t ph = (phase_bits >> head) & 1u;
        while (!dev::mbar_try_wait(&bars[head], ph)) {
            if (dev::globaltimer_ns() > deadline) {
                ok = false;
                break;
            }
        }
        if (!ok) break;
        phase_bits ^= 1u << head;
        const IoPiece& pc = pcs[q_of[head]];
        for (std::uint32_t g = 0; g < groups; ++g) {
            char* dst = to_memory ? reinterpret_cast<char*>(pcs[g * c.n_pieces + q_of[head]].mem) + off_of[head]
                                  : stage + pc.off + off_of[head];
            dev::bulk_s2g(dst, ring + head * kBulkChunk, bytes_of[head]);
        }
        dev::bulk_commit();
        --in_flight;
        std::uint32_t q, off, bytes;
        if (next_chunk(q, off, bytes)) {
            dev::bulk_wait_read<0>();  // the stage is refilled once its stores have read it
            issue_load(head, q, off, bytes);
            ++in_flight;
        }
        head = (head + 1) % kBulkStages;
    }
    if (!ok) {
        // Loads still in flight complete on their barriers; wait for them (bounded)
        // so no copy lands in shared memory after this CTA moves on.
        for (std::uint32_t k = 0; k < in_flight; ++k) {
            const std::uint32_t st = (head + k) % kBulkStages;
            const unsigned long long t = dev::globaltimer_ns();
            while (!dev::mbar_try_wait(&bars[st], (phase_bits >> st) & 1u) && dev::globaltimer_ns() - t < kMoverGraceNs) {
            }
            phase_bits ^= 1u << st;
        }
    }
    dev::bulk_wait<0>();  // the stores are complete (visible) before the slot changes state
    return ok;
}

// Bus address of [addr, addr + bytes) inside one registered region, 0 if none holds it.
__device__ std::uint64_t region_bus(const IoKernelParams& p, std::uint64_t addr, std::uint64_t bytes) {
    int lo = 0, hi = static_cast<int>(p.n_regions) - 1, at = -1;
    while (lo <= hi) {  // last region starting at or below addr
        const int mid = (lo + hi) >> 1;
        if (p.regions[mid].lo <= addr) {
            at = mid;
            lo = mid + 1;
        } else {
            hi = mid - 1;
        }
    }
    if (at < 0) return 0;
    const DmaRegion& r = p.regions[at];
    if (addr >= r.hi || bytes > r.hi - addr) return 0;
    const std::uint64_t off = addr - r.va;
    if (r.page_shift == 0) return r.bus[0] + off;
    const std::uint64_t first = off >> r.page_shift, last = (off + bytes - 1) >> r.page_shift;
    if (first != last) return 0;  // the range crosses a bus page
    return r.bus[first] + (off & ((1ull << r.page_shift) - 1));
}

// Bus address of 4 KiB page `j` of a direct command (its pieces cover the
// command contiguously in whole pages; checked by fill_direct_list).
__device__ std::uint64_t direct_page_bus(const IoKernelParams& p, const IoCommand& c, std::uint32_t j) {
    const IoPiece* pcs = p.pieces + c.first_piece;
    const std::uint32_t off = j << 12;
    for (std::uint32_t q = 0; q < c.n_pieces; ++q)
        if (off >= pcs[q].off && off - pcs[q].off < pcs[q].bytes) return region_bus(p, pcs[q].mem + (off - pcs[q].off), 4096);
    return 0;
}

// Decides whether read `c` can be served by drive DMA straight into its
// destination pages and, if so, writes the bus address of each of its pages
// into `list` (the slot's direct PRP-list page). Needs: no transform, one
// destination group, pieces that tile [0, bytes) in order in whole 4 KiB
// pages at 4 KiB-aligned addresses, each page inside a registered region.
__device__ bool fill_direct_list(const IoKernelParams& p, const IoCommand& c, std::uint64_t* list) {
    if (p.n_regions == 0 || p.phase != kPhaseFull || c.opcode != nvme::kOpRead || c.transform != kXformNone ||
        c.replicas > 1 || (c.bytes & 4095u) != 0 || c.bytes > 512u * 4096u)
        return false;
    const IoPiece* pcs = p.pieces + c.first_piece;
    std::uint32_t next = 0, j = 0;
    for (std::uint32_t q = 0; q < c.n_pieces; ++q) {
        const IoPiece pc = pcs[q];
        if (pc.off != next || (pc.bytes & 4095u) != 0 || (pc.mem & 4095u) != 0) return false;
        for (std::uint32_t k = 0; k < pc.bytes; k += 4096) {
            const std::uint64_t bus = region_bus(p, pc.mem + k, 4096);
            if (bus == 0) return false;
            list[j++] = bus;
        }
        next += pc.bytes;
    }
    return next == c.bytes;
}

struct Shared {
    bool direct[kMaxSlots];  // the slot's read is DMA'd straight into its destination
    volatile int state[kMaxSlots];
    int cmd[kMaxSlots];
    std::uint32_t pending[kMaxSlots];
    std::uint32_t status[kMaxSlots];
    unsigned long long t0[kMaxSlots];
    QueueCursor cur[kMaxDevices];
    std::uint32_t inflight_dev[kMaxDevices];
    volatile int ready_q[kMaxSlots];
    volatile std::uint32_t rq_tail;  // written by the engine only
    std::uint32_t rq_claim;          // advanced by mover-group leaders (atomicCAS)
    volatile int done;
    volatile int group_slot[kMoverGroups];
    std::uint32_t error;
    alignas(8) std::uint64_t bars[kMoverGroups][kBulkStages];  // bulk movers' ring barriers
};

__device__ void push_ready(Shared& sh, int s, int slots) {
    sh.ready_q[sh.rq_tail % slots] = s;
    __threadfence_block();
    sh.rq_tail = sh.rq_tail + 1;
}

// Resolves command `ci` into slot `s` and writes its SQEs (one per device /
// extent / MDTS piece) into this lease's queues; the slot becomes INFLIGHT.
// Returns false (and the status in *err) when the command cannot be resolved.
__device__ bool issue_cmd(const IoKernelParams& p, Shared& sh, int ci, int s, std::uint32_t lease,
                          unsigned long long now, std::uint32_t* touched, std::uint32_t* err) {
    const std::uint64_t lease_slot0 = static_cast<std::uint64_t>(lease) * p.slots_per_lease;
    const IoCommand c = p.cmds[ci];
    SubCmd sub[kMaxSub];
    const int n = resolve_cmd(p, c, sub, err);
    if (n == 0) return false;
    const std::uint64_t slot_index = lease_slot0 + s;
    const std::uint64_t* pages = p.page_bus + slot_index * (p.slot_bytes >> 12);
    // Direct read: PRPs name the destination pages (list written for this command).
    const bool direct = p.direct_lists && fill_direct_list(p, c, p.direct_lists + slot_index * 512);
    const std::uint64_t list_bus = direct ? p.direct_list_bus[slot_index] : p.list_bus[slot_index];
    sh.direct[s] = direct;
    for (int k = 0; k < n; ++k) {
        const std::uint32_t dv = sub[k].device;
        const DevDevice& d = p.devices[dv];
        const nvme::QueuePairView& q = d.queues[lease];
        const std::uint32_t page0 = sub[k].off >> 12;
        const std::uint64_t prp1 = (direct ? direct_page_bus(p, c, page0) : pages[page0]) + (sub[k].off & 4095u);
        const std::uint32_t extra = nvme::prp_extra_pages(prp1 & 4095u, sub[k].bytes);
        std::uint64_t prp2 = 0;
        if (extra == 1)
            prp2 = direct ? direct_page_bus(p, c, page0 + 1) : pages[page0 + 1];
        else if (extra > 1)
            prp2 = list_bus + 8ull * (page0 + 1);
        nvme::Sqe e;
        nvme::build_rw_sqe(e, static_cast<std::uint8_t>(c.opcode), static_cast<std::uint16_t>(s * kMaxSub + k), d.nsid,
                           sub[k].lba, sub[k].bytes >> d.lba_shift, prp1, prp2);
        uint4* dst = reinterpret_cast<uint4*>(q.sq + sh.cur[dv].sq_tail);
        const uint4* src = reinterpret_cast<const uint4*>(&e);
#pragma unroll
        for (int w = 0; w < 4; ++w) dst[w] = src[w];
        sh.cur[dv].sq_tail = (sh.cur[dv].sq_tail + 1) % q.depth;
        sh.inflight_dev[dv] += 1;
        *touched |= 1u << dv;
    }
    sh.pending[s] = n;
    sh.t0[s] = now;
    sh.state[s] = S_INFLIGHT;
    if (p.timing) p.timing[4ull * ci + 1] = now;
    return true;
}

// One doorbell write. A doorbell in host memory (emulated drive) takes a
// system-scope release store. A controller register in BAR0 takes an .mmio
// store (performed exactly once, never merged or served from a cache), after a
// system-scope fence that orders the ring accesses before it (a relaxed .mmio
// store orders nothing by itself).
__device__ __forceinline__ void write_doorbell(const nvme::QueuePairView& q, std::uint32_t* db, std::uint32_t v) {
    if (q.flags & nvme::kQueueMmioDoorbells) {
        asm volatile("fence.sc.sys;" ::: "memory");
        asm volatile("st.mmio.relaxed.sys.global.u32 [%0], %1;" ::"l"(db), "r"(v) : "memory");
    } else {
        st_release_sys(db, v);
    }
}

// SQEs before the tail doorbells (system scope: the controller is a peer).
__device__ void ring_doorbells(const IoKernelParams& p, Shared& sh, std::uint32_t lease, std::uint32_t touched) {
    if (!touched) return;
    __threadfence_system();
    for (std::uint32_t d = 0; d < p.n_devices; ++d)
        if (touched & (1u << d)) {
            const nvme::QueuePairView& q = p.devices[d].queues[lease];
            write_doorbell(q, q.sq_doorbell, sh.cur[d].sq_tail);
        }
}

// Split completion, submit phase: fill this lease's slots with read commands,
// ring the doorbells once and return without waiting.
__device__ void engine_submit_phase(const IoKernelParams& p, Shared& sh, std::uint32_t lease, int S) {
    const unsigned long long now = globaltimer_ns();
    std::uint32_t touched = 0;
    bool exhausted = false;
    for (int s = 0; s < S && !exhausted; ++s) {
        for (;;) {
            const std::uint32_t ci = atomicAdd(p.cursor, 1u);
            if (ci >= p.n_cmds) {
                exhausted = true;
                break;
            }
            if (p.timing) p.timing[4ull * ci + 0] = now;
            sh.cmd[s] = static_cast<int>(ci);
            sh.status[s] = 0;
            std::uint32_t err = 0;
            if (issue_cmd(p, sh, static_cast<int>(ci), s, lease, now, &touched, &err)) break;
            p.cmd_status[ci] = err;  // unresolvable: report it and claim another for this slot
            sh.cmd[s] = -1;
        }
    }
    ring_doorbells(p, sh, lease, touched);
}

// Engine: everything that touches the queues. Runs on warp 0, lane 0.
__device__ void engine_loop(const IoKernelParams& p, Shared& sh, std::uint32_t lease, int S) {
    bool exhausted = false;
    unsigned idle = 0;
    unsigned long long last_progress = globaltimer_ns();
    for (;;) {
        bool progressed = false;
        std::uint32_t touched = 0;
        const unsigned long long now = globaltimer_ns();
        // (a) claim and submit
        for (int s = 0; s < S; ++s) {
            int st = sh.state[s];
            while (st == S_FREE && !exhausted) {
                const std::uint32_t ci = atomicAdd(p.cursor, 1u);
                if (ci >= p.n_cmds) {
                    exhausted = true;
                    break;
                }
                progressed = true;
                if (p.timing) p.timing[4ull * ci + 0] = now;
                sh.cmd[s] = static_cast<int>(ci);
                sh.status[s] = 0;
                if (p.cmds[ci].opcode == nvme::kOpWrite) {
                    sh.state[s] = st = S_GATHER;
                    push_ready(sh, s, S);
                } else {
                    sh.state[s] = st = S_SUBMIT;
                }
            }
            if (st != S_SUBMIT) continue;
            const int ci = sh.cmd[s];
            std::uint32_t err = 0;
            if (!issue_cmd(p, sh, ci, s, lease, now, &touched, &err)) {
                p.cmd_status[ci] = err;
                sh.state[s] = S_FREE;
                progressed = true;
                --s;  // refill this slot
                continue;
            }
            progressed = true;
        }
        ring_doorbells(p, sh, lease, touched);
        // (b) drain completions
        for (std::uint32_t d = 0; d < p.n_devices; ++d) {
            if (sh.inflight_dev[d] == 0) continue;
            const nvme::QueuePairView& q = p.devices[d].queues[lease];
            bool got = false;
            for (std::uint32_t k = 0; k < q.depth; ++k) {
                const std::uint32_t dw3 = ld_acquire_sys(&q.cq[sh.cur[d].cq_head].dw3);
                if (nvme::cqe_phase(dw3) != sh.cur[d].phase) break;
                got = true;
                const int s = nvme::cqe_cid(dw3) / kMaxSub;
                const std::uint32_t st = nvme::cqe_status(dw3);
                if (s < S && (sh.state[s] == S_INFLIGHT || sh.state[s] == S_POISON) && sh.pending[s] > 0) {
                    sh.pending[s] -= 1;
                    if (st != 0 && sh.status[s] == 0) sh.status[s] = kCmdNvme | (st & 0xFFFFu);
                }
                if (sh.inflight_dev[d] > 0) sh.inflight_dev[d] -= 1;
                sh.cur[d].cq_head = (sh.cur[d].cq_head + 1) % q.depth;
                if (sh.cur[d].cq_head == 0) sh.cur[d].phase ^= 1u;
            }
            if (got) {
                write_doorbell(q, q.cq_doorbell, sh.cur[d].cq_head);
                progressed = true;
            }
        }
        // (c) completions, deadlines, termination
        const unsigned long long t1 = globaltimer_ns();
        bool busy = false, only_poison = true;
        for (int s = 0; s < S; ++s) {
            const int st = sh.state[s];
            if (st == S_INFLIGHT) {
                const int ci = sh.cmd[s];
                if (sh.pending[s] == 0) {
                    if (p.timing) p.timing[4ull * ci + 2] = t1;
                    if (sh.status[s] == 0 && p.cmds[ci].opcode == nvme::kOpRead && !sh.direct[s]) {
                        sh.state[s] = S_READY;
                        push_ready(sh, s, S);
                    } else {  // written, failed, or read straight into its destination
                        p.cmd_status[ci] = sh.status[s];
                        if (p.timing) p.timing[4ull * ci + 3] = t1;
                        sh.state[s] = S_FREE;
                    }
                    progressed = true;
                } else if (t1 - sh.t0[s] > p.timeout_ns) {
                    p.cmd_status[ci] = kCmdTimeout;
                    sh.state[s] = S_POISON;  // the controller may still write this slot
                    progressed = true;
                }
            } else if (st == S_POISON && sh.pending[s] == 0) {
                sh.state[s] = S_FREE;  // late completions drained; slot reusable
            }
            const int now_st = sh.state[s];
            if (now_st != S_FREE) busy = true;
            if (now_st != S_FREE && now_st != S_POISON) only_poison = false;
        }
        if (progressed) {
            idle = 0;
            last_progress = t1;
        }
        if (exhausted && (!busy || only_poison)) break;
        // Failsafe: nothing moved for a whole deadline (every command in flight
        // reaches its own deadline sooner, which counts as progress), e.g.
        // movers wedged: stop.
        if (t1 - last_progress > p.timeout_ns + kEngineGraceNs) {
            atomicOr(&sh.error, 1u);
            break;
        }
        if (!progressed) __nanosleep(++idle < 64 ? 64 : 512);
    }
    sh.done = 1;
    __threadfence_block();
}

template <int W, bool BULK>
__device__ void mover_loop(const IoKernelParams& p, Shared& sh, std::uint32_t lease, int S, int group, int gwarp,
                           int lane, unsigned char* ring) {
    const bool leader = gwarp == 0 && lane == 0;
    const int bar_id = 1 + group;
    const std::uint64_t lease_slot0 = static_cast<std::uint64_t>(lease) * p.slots_per_lease;
    std::uint32_t phase_bits = 0;  // bulk ring barrier phases (leader lane)
    for (;;) {
        if (leader) {
            int got = -1;
            const unsigned long long t0 = dev::globaltimer_ns();
            for (;;) {
                const std::uint32_t h = *reinterpret_cast<volatile std::uint32_t*>(&sh.rq_claim);
                if (h != sh.rq_tail) {
                    if (atomicCAS(&sh.rq_claim, h, h + 1) == h) {
                        got = sh.ready_q[h % S];
                        break;
                    }
                    continue;
                }
                if (sh.done) break;
                if (dev::globaltimer_ns() - t0 > p.timeout_ns + kMoverGraceNs) {
                    atomicOr(&sh.error, 2u);  // the engine went quiet past its own failsafe
                    break;
                }
                __nanosleep(128);
            }
            sh.group_slot[group] = got;
            __threadfence_block();
        }
        __syncwarp();
        if (W > 1) named_barrier(bar_id, W * 32);
        const int s = sh.group_slot[group];
        if (s < 0) break;
        const int ci = sh.cmd[s];
        const bool to_memory = sh.state[s] == S_READY;
        char* stage = p.staging_dev + (lease_slot0 + s) * static_cast<std::uint64_t>(p.slot_bytes);
        const IoCommand c = p.cmds[ci];
        bool moved = true;
        if (BULK && c.transform == kXformNone) {
            if (lane == 0) moved = move_slot_bulk(p, c, stage, to_memory, ring, sh.bars[group], phase_bits);
        } else {
            move_slot<W>(p, c, stage, to_memory, gwarp, lane);
        }
        if (!to_memory) __threadfence_system();  // gathered bytes visible to the controller
        __syncwarp();
        if (W > 1) named_barrier(bar_id, W * 32);
        if (leader) {
            if (!moved) {
                atomicOr(&sh.error, 4u);
                p.cmd_status[ci] = kCmdTimeout;
                sh.state[s] = S_FREE;
            } else if (to_memory) {
                p.cmd_status[ci] = kCmdOk;
                if (p.timing) p.timing[4ull * ci + 3] = dev::globaltimer_ns();
                sh.state[s] = S_FREE;
            } else {
                sh.state[s] = S_SUBMIT;
            }
            __threadfence_block();
        }
    }
}

}  // namespace

template <int W, bool BULK>
__global__ void __launch_bounds__(32 * (1 + kMoverGroups * W), 1) nvme_io_kernel(const IoKernelParams p) {
    __shared__ Shared sh;
    extern __shared__ __align__(128) unsigned char bulk_ring[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const std::uint32_t lease = p.lease_ids[blockIdx.x];
    const int S = static_cast<int>(p.slots_per_lease);
    if (tid == 0) {
        for (std::uint32_t d = 0; d < p.n_devices; ++d) {
            sh.cur[d] = p.devices[d].cursors[lease];
            sh.inflight_dev[d] = 0;
        }
        for (int s = 0; s < kMaxSlots; ++s) {
            sh.state[s] = S_FREE;
            sh.pending[s] = 0;
            sh.cmd[s] = -1;
            sh.direct[s] = false;
        }
        sh.rq_tail = 0;
        sh.rq_claim = 0;
        sh.done = 0;
        sh.error = 0;
        if (BULK) {
            for (int g = 0; g < kMoverGroups; ++g)
                for (std::uint32_t k = 0; k < kBulkStages; ++k) dev::mbar_init(&sh.bars[g][k], 1);
            dev::fence_barrier_init();
        }
    }
    if (tid == 0 && p.phase == kPhaseDrain) {
        const LeaseCarry& k = p.carry[blockIdx.x];
        for (int s = 0; s < S; ++s) {
            if (k.cmd[s] < 0) continue;
            sh.cmd[s] = k.cmd[s];
            sh.pending[s] = k.pending[s];
            sh.status[s] = k.status[s];
            sh.t0[s] = k.t0[s];
            sh.state[s] = S_INFLIGHT;
        }
        for (std::uint32_t d = 0; d < p.n_devices; ++d) sh.inflight_dev[d] = k.inflight_dev[d];
    }
    __syncthreads();
    if (p.phase == kPhaseSubmit) {
        if (tid == 0) {
            engine_submit_phase(p, sh, lease, S);
            LeaseCarry& k = p.carry[blockIdx.x];
            for (int s = 0; s < kMaxSlots; ++s) {
                const bool used = s < S && sh.state[s] == S_INFLIGHT;
                k.cmd[s] = used ? sh.cmd[s] : -1;
                k.pending[s] = used ? sh.pending[s] : 0;
                k.status[s] = 0;
                k.t0[s] = used ? sh.t0[s] : 0;
            }
            for (std::uint32_t d = 0; d < static_cast<std::uint32_t>(kMaxDevices); ++d)
                k.inflight_dev[d] = d < p.n_devices ? sh.inflight_dev[d] : 0;
            // the queues stay owned by the commands in flight until the drain phase
            for (std::uint32_t d = 0; d < p.n_devices; ++d) {
                QueueCursor c = sh.cur[d];
                c.dirty = 0;
                p.devices[d].cursors[lease] = c;
            }
        }
        return;
    }
    if (warp == 0) {
        if (lane == 0) engine_loop(p, sh, lease, S);
    } else {
        const int group = (warp - 1) / W;
        const int gwarp = (warp - 1) % W;
        mover_loop<W, BULK>(p, sh, lease, S, group, gwarp, lane,
                            BULK ? bulk_ring + group * kBulkStages * kBulkChunk : nullptr);
    }
    __syncwarp();
    __syncthreads();
    if (tid == 0) {
        bool dirty = false;
        for (int s = 0; s < S; ++s)
            if (sh.state[s] != S_FREE) dirty = true;
        // Commands the engine never finished stay "not run"; their queues are reset.
        if (sh.error) dirty = true;
        for (std::uint32_t d = 0; d < p.n_devices; ++d) {
            QueueCursor c = sh.cur[d];
            c.dirty = (dirty && (sh.inflight_dev[d] > 0 || sh.error)) ? 1u : 0u;
            p.devices[d].cursors[lease] = c;
        }
    }
}

cudaError_t launch_nvme_io(const IoKernelParams& p, std::uint32_t n_leases, cudaStream_t stream) {
    if (n_leases == 0 || p.n_cmds == 0) return cudaSuccess;
    if (p.phase != kPhaseFull && !p.carry) return cudaErrorInvalidValue;
    const bool submit_only = p.phase == kPhaseSubmit;
    if (p.movers == kMoversBulk) {
        static const cudaError_t attr = cudaFuncSetAttribute(
            nvme_io_kernel<1, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kBulkSmemBytes));
        if (attr != cudaSuccess) return attr;
        nvme_io_kernel<1, true><<<n_leases, submit_only ? 32 : kIoThreadsBulk, submit_only ? 0 : kBulkSmemBytes,
                                  stream>>>(p);
    } else {
        nvme_io_kernel<5, false><<<n_leases, submit_only ? 32 : kIoThreads, 0, stream>>>(p);
    }
    return cudaGetLastError();
}

}  // namespace io
}  // namespace tutti
