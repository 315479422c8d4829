// Fused GPU NVMe io kernel for sm_100a.
//
// CTA structure (512 threads):
//   * thread 0 is the queue engine: it claims commands from the global cursor,
//     resolves each command's logical range against the target's extents
//     (device, LBA, extent and MDTS splits), writes SQEs into the CTA's own SQ
//     on every device it touches, rings each SQ tail doorbell once per round,
//     drains CQEs by phase bit (one CQ head doorbell per device per round) and
//     enforces a %globaltimer deadline per command;
//   * all 16 warps then move data for the slots that became ready: staging ->
//     caller memory for reads (the paged scatter), caller memory -> staging for
//     writes (the paged gather) before their SQEs go out.
// Staging reads use ld.global.cv (the controller rewrites a slot between uses),
// caller-memory stores use st.global.cs (streamed, not reused by this kernel).
// Every wait is bounded: a command past its deadline is reported as a timeout
// and its slot is quarantined until its late completions drain; a launch that
// ends with commands still owned by the controller marks the queue dirty so the
// host resets it before the next launch.

#include "io_kernel.h"

namespace tutti {
namespace io {

namespace {

enum SlotStateKind : int { S_FREE = 0, S_INFLIGHT, S_READY, S_GATHER, S_SUBMIT_W, S_POISON };

struct SlotState {
    int cmd;
    int state;
    std::uint32_t pending;   // NVMe commands not yet completed
    std::uint32_t status;    // first error seen
    unsigned long long t0;   // submission time (ns)
    std::uint32_t nsub;
    std::uint32_t pad;
};

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
    asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}

__device__ __forceinline__ uint4 ld_v4(const void* p) {
    return *reinterpret_cast<const uint4*>(p);
}

__device__ __forceinline__ void st_v4(void* p, uint4 v) { *reinterpret_cast<uint4*>(p) = v; }

// Extent containing `pos` (binary search); -1 if none.
__device__ int find_extent(const DevTarget& t, std::uint64_t pos) {
    int lo = 0, hi = static_cast<int>(t.n_extents) - 1;
    while (lo <= hi) {
        int mid = (lo + hi) >> 1;
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
    std::uint32_t off;    // byte offset within the slot
    std::uint32_t bytes;
};

// Resolve a command into NVMe-sized pieces; returns count or 0 with *err set.
__device__ int resolve_cmd(const IoKernelParams& p, const IoCommand& c, SubCmd* out, std::uint32_t* err) {
    if (c.target == 0xFFFFFFFFu) {
        *err = kCmdResolve;
        return 0;
    }
    const DevTarget t = p.targets[c.target];
    if (t.extents == nullptr || c.logical + c.bytes > t.size || c.bytes == 0 || c.bytes > p.slot_bytes) {
        *err = kCmdResolve;
        return 0;
    }
    std::uint64_t pos = c.logical;
    std::uint32_t rem = c.bytes, off = 0;
    int n = 0;
    while (rem > 0) {
        int ei = find_extent(t, pos);
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
        std::uint64_t in_ext = e.logical + e.length - pos;
        std::uint32_t len = rem;
        if (in_ext < len) len = static_cast<std::uint32_t>(in_ext);
        if (d.mdts_bytes < len) len = d.mdts_bytes;
        std::uint64_t phys = e.physical + (pos - e.logical);
        const std::uint64_t lba_mask = (1ull << d.lba_shift) - 1;
        if ((phys & lba_mask) || (len & lba_mask)) {
            *err = kCmdResolve;
            return 0;
        }
        out[n].lba = phys >> d.lba_shift;
        out[n].device = e.device;
        out[n].off = off;
        out[n].bytes = len;
        ++n;
        pos += len;
        off += len;
        rem -= len;
    }
    return n;
}

// Move one slot's data: staging <-> caller memory, warp per 4 KiB chunk.
__device__ void move_slot(const IoKernelParams& p, const IoCommand& c, const char* stage_c, char* stage,
                          bool to_memory, int warp, int lane, int nwarps) {
    const IoPiece* pcs = p.pieces + c.first_piece;
    const std::uint32_t nchunks = (c.bytes + 4095u) >> 12;
    for (std::uint32_t ch = warp; ch < nchunks; ch += nwarps) {
        const std::uint32_t co = ch << 12;
        const std::uint32_t ce = min(co + 4096u, c.bytes);
        // piece containing co (binary search over offsets)
        int lo = 0, hi = static_cast<int>(c.n_pieces) - 1, pi = 0;
        while (lo <= hi) {
            int mid = (lo + hi) >> 1;
            if (pcs[mid].off <= co) {
                pi = mid;
                lo = mid + 1;
            } else {
                hi = mid - 1;
            }
        }
        const IoPiece first = pcs[pi];
        if (first.off <= co && first.off + first.bytes >= ce) {
            // fast path: one piece covers the chunk; 16 B per lane x 8 in flight
            char* mem = reinterpret_cast<char*>(first.mem) + (co - first.off);
            const std::uint32_t units = (ce - co) >> 4;
            if (to_memory) {
                uint4 v[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    std::uint32_t u = lane + 32 * k;
                    if (u < units) v[k] = ld_cv_v4(stage_c + co + (u << 4));
                }
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    std::uint32_t u = lane + 32 * k;
                    if (u < units) st_cs_v4(mem + (u << 4), v[k]);
                }
            } else {
                uint4 v[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    std::uint32_t u = lane + 32 * k;
                    if (u < units) v[k] = ld_v4(mem + (u << 4));
                }
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    std::uint32_t u = lane + 32 * k;
                    if (u < units) st_v4(stage + co + (u << 4), v[k]);
                }
            }
        } else {
            // general path: chunk straddles pieces
            for (int q = pi; q < static_cast<int>(c.n_pieces) && pcs[q].off < ce; ++q) {
                const IoPiece pc = pcs[q];
                std::uint32_t a = max(co, pc.off), b = min(ce, pc.off + pc.bytes);
                char* mem = reinterpret_cast<char*>(pc.mem);
                for (std::uint32_t o = a + (lane << 4); o < b; o += 512) {
                    if (to_memory)
                        st_cs_v4(mem + (o - pc.off), ld_cv_v4(stage_c + o));
                    else
                        st_v4(stage + o, ld_v4(mem + (o - pc.off)));
                }
            }
        }
    }
}

}  // namespace

__global__ void __launch_bounds__(kIoThreads, 1) nvme_io_kernel(const IoKernelParams p) {
    __shared__ SlotState slots[kMaxSlots];
    __shared__ QueueCursor cur[kMaxDevices];
    __shared__ std::uint32_t inflight_dev[kMaxDevices];
    __shared__ int copy_list[kMaxSlots];
    __shared__ int n_copy;
    __shared__ int done;
    __shared__ int exhausted;
    __shared__ int gathered_any;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
    const std::uint32_t lease = p.lease_ids[blockIdx.x];
    const int S = static_cast<int>(p.slots_per_lease);
    const std::uint64_t lease_slot0 = static_cast<std::uint64_t>(lease) * p.slots_per_lease;

    if (tid == 0) {
        for (std::uint32_t d = 0; d < p.n_devices; ++d) {
            cur[d] = p.devices[d].cursors[lease];
            inflight_dev[d] = 0;
        }
        for (int s = 0; s < kMaxSlots; ++s) {
            slots[s].state = S_FREE;
            slots[s].pending = 0;
            slots[s].cmd = -1;
        }
        exhausted = 0;
        done = 0;
    }
    __syncthreads();

    unsigned idle_rounds = 0;
    for (;;) {
        if (tid == 0) {
            n_copy = 0;
            gathered_any = 0;
            bool progressed = false;
            std::uint32_t touched = 0;
            const unsigned long long now = globaltimer_ns();
            // (a) claim and submit
            for (int s = 0; s < S; ++s) {
                SlotState& sl = slots[s];
                while (sl.state == S_FREE && !exhausted) {
                    std::uint32_t ci = atomicAdd(p.cursor, 1u);
                    if (ci >= p.n_cmds) {
                        exhausted = 1;
                        break;
                    }
                    progressed = true;
                    if (p.timing) p.timing[4ull * ci + 0] = now;
                    sl.cmd = static_cast<int>(ci);
                    sl.status = 0;
                    if (p.cmds[ci].opcode == nvme::kOpWrite) {
                        sl.state = S_GATHER;
                        copy_list[n_copy++] = s;
                    } else {
                        sl.state = S_SUBMIT_W;  // reads go straight to submission
                    }
                }
                if (sl.state == S_SUBMIT_W) {
                    const IoCommand c = p.cmds[sl.cmd];
                    SubCmd sub[kMaxSub];
                    std::uint32_t err = 0;
                    int n = resolve_cmd(p, c, sub, &err);
                    if (n == 0) {
                        p.cmd_status[sl.cmd] = err;
                        sl.state = S_FREE;
                        --s;  // refill this slot
                        continue;
                    }
                    const std::uint64_t slot_index = lease_slot0 + s;
                    const std::uint64_t slot_iova = p.staging_iova + slot_index * p.slot_bytes;
                    const std::uint64_t list_iova = p.prp_iova + slot_index * nvme::kMemoryPageBytes;
                    for (int k = 0; k < n; ++k) {
                        const std::uint32_t dv = sub[k].device;
                        const DevDevice& d = p.devices[dv];
                        const nvme::QueuePairView& q = d.queues[lease];
                        const std::uint64_t prp1 = slot_iova + sub[k].off;
                        const std::uint32_t page0 = sub[k].off >> 12;
                        const std::uint32_t extra = nvme::prp_extra_pages(prp1 & 4095u, sub[k].bytes);
                        std::uint64_t prp2 = 0;
                        if (extra == 1)
                            prp2 = slot_iova + (static_cast<std::uint64_t>(page0 + 1) << 12);
                        else if (extra > 1)
                            prp2 = list_iova + 8ull * (page0 + 1);
                        nvme::Sqe e;
                        nvme::build_rw_sqe(e, static_cast<std::uint8_t>(c.opcode),
                                           static_cast<std::uint16_t>(s * kMaxSub + k), d.nsid, sub[k].lba,
                                           sub[k].bytes >> d.lba_shift, prp1, prp2);
                        uint4* dst = reinterpret_cast<uint4*>(q.sq + cur[dv].sq_tail);
                        const uint4* src = reinterpret_cast<const uint4*>(&e);
#pragma unroll
                        for (int w = 0; w < 4; ++w) dst[w] = src[w];
                        cur[dv].sq_tail = (cur[dv].sq_tail + 1) % q.depth;
                        inflight_dev[dv] += 1;
                        touched |= 1u << dv;
                    }
                    sl.nsub = n;
                    sl.pending = n;
                    sl.t0 = now;
                    sl.state = S_INFLIGHT;
                    if (p.timing) p.timing[4ull * sl.cmd + 1] = now;
                }
            }
            if (touched) {
                __threadfence_system();
                for (std::uint32_t d = 0; d < p.n_devices; ++d)
                    if (touched & (1u << d)) st_release_sys(p.devices[d].queues[lease].sq_doorbell, cur[d].sq_tail);
            }
            // (b) drain completions
            for (std::uint32_t d = 0; d < p.n_devices; ++d) {
                if (inflight_dev[d] == 0) continue;
                const nvme::QueuePairView& q = p.devices[d].queues[lease];
                bool got = false;
                for (std::uint32_t k = 0; k < q.depth; ++k) {
                    const std::uint32_t dw3 = ld_acquire_sys(&q.cq[cur[d].cq_head].dw3);
                    if (nvme::cqe_phase(dw3) != cur[d].phase) break;
                    got = true;
                    const std::uint16_t cid = nvme::cqe_cid(dw3);
                    const std::uint32_t st = nvme::cqe_status(dw3);
                    const int s = cid / kMaxSub;
                    if (s < S && (slots[s].state == S_INFLIGHT || slots[s].state == S_POISON) &&
                        slots[s].pending > 0) {
                        slots[s].pending -= 1;
                        if (st != 0 && slots[s].status == 0) slots[s].status = kCmdNvme | (st & 0xFFFFu);
                    }
                    inflight_dev[d] -= inflight_dev[d] > 0 ? 1 : 0;
                    cur[d].cq_head = (cur[d].cq_head + 1) % q.depth;
                    if (cur[d].cq_head == 0) cur[d].phase ^= 1u;
                }
                if (got) {
                    st_release_sys(q.cq_doorbell, cur[d].cq_head);
                    progressed = true;
                }
            }
            // (c) completions and deadlines
            const unsigned long long t1 = globaltimer_ns();
            bool busy = false;
            for (int s = 0; s < S; ++s) {
                SlotState& sl = slots[s];
                if (sl.state == S_INFLIGHT) {
                    if (sl.pending == 0) {
                        if (p.timing) p.timing[4ull * sl.cmd + 2] = t1;
                        const bool is_read = p.cmds[sl.cmd].opcode == nvme::kOpRead;
                        if (sl.status == 0 && is_read) {
                            sl.state = S_READY;
                            copy_list[n_copy++] = s;
                        } else {
                            p.cmd_status[sl.cmd] = sl.status;
                            if (p.timing) p.timing[4ull * sl.cmd + 3] = t1;
                            sl.state = S_FREE;
                        }
                    } else if (t1 - sl.t0 > p.timeout_ns) {
                        p.cmd_status[sl.cmd] = kCmdTimeout;
                        sl.state = S_POISON;  // the controller may still write this slot
                    }
                } else if (sl.state == S_POISON && sl.pending == 0) {
                    sl.state = S_FREE;  // late completions drained; slot reusable
                }
                if (sl.state != S_FREE) busy = true;
            }
            if (exhausted && !busy) done = 1;
            // Only quarantined slots left: stop waiting for them.
            if (exhausted && busy && n_copy == 0) {
                bool only_poison = true;
                for (int s = 0; s < S; ++s)
                    if (slots[s].state != S_FREE && slots[s].state != S_POISON) only_poison = false;
                if (only_poison) done = 1;
            }
            if (progressed || n_copy > 0) {
                idle_rounds = 0;
            } else if (!done) {
                ++idle_rounds;
                __nanosleep(idle_rounds < 64 ? 100 : 1000);
            }
        }
        __syncthreads();
        if (done) break;
        // (d) move data for ready slots
        const int nc = n_copy;
        for (int i = 0; i < nc; ++i) {
            const int s = copy_list[i];
            const SlotState& sl = slots[s];
            const IoCommand c = p.cmds[sl.cmd];
            char* stage = p.staging_dev + (lease_slot0 + s) * static_cast<std::uint64_t>(p.slot_bytes);
            const bool to_memory = sl.state == S_READY;
            move_slot(p, c, stage, stage, to_memory, warp, lane, nwarps);
            if (!to_memory) gathered_any = 1;
        }
        if (nc > 0 && gathered_any) __threadfence_system();  // gathered bytes visible to the controller
        __syncthreads();
        if (tid == 0) {
            const unsigned long long t2 = globaltimer_ns();
            for (int i = 0; i < nc; ++i) {
                SlotState& sl = slots[copy_list[i]];
                if (sl.state == S_READY) {
                    p.cmd_status[sl.cmd] = kCmdOk;
                    if (p.timing) p.timing[4ull * sl.cmd + 3] = t2;
                    sl.state = S_FREE;
                } else if (sl.state == S_GATHER) {
                    sl.state = S_SUBMIT_W;
                }
            }
        }
    }
    if (tid == 0) {
        std::uint32_t dirty = 0;
        for (int s = 0; s < S; ++s)
            if (slots[s].state != S_FREE) dirty = 1;
        for (std::uint32_t d = 0; d < p.n_devices; ++d) {
            QueueCursor c = cur[d];
            c.dirty = (dirty && inflight_dev[d] > 0) ? 1u : 0u;
            p.devices[d].cursors[lease] = c;
        }
    }
}

cudaError_t launch_nvme_io(const IoKernelParams& p, std::uint32_t n_leases, cudaStream_t stream) {
    if (n_leases == 0 || p.n_cmds == 0) return cudaSuccess;
    nvme_io_kernel<<<n_leases, kIoThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace io
}  // namespace tutti
