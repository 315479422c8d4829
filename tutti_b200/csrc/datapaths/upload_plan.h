#pragma once
// Host -> device copies an operation owes, coalesced into as few copies as possible.
//
// Each upload names the allocation it writes into. Uploads of one allocation
// are sorted by address, and neighbours at most `max_gap` bytes apart become
// one run; the gap between them is zero-filled (it belongs to no object, e.g.
// alignment padding between bump-allocated extent arrays). Runs never span two
// allocations: separately allocated ranges may be adjacent in the address
// space, but one copy must stay inside one allocation. Later uploads to the
// same bytes win (a run is built in submission order within equal addresses).

#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <vector>

namespace tutti {

struct DeviceUpload {
    const char* alloc = nullptr;  // base of the allocation `dst` lies in
    char* dst = nullptr;
    std::vector<char> bytes;
};

struct UploadRun {
    char* dst = nullptr;
    std::vector<char> bytes;
};

inline std::vector<UploadRun> coalesce_uploads(std::vector<DeviceUpload> ups, std::size_t max_gap) {
    std::stable_sort(ups.begin(), ups.end(), [](const DeviceUpload& a, const DeviceUpload& b) {
        return a.alloc != b.alloc ? a.alloc < b.alloc : a.dst < b.dst;
    });
    std::vector<UploadRun> runs;
    for (std::size_t i = 0; i < ups.size();) {
        UploadRun r{ups[i].dst, ups[i].bytes};
        std::size_t k = i + 1;
        while (k < ups.size() && ups[k].alloc == ups[i].alloc && ups[k].dst <= r.dst + r.bytes.size() + max_gap) {
            const std::size_t at = static_cast<std::size_t>(ups[k].dst - r.dst);
            if (r.bytes.size() < at + ups[k].bytes.size()) r.bytes.resize(at + ups[k].bytes.size(), 0);
            std::copy(ups[k].bytes.begin(), ups[k].bytes.end(), r.bytes.begin() + static_cast<std::ptrdiff_t>(at));
            ++k;
        }
        runs.push_back(std::move(r));
        i = k;
    }
    return runs;
}

}  // namespace tutti
