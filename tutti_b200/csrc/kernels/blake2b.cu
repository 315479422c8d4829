// Prefix-key hashing and KV block checksums on sm_100a.
//
// prefix_hash: the chained chunk keys of the semantic index,
//   key_i = BLAKE2b-128(parent_{i-1} || le64(tokens of chunk i)),
// computed on the GPU from token ids already in HBM, one request per quad of
// lanes (the chain is sequential; the four G functions of a round step are not). BLAKE2b follows
// RFC 7693 (unkeyed, digest length 16): the SHA-512 initial values, the
// ten-row message schedule, rotations 32/24/16/63, 12 rounds, the final-block
// flag, and a little-endian byte counter. The parent is 0 bytes (empty
// namespace, first chunk) or 16 bytes (a previous key), so every 128-byte
// message block is a run of 8-byte words.
//
// checksum: an order-sensitive 64-bit digest of each (src, bytes) item,
// sum over 8-byte words w_i of fmix64(w_i xor (i * 0x9E3779B97F4A7C15)) mod 2^64,
// where fmix64 is the MurmurHash3 64-bit finaliser. The sum makes it a
// parallel reduction at HBM speed; it detects corruption of restored KV
// without routing payload through the host (the reference never checksums
// payload for that reason: storage_object_store.h:280-320).

#include "ops_kernels.h"

namespace tutti {
namespace ops {

namespace {

__constant__ std::uint64_t kIV[8] = {0x6a09e667f3bcc908ull, 0xbb67ae8584caa73bull, 0x3c6ef372fe94f82bull,
                                     0xa54ff53a5f1d36f1ull, 0x510e527fade682d1ull, 0x9b05688c2b3e6c1full,
                                     0x1f83d9abfb41bd6bull, 0x5be0cd19137e2179ull};

// The message schedule, evaluated at compile time: with every round unrolled,
// each m[...] index is a constant and the message block stays in registers.
__host__ __device__ constexpr std::uint8_t sigma_of(int r, int i) {
    constexpr std::uint8_t t[10][16] = {
    {0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15}, {14, 10, 4, 8, 9, 15, 13, 6, 1, 12, 0, 2, 11, 7, 5, 3},
    {11, 8, 12, 0, 5, 2, 15, 13, 10, 14, 3, 6, 7, 1, 9, 4}, {7, 9, 3, 1, 13, 12, 11, 14, 2, 6, 5, 10, 4, 0, 15, 8},
    {9, 0, 5, 7, 2, 4, 10, 15, 14, 1, 11, 12, 6, 8, 3, 13}, {2, 12, 6, 10, 0, 11, 8, 3, 4, 13, 7, 5, 15, 14, 1, 9},
    {12, 5, 1, 15, 14, 13, 4, 10, 0, 7, 6, 3, 9, 2, 8, 11}, {13, 11, 7, 14, 12, 1, 3, 9, 5, 0, 15, 4, 8, 6, 2, 10},
    {6, 15, 14, 9, 11, 3, 0, 8, 12, 2, 13, 7, 1, 4, 10, 5}, {10, 2, 8, 4, 7, 6, 1, 5, 15, 11, 9, 14, 3, 12, 13, 0}};
    return t[r][i];
}
template <int R, int I>
struct Sig {
    static constexpr int value = sigma_of(R % 10, I);
};

__device__ __forceinline__ std::uint64_t rotr(std::uint64_t x, int n) { return (x >> n) | (x << (64 - n)); }

// One request per quad of lanes. Lane q of the quad holds column q of the
// 4x4 state (v[q], v[4+q], v[8+q], v[12+q]), so the four G functions of a
// column step run in parallel; for the diagonal step b, c and d are rotated
// across the quad by 1, 2 and 3 lanes with shuffles and rotated back after.
// The 128-byte message block sits in shared memory (one block per quad), and
// the schedule row of each round is a compile-time constant packed in nibbles.
__host__ __device__ constexpr std::uint64_t sigma_row(int r) {
    std::uint64_t v = 0;
    for (int i = 0; i < 16; ++i) v |= static_cast<std::uint64_t>(sigma_of(r, i)) << (4 * i);
    return v;
}
template <int R>
struct Row {
    static constexpr std::uint64_t value = sigma_row(R % 10);
};

__device__ __forceinline__ void g(std::uint64_t& a, std::uint64_t& b, std::uint64_t& c, std::uint64_t& d,
                                  std::uint64_t x, std::uint64_t y) {
    a = a + b + x;
    d = rotr(d ^ a, 32);
    c = c + d;
    b = rotr(b ^ c, 24);
    a = a + b + y;
    d = rotr(d ^ a, 16);
    c = c + d;
    b = rotr(b ^ c, 63);
}

struct Quad {
    unsigned mask;  // the quad's four lanes
    int base;       // lane index of the quad's lane 0
    int q;          // this lane's column
};

template <int R>
__device__ __forceinline__ void round_quad(std::uint64_t& a, std::uint64_t& b, std::uint64_t& c, std::uint64_t& d,
                                           const std::uint64_t* m, const Quad& k) {
    constexpr std::uint64_t row = Row<R>::value;
    g(a, b, c, d, m[(row >> (8 * k.q)) & 15], m[(row >> (8 * k.q + 4)) & 15]);
    std::uint64_t b1 = __shfl_sync(k.mask, b, k.base + ((k.q + 1) & 3));
    std::uint64_t c1 = __shfl_sync(k.mask, c, k.base + ((k.q + 2) & 3));
    std::uint64_t d1 = __shfl_sync(k.mask, d, k.base + ((k.q + 3) & 3));
    g(a, b1, c1, d1, m[(row >> (32 + 8 * k.q)) & 15], m[(row >> (36 + 8 * k.q)) & 15]);
    b = __shfl_sync(k.mask, b1, k.base + ((k.q + 3) & 3));
    c = __shfl_sync(k.mask, c1, k.base + ((k.q + 2) & 3));
    d = __shfl_sync(k.mask, d1, k.base + ((k.q + 1) & 3));
}

// h0 = h[q], h1 = h[4+q] of this lane.
__device__ __forceinline__ void compress_quad(std::uint64_t& h0, std::uint64_t& h1, const std::uint64_t* m,
                                              std::uint64_t t, bool last, const Quad& k) {
    std::uint64_t a = h0, b = h1, c = kIV[k.q], d = kIV[4 + k.q];
    if (k.q == 0) d ^= t;           // v[12]: byte counter (far below 2^64 bytes here)
    if (k.q == 2 && last) d = ~d;   // v[14]: final-block flag
    round_quad<0>(a, b, c, d, m, k);
    round_quad<1>(a, b, c, d, m, k);
    round_quad<2>(a, b, c, d, m, k);
    round_quad<3>(a, b, c, d, m, k);
    round_quad<4>(a, b, c, d, m, k);
    round_quad<5>(a, b, c, d, m, k);
    round_quad<6>(a, b, c, d, m, k);
    round_quad<7>(a, b, c, d, m, k);
    round_quad<8>(a, b, c, d, m, k);
    round_quad<9>(a, b, c, d, m, k);
    round_quad<10>(a, b, c, d, m, k);
    round_quad<11>(a, b, c, d, m, k);
    h0 ^= a ^ c;
    h1 ^= b ^ d;
}

// BLAKE2b-128 of the parent (0 or 2 words p0, p1) followed by `n` little-endian
// int64 tokens; every lane of the quad returns the digest.
__device__ void hash_chunk_quad(std::uint64_t p0, std::uint64_t p1, int parent_words, const std::int64_t* tok,
                                std::uint32_t n, std::uint64_t* m, const Quad& k, std::uint64_t out[2]) {
    std::uint64_t h0 = kIV[k.q], h1 = kIV[4 + k.q];
    if (k.q == 0) h0 ^= 0x01010000ull ^ 16ull;  // depth 1, fanout 1, no key, 16-byte digest
    const std::uint64_t total_words = parent_words + n;
    const std::uint64_t total_bytes = total_words * 8;
    std::uint64_t w = 0;
    if (total_words == 0) {
#pragma unroll
        for (int j = 0; j < 4; ++j) m[k.q + 4 * j] = 0;
        __syncwarp(k.mask);
        compress_quad(h0, h1, m, 0, true, k);
    }
    while (w < total_words) {
        const std::uint64_t remaining = total_words - w;
        const int take = remaining > 16 ? 16 : static_cast<int>(remaining);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = k.q + 4 * j;
            const std::uint64_t idx = w + i;
            std::uint64_t val = 0;
            if (i < take)
                val = idx < static_cast<std::uint64_t>(parent_words)
                          ? (idx == 0 ? p0 : p1)
                          : static_cast<std::uint64_t>(tok[idx - parent_words]);
            m[i] = val;
        }
        __syncwarp(k.mask);
        w += take;
        const bool last = w == total_words;
        compress_quad(h0, h1, m, last ? total_bytes : w * 8, last, k);
        __syncwarp(k.mask);  // the block is read by every lane before the next one overwrites it
    }
    out[0] = __shfl_sync(k.mask, h0, k.base);      // h[0]: lane 0's h[q]
    out[1] = __shfl_sync(k.mask, h0, k.base + 1);  // h[1]: lane 1's h[q]
}

constexpr int kHashThreads = 128;  // 32 requests per CTA

__global__ void __launch_bounds__(kHashThreads) prefix_hash_kernel(
    const std::int64_t* tokens, const std::int64_t* starts, const std::int64_t* lengths, const std::uint8_t* parents,
    const std::int32_t* parent_len, const std::int64_t* key_offsets, std::uint8_t* keys, std::uint32_t requests,
    std::uint32_t chunk_tokens) {
    __shared__ std::uint64_t msg[kHashThreads / 4][16];
    const int lane = threadIdx.x & 31;
    Quad k;
    k.q = lane & 3;
    k.base = lane & ~3;
    k.mask = 0xFu << k.base;
    const std::uint32_t r = (blockIdx.x * blockDim.x + threadIdx.x) >> 2;
    if (r >= requests) return;  // the whole quad leaves together
    std::uint64_t* m = msg[threadIdx.x >> 2];
    const std::int64_t* tok = tokens + starts[r];
    const std::int64_t nchunks = lengths[r] / chunk_tokens;
    std::uint64_t p0 = 0, p1 = 0;
    int pw = 0;
    if (parent_len[r] == 16) {
        const std::uint64_t* p = reinterpret_cast<const std::uint64_t*>(parents + 16ull * r);
        p0 = p[0];
        p1 = p[1];
        pw = 2;
    }
    std::uint64_t* out = reinterpret_cast<std::uint64_t*>(keys + 16ull * key_offsets[r]);
    for (std::int64_t c = 0; c < nchunks; ++c) {
        std::uint64_t d[2];
        hash_chunk_quad(p0, p1, pw, tok + c * chunk_tokens, chunk_tokens, m, k, d);
        if (k.q == 0) {
            out[2 * c] = d[0];
            out[2 * c + 1] = d[1];
        }
        p0 = d[0];
        p1 = d[1];
        pw = 2;
    }
}

__device__ __forceinline__ std::uint64_t fmix64(std::uint64_t k) {
    k ^= k >> 33;
    k *= 0xff51afd7ed558ccdull;
    k ^= k >> 33;
    k *= 0xc4ceb9fe1a85ec53ull;
    k ^= k >> 33;
    return k;
}

__global__ void __launch_bounds__(256) checksum_kernel(const CopyItem* items, std::uint32_t n, std::uint64_t* out) {
    __shared__ std::uint64_t part[8];
    for (std::uint32_t i = blockIdx.x; i < n; i += gridDim.x) {
        const CopyItem it = items[i];
        const std::uint64_t* p = reinterpret_cast<const std::uint64_t*>(it.src);
        const std::uint64_t words = it.bytes / 8;
        std::uint64_t acc = 0;
        for (std::uint64_t w = threadIdx.x; w < words; w += blockDim.x)
            acc += fmix64(p[w] ^ (w * 0x9E3779B97F4A7C15ull));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
        __syncthreads();
        if (threadIdx.x == 0) {
            std::uint64_t s = 0;
            for (int k = 0; k < static_cast<int>(blockDim.x >> 5); ++k) s += part[k];
            out[i] = s;
        }
        __syncthreads();
    }
}

// Items of one size: warps take 16 KiB segments of items (all warps busy
// however few or large the items are), read them with 16-byte loads four deep
// and add each segment's sum into its item's digest. Sums commute, so the
// digest equals checksum_kernel's.
constexpr std::uint64_t kSegBytes = 16384;

__global__ void __launch_bounds__(256) checksum_uniform_kernel(const CopyItem* items, std::uint32_t n,
                                                               std::uint64_t bytes, std::uint64_t* out) {
    const int lane = threadIdx.x & 31;
    const std::uint64_t segs = (bytes + kSegBytes - 1) / kSegBytes;
    const std::uint64_t units = std::uint64_t(n) * segs;
    const std::uint64_t warps = std::uint64_t(gridDim.x) * (blockDim.x >> 5);
    const std::uint64_t words = bytes / 8;
    for (std::uint64_t u = std::uint64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); u < units;
         u += warps) {
        const std::uint64_t i = u / segs, seg = u % segs;
        const std::uint64_t* p = reinterpret_cast<const std::uint64_t*>(items[i].src);
        const std::uint64_t w0 = seg * (kSegBytes / 8);
        const std::uint64_t w1 = min(words, w0 + kSegBytes / 8);
        std::uint64_t acc = 0;
        // pairs of words (16 bytes) per lane, 4 in flight
        std::uint64_t w = w0 + 2 * lane;
        for (; w + 2 * 32 * 3 + 1 < w1; w += 2 * 32 * 4) {
            uint4 v[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = *reinterpret_cast<const uint4*>(p + w + 64 * k);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const std::uint64_t a = (std::uint64_t(v[k].y) << 32) | v[k].x;
                const std::uint64_t b = (std::uint64_t(v[k].w) << 32) | v[k].z;
                const std::uint64_t wi = w + 64 * k;
                acc += fmix64(a ^ (wi * 0x9E3779B97F4A7C15ull)) + fmix64(b ^ ((wi + 1) * 0x9E3779B97F4A7C15ull));
            }
        }
        for (; w < w1; w += 64) {
            acc += fmix64(p[w] ^ (w * 0x9E3779B97F4A7C15ull));
            if (w + 1 < w1) acc += fmix64(p[w + 1] ^ ((w + 1) * 0x9E3779B97F4A7C15ull));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) atomicAdd(reinterpret_cast<unsigned long long*>(out + i), static_cast<unsigned long long>(acc));
    }
}

}  // namespace

cudaError_t launch_checksum_uniform(const CopyItem* items, std::uint32_t n, std::uint64_t bytes, std::uint64_t* out,
                                    cudaStream_t stream) {
    if (!n) return cudaSuccess;
    if (bytes % 16) return cudaErrorInvalidValue;
    cudaError_t e = cudaMemsetAsync(out, 0, std::size_t(n) * sizeof(std::uint64_t), stream);
    if (e != cudaSuccess) return e;
    const std::uint64_t units = std::uint64_t(n) * ((bytes + kSegBytes - 1) / kSegBytes);
    const unsigned grid = static_cast<unsigned>(std::max<std::uint64_t>(1, std::min<std::uint64_t>((units + 7) / 8, 148 * 8)));
    checksum_uniform_kernel<<<grid, 256, 0, stream>>>(items, n, bytes, out);
    return cudaGetLastError();
}

cudaError_t launch_prefix_hash(const std::int64_t* tokens, const std::int64_t* starts, const std::int64_t* lengths,
                               const std::uint8_t* parents, const std::int32_t* parent_len,
                               const std::int64_t* key_offsets, std::uint8_t* keys, std::uint32_t requests,
                               std::uint32_t chunk_tokens, cudaStream_t stream) {
    if (!requests) return cudaSuccess;
    const std::uint64_t threads = 4ull * requests;  // a quad of lanes per request
    prefix_hash_kernel<<<static_cast<unsigned>((threads + kHashThreads - 1) / kHashThreads), kHashThreads, 0, stream>>>(
        tokens, starts, lengths, parents, parent_len, key_offsets, keys, requests, chunk_tokens);
    return cudaGetLastError();
}

cudaError_t launch_checksum(const CopyItem* items, std::uint32_t n, std::uint64_t* out, cudaStream_t stream) {
    if (!n) return cudaSuccess;
    checksum_kernel<<<std::min<std::uint32_t>(n, 148 * 8), 256, 0, stream>>>(items, n, out);
    return cudaGetLastError();
}

}  // namespace ops
}  // namespace tutti
