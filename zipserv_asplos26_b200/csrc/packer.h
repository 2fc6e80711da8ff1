// Host TCA-TBE encoder. Output is byte-identical to the reference encoder
// (csrc/HostPacker.h:95-183) for every input, base and worker count; see
// codec.h for the format.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cstdlib>
#include <memory>

namespace zs {

struct FreeDeleter {
    void operator()(void* p) const noexcept { std::free(p); }
};
template <class T>
using HostBuffer = std::unique_ptr<T, FreeDeleter>;

struct HostPacked {
    HostBuffer<uint8_t> sm;        // sign|mantissa bytes of common elements
    HostBuffer<uint16_t> rare;     // whole BF16 words of rare elements
    HostBuffer<uint64_t> b1, b2, b3;  // code bit planes, 64 words per global tile
    HostBuffer<int32_t> small;     // optional per-small-tile (common, rare) counts
    HostBuffer<int32_t> medium;    // per-band (common, rare) offsets inside a tile
    HostBuffer<int32_t> global;    // exclusive prefix of padded counts, (T+1) pairs
    int tiles = 0, base = 0, max_common = 0, max_rare = 0;

    uint64_t sm_bytes() const { return uint64_t(global.get()[2 * tiles]); }
    uint64_t rare_bytes() const { return uint64_t(global.get()[2 * tiles + 1]) * 2; }
};

// Pack raw BF16 words (host byte order, row-major m x k). base = -1 picks the
// most populated 7-exponent window. workers = 0 picks a count from the
// hardware and the matrix size; the output never depends on it. Throws
// std::invalid_argument on bad arguments and std::bad_alloc on allocation
// failure; nothing is leaked either way.
HostPacked pack_bf16(const void* words, int m, int k, int base = -1,
                     bool include_small = false, unsigned workers = 0);

// Worker count used when workers == 0.
unsigned default_workers(int tiles);

}  // namespace zs
