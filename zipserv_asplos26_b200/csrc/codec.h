// TCA-TBE format constants, shape contracts and exponent arithmetic shared by
// the host encoder and the CUDA kernels.
//
// Format (bit-compatible with the reference, csrc/HostPacker.h:95-183):
//   * W is M x K BF16 row-major, M and K positive multiples of 64.
//   * Global tiles are 64x64, numbered row-major: t = (row/64)*(K/64) + col/64.
//   * A global tile holds 64 small 8x8 tiles numbered
//       s = band*16 + group*4 + column*2 + row_tile
//     (band = 16-row band, group = 16-column block, column = 8-column half,
//     row_tile = 8-row half). Inside a small tile, bit pos = r*8 + c.
//   * An element is "common" when its exponent e lies in [base, base+7); its
//     3-bit code e-base+1 is split over bitmaps b1/b2/b3 and its sign+mantissa
//     byte goes to the `sm` stream. Other elements go whole to the `rare`
//     stream and have code 0.
//   * Per global tile the common count is padded to 16 bytes and the rare
//     count to 8 words; `global` holds the exclusive prefix of the padded
//     counts ((T+1) pairs), `medium` the unpadded per-band offsets inside the
//     tile (4 pairs per tile).
#pragma once
#include <climits>
#include <cstdint>

#if defined(__CUDACC__)
#define ZS_HD __host__ __device__ __forceinline__
#else
#define ZS_HD inline
#endif

namespace zs {

constexpr int kTile = 64;            // global tile edge
constexpr int kSmallPerTile = 64;    // 8x8 small tiles per global tile
constexpr int kTileBitmapBytes = 512;  // one of b1/b2/b3 for one global tile
constexpr int kTileMediumBytes = 32;   // 4 (common, rare) int pairs

// csrc/CodecUtils.h:11-14
ZS_HD bool valid_matrix(int m, int k) {
    return m > 0 && k > 0 && m % 64 == 0 && k % 64 == 0 && int64_t(m) * k <= INT_MAX;
}

// csrc/CodecUtils.h:16-24: int32 offsets everywhere, and the reference's
// grid.y bound (M/64)*Split_K <= 65535 is kept as an API contract.
ZS_HD bool valid_gemm(int m, int n, int k, int split_k) {
    if (!valid_matrix(m, k) || n < 0 || split_k < 1 || (k / 64) % split_k != 0) return false;
    if (int64_t(m) * n > INT_MAX || int64_t(k) * n > INT_MAX) return false;
    return int64_t(m) * n * split_k <= INT_MAX && int64_t(m / 64) * split_k <= 65535;
}

// csrc/CodecUtils.h:26-29: maxima of padded per-tile counts.
ZS_HD bool valid_counts(int common, int rare) {
    return common >= 0 && common <= 4096 && common % 16 == 0 && rare >= 0 && rare <= 4096 &&
           rare % 8 == 0 && common + rare >= 4096;
}

// csrc/CodecUtils.h:31-36: seven consecutive exponents starting in [0, 249].
ZS_HD bool valid_exponents(const int* e) {
    if (!e || e[0] < 0 || e[0] > 249) return false;
    for (int i = 1; i < 7; ++i)
        if (e[i] != e[0] + i) return false;
    return true;
}

// The window [base, base+width) holding the most elements; ties resolve to
// the lowest base (csrc/CodecUtils.h:40-53). Returns -1 for a bad width.
inline int best_window(const uint64_t* counts, int width = 7) {
    if (!counts || width < 1 || width > 7) return -1;
    uint64_t sum = 0;
    for (int i = 0; i < width; ++i) sum += counts[i];
    uint64_t best = sum;
    int base = 0;
    for (int b = 1; b + width <= 256; ++b) {
        sum += counts[b + width - 1];
        sum -= counts[b - 1];
        if (sum > best) best = sum, base = b;
    }
    return base;
}

// Exponent field of a common element: (start_exp + code) mod 256, shifted to
// bit 7. start_exp = base - 1 (mod 256), so base 0 stores 255 and the 8-bit
// wrap matters (csrc/CodecUtils.h:55-62).
ZS_HD uint16_t exponent_field(uint8_t start_exp, uint8_t code) {
    return uint16_t(uint8_t(start_exp + code)) << 7;
}

// Byte lengths of the seven ABI buffers given the global offsets table.
struct PackedLengths {
    uint64_t sm, rare, bitmap, medium, global;
};
inline PackedLengths packed_lengths(const int32_t* global, int tiles) {
    return {uint64_t(global[2 * tiles]), uint64_t(global[2 * tiles + 1]) * 2,
            uint64_t(tiles) * 512, uint64_t(tiles) * 32, (uint64_t(tiles) + 1) * 8};
}

}  // namespace zs
