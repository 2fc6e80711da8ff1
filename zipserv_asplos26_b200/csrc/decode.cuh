// TCA-TBE row decoder shared by the fused GEMM and the standalone decompress
// kernel.
//
// Mapping: one thread owns one matrix row of a 64x64 global tile and rebuilds
// the row's 64 BF16 weights (32 packed 32-bit words, element k in half k&1 of
// word k/2). A warp owns one 16-row band of TWO tiles: lanes 0-15 hold band b
// of one tile and lanes 16-31 band b of the other (lane = tile*16 + rt*8 + r);
// callers place the two tiles' data 64 bytes apart modulo 128 so the two
// half-warps read different shared-memory banks. Inside a band the stream of a pair of
// small tiles (2j, 2j+1) is rows 0..7 of 2j then rows 0..7 of 2j+1: exactly
// the lane order of a 16-lane half, so every stream offset is one byte-packed
// 16-lane prefix sum, done once per K slice for all eight column blocks.
//
// Per row segment (8 elements = one small-tile row):
//   * the three bitmap bytes give the 8 codes as nibbles through a lookup
//     table replicated per lane (bank-conflict free); OR-ing the three
//     lookups gives the "common" flag per nibble, and one multiply by
//     0x11111110 turns those flags into each position's rank among the common
//     elements (nibble-wise prefix sum), which is the byte-permute selector
//     that spreads the compact payload bytes to their positions;
//   * the compact common payload bytes come from one funnel-shift pair;
//   * exponents come from one 8-byte palette indexed by the code nibbles,
//     holding each exponent rotated right by one bit: bit 7 (exponent LSB)
//     is what the low byte takes, bits 0-6 (exponent >> 1) what the high
//     byte takes, so one byte permute serves both byte planes;
//   * the row is written with eight 16-byte stores into a 128-byte-swizzled
//     tile row (the layout the tensor cores and TMA stores read), then one
//     loop over the row's rare bits patches each rare element with one
//     16-bit store: the common-element arithmetic never looks at rares.
// Reference decoder semantics: csrc/L_Kernel.cuh:146-250 and :1022-1143;
// bit-exact results are checked against oracle/oracle.c:oracle_decode.
#pragma once
#include <cstdint>

#include "ptx.cuh"

namespace zs {

constexpr uint32_t kFullMask = 0xFFFFFFFFu;
// The code table is replicated kTableCopies times (lane l reads copy l % 32):
// a warp's lookups never meet bank conflicts.
constexpr int kTableCopies = 32;
constexpr int kCodeTableBytes = 256 * kTableCopies * 4;  // per bitmap byte x per copy
constexpr int kTableBytes = kCodeTableBytes;
// Bytes of readable shared memory required after the slot ring: payload
// reads are not clamped per row segment and may run past a corrupted tile.
constexpr int kRingPadBytes = 2048;

// ------------------------------------------------------- lookup tables
struct DecodeTables {
    // Code table: bit p of a bitmap byte -> bit 0 of nibble p, replicated
    // (entry m of copy c at [m][c]).
    uint32_t code[256][kTableCopies];
};

__host__ __device__ constexpr DecodeTables make_decode_tables() {
    DecodeTables t{};
    for (int m = 0; m < 256; ++m) {
        uint32_t v = 0;
        for (int p = 0; p < 8; ++p) v |= uint32_t((m >> p) & 1) << (4 * p);
        for (int l = 0; l < kTableCopies; ++l) t.code[m][l] = v;
    }
    return t;
}

// Payload capacity per tile rounded to 128 bytes, so tile 1's region can be
// placed 64 bytes off tile 0's modulo 128 (different shared-memory banks).
__host__ __device__ constexpr uint32_t common_capacity(int max_common) {
    return (uint32_t(max_common) + 127u) / 128u * 128u;
}

// Copied into shared memory at kernel start with one bulk copy.
__device__ const DecodeTables g_decode_tables alignas(16) = make_decode_tables();

// --------------------------------------------------------------- decoder
// What decode() leaves for store(): where each segment's rare words start
// (16 bits per segment) and which positions are rare.
struct RareState {
    uint32_t ro[4];    // segment 2h in bits 0-15, segment 2h+1 in bits 16-31
    uint32_t i03, i47;  // bitmap OR of segments 0-3 / 4-7 (bit set = common)
};

struct RowDecoder {
    uint32_t ct;         // shared address of code table + lane*4
    uint32_t bm_byte;    // offset of this row's bitmap byte (segment 0) inside one plane
    int band;            // 16-row band inside the tile
    uint32_t lane16;     // lane inside the 16-lane half
    uint32_t row_elems;  // 64*rt + 8*r: elements before this row in its small-tile pair
    // Exponent palette indexed by code: byte c = exponent rotated right by one
    // bit (bit 7 = exponent bit 0, bits 0-6 = exponent >> 1), i.e. exactly the
    // bits a common element's low byte and high byte take from it.
    uint32_t xp_lo, xp_hi;
    // Multipliers kept in registers so address and selector arithmetic runs
    // as IMAD on the FMA pipe instead of shifts on the integer ALU pipe.
    uint32_t kone, k2, k4, k8, kent, krank, khi;

    // The warp decodes band `band_` of both tiles; lane = tau*16 + rt*8 + r.
    __device__ __forceinline__ void init(uint32_t tables_smem, int lane, int band_,
                                         uint32_t start_exp) {
        const int r = lane & 7, rt = (lane >> 3) & 1;
        band = band_;
        ct = tables_smem + uint32_t(lane % kTableCopies) * 4u;
        // Small tile (band, j, rt) is bitmap word pair band*16 + 2j + rt; byte r is row r.
        bm_byte = uint32_t((band * 16 + rt) * 8 + r);
        lane16 = uint32_t(lane) & 15u;
        row_elems = uint32_t(64 * rt + 8 * r);
        uint32_t xp[2] = {0, 0};
        for (int c = 1; c < 8; ++c) {
            const uint32_t e = (start_exp + uint32_t(c)) & 255u;
            xp[c >> 2] |= (((e & 1u) << 7) | (e >> 1)) << (8 * (c & 3));
        }
        xp_lo = xp[0], xp_hi = xp[1];
        kone = ptx::launder(1u);
        k2 = ptx::launder(2u);
        k4 = ptx::launder(4u);
        k8 = ptx::launder(8u);
        kent = ptx::launder(uint32_t(kTableCopies) * 4u);
        krank = ptx::launder(0x11111110u);
        khi = ptx::launder(0x10000u);
    }

    // Decode this thread's row of one 64x64 tile whose data sits in shared
    // memory at: `plane` (bitmap1; bitmap2/3 follow at +plane_stride,
    // +2*plane_stride), `medium` (the tile's four band offset pairs),
    // `common` (the tile's common payload). All 32 lanes of the warp must call
    // this together (lanes 0-15 and 16-31 may pass different tiles). out[]
    // receives the row with every common element in place and don't-care
    // bits at rare positions; store() writes it out and patches the rare
    // words. cap_c / cap_r (bytes / words) bound the band offsets; payload
    // reads stay within kRingPadBytes past the tile's data.
    __device__ __forceinline__ void decode(uint32_t plane, uint32_t plane_stride, uint32_t medium,
                                           uint32_t common, uint32_t cap_c, uint32_t cap_r,
                                           uint32_t (&out)[32], RareState& rs) const {
        plane += bm_byte;
        const int2 med = ptx::lds_s64(medium + uint32_t(band) * 8u);
        uint32_t code[8], flag[8], ind[8];
        uint32_t k0 = 0, k1 = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t m1 = ptx::lds_u8(plane + 16u * j);
            const uint32_t m2 = ptx::lds_u8(plane + plane_stride + 16u * j);
            const uint32_t m3 = ptx::lds_u8(plane + 2u * plane_stride + 16u * j);
            const uint32_t t1 = ptx::lds_s32(ptx::mad_lo(m1, kent, ct));
            const uint32_t t2 = ptx::lds_s32(ptx::mad_lo(m2, kent, ct));
            const uint32_t t3 = ptx::lds_s32(ptx::mad_lo(m3, kent, ct));
            code[j] = ptx::mad_lo(t3, k4, ptx::mad_lo(t2, k2, t1));
            flag[j] = t1 | t2 | t3;  // nibble p = 1 when position p is common
            ind[j] = m1 | m2 | m3;
            const uint32_t cnt = __popc(ind[j]);
            if (j < 4) k0 = ptx::mad_lo(cnt, 1u << (8 * j), k0);
            else k1 = ptx::mad_lo(cnt, 1u << (8 * (j - 4)), k1);
        }
        // Inclusive 16-lane scan of the byte-packed row counts (a pair of
        // small tiles holds at most 128 common elements: bytes never carry).
        const uint32_t own0 = k0, own1 = k1;
#pragma unroll
        for (int d = 1; d < 16; d <<= 1) {
            const uint32_t a = __shfl_up_sync(kFullMask, k0, d, 16);
            const uint32_t b = __shfl_up_sync(kFullMask, k1, d, 16);
            if (lane16 >= uint32_t(d)) k0 += a, k1 += b;
        }
        const uint32_t tot0 = __shfl_sync(kFullMask, k0, 15, 16);
        const uint32_t tot1 = __shfl_sync(kFullMask, k1, 15, 16);
        const uint32_t ex0 = k0 - own0, ex1 = k1 - own1;
        const uint32_t cb = min(uint32_t(max(med.x, 0)), cap_c);
        const uint32_t rbase = min(uint32_t(max(med.y, 0)), cap_r);
        // off[j]: shared address of segment j's first payload byte (the
        // additions run on the FMA pipe, which has room to spare).
        uint32_t off[8];
        uint32_t run = common + cb;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t ex = j < 4 ? ex0 : ex1, tot = j < 4 ? tot0 : tot1;
            off[j] = ptx::mad_lo(__byte_perm(ex, 0, 0x4440 | (j & 3)), kone, run);
            run = ptx::mad_lo(__byte_perm(tot, 0, 0x4440 | (j & 3)), kone, run);
        }
        // Rare words: segment j's run starts at rbase + (elements before the
        // row segment in the band) - (common elements before it); `common`
        // cancels out of the difference.
        const uint32_t rconst = rbase + common + cb + row_elems;
#pragma unroll
        for (int h = 0; h < 4; ++h)
            rs.ro[h] = __byte_perm(rconst + 128u * (2 * h) - off[2 * h],
                                   rconst + 128u * (2 * h + 1) - off[2 * h + 1], 0x5410);
        rs.i03 = __byte_perm(__byte_perm(ind[0], ind[1], 0x0040),
                             __byte_perm(ind[2], ind[3], 0x0040), 0x5410);
        rs.i47 = __byte_perm(__byte_perm(ind[4], ind[5], 0x0040),
                             __byte_perm(ind[6], ind[7], 0x0040), 0x5410);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            // The funnel shift takes the byte offset inside the word from
            // the address's low bits.
            const uint32_t co = off[j];
            const uint32_t aw = co & ~3u;
            const uint32_t w0 = ptx::lds_s32(aw), w1 = ptx::lds_s32(aw + 4), w2 = ptx::lds_s32(aw + 8);
            const uint32_t sh = ptx::mad_lo(co, k8, 0);
            const uint32_t q0 = __funnelshift_r(w0, w1, sh);
            const uint32_t q1 = __funnelshift_r(w1, w2, sh);
            // Nibble p of `rank` = number of common positions before p: the
            // byte-permute selector that spreads the compact payload bytes.
            const uint32_t rank = ptx::mad_lo(flag[j], krank, 0);
            const uint32_t rank_hi = ptx::mul_hi(rank, khi);
            const uint32_t cj = code[j];
            {
                const uint32_t pe = __byte_perm(q0, q1, rank);
                const uint32_t xv = __byte_perm(xp_lo, xp_hi, cj);
                const uint32_t a = (pe & 0x7F7F7F7Fu) | (xv & 0x80808080u);
                const uint32_t b = (pe & 0x80808080u) | (xv & 0x7F7F7F7Fu);
                out[4 * j] = __byte_perm(a, b, 0x5140);
                out[4 * j + 1] = __byte_perm(a, b, 0x7362);
            }
            {
                const uint32_t pe = __byte_perm(q0, q1, rank_hi);
                const uint32_t xv = __byte_perm(xp_lo, xp_hi, ptx::mul_hi(cj, khi));
                const uint32_t a = (pe & 0x7F7F7F7Fu) | (xv & 0x80808080u);
                const uint32_t b = (pe & 0x80808080u) | (xv & 0x7F7F7F7Fu);
                out[4 * j + 2] = __byte_perm(a, b, 0x5140);
                out[4 * j + 3] = __byte_perm(a, b, 0x7362);
            }
        }
    }

    // Write a decoded row into a 128-byte row of a tile in the 128-byte
    // swizzled layout (16-byte chunk c at (c ^ (row & 7)) * 16; `swz` =
    // (row & 7) << 4), then overwrite its rare elements with their words from
    // `rare` (indices clamped below cap_r). Pass all_common = true for a row
    // that must not be patched.
    __device__ __forceinline__ void store(uint32_t row, uint32_t swz, const uint32_t (&out)[32],
                                          const RareState& rs, uint32_t rare, uint32_t cap_r,
                                          bool all_common) const {
#pragma unroll
        for (int c = 0; c < 8; ++c)
            ptx::sts128(row + ((uint32_t(c) << 4) ^ swz),
                        make_uint4(out[4 * c], out[4 * c + 1], out[4 * c + 2], out[4 * c + 3]));
        const uint32_t rcap = cap_r ? cap_r - 1 : 0;
        uint32_t rlo = all_common ? 0u : ~rs.i03, rhi = all_common ? 0u : ~rs.i47;
        // Rares are visited in row order; `run` counts the rares already
        // patched in the current segment, so the word of the rare at (j, c)
        // is ro_j + run.
        uint32_t prev = 8u, run = 0u;
        while (rlo | rhi) {
            const bool hi = rlo == 0u;
            const uint32_t m = hi ? rhi : rlo;
            const uint32_t p = uint32_t(__ffs(m) - 1) + (hi ? 32u : 0u);  // 0..63
            const uint32_t m2 = m & (m - 1u);
            rlo = hi ? rlo : m2;
            rhi = hi ? m2 : rhi;
            const uint32_t j = p >> 3;
            run = j == prev ? run + 1u : 0u;
            prev = j;
            // ro_j: 16-bit lane (j & 3) of the pair of words holding segments 4*hi .. 4*hi+3.
            const uint32_t ro = __byte_perm(hi ? rs.ro[2] : rs.ro[0], hi ? rs.ro[3] : rs.ro[1],
                                            (j & 3u) * 0x22u + 0x10u);
            const uint32_t idx = min((ro + run) & 0xFFFFu, rcap);
            const uint32_t word = ptx::lds_u16(ptx::mad_lo(idx, k2, rare));
            // Element c of segment j: byte 2c of 16-byte chunk j, swizzled.
            ptx::sts16(row + (((2u * p) & 0x7Eu) ^ swz), word);
        }
    }
};

}  // namespace zs
