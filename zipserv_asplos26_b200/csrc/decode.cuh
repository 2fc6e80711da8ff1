// TCA-TBE row decoder shared by the fused GEMM and the standalone decompress
// kernel.
//
// Mapping: one thread owns one matrix row of a 64x64 global tile and rebuilds
// the row's 64 BF16 words (32 packed 32-bit words, element k in half k&1 of
// word k/2). A warp owns 32 rows = two 16-row bands of one tile; lanes 0-15
// hold one band and lanes 16-31 the next. In band order the stream of a pair
// of small tiles (2j, 2j+1) is rows 0..7 of small tile 2j then rows 0..7 of
// 2j+1, which is exactly lane order inside a 16-lane half (lane = rt*8 + r).
// That makes every stream offset a 16-lane prefix sum, done once per K slice
// for all eight column blocks with byte-packed (SWAR) shuffles.
//
// Per row segment (8 elements = one small-tile row) the work is branch-free
// except for the rare elements:
//   * the three bitmap bytes give the 8 codes as nibbles (lookup in a
//     per-lane replicated table, so lookups never conflict on banks);
//   * the compact common payload bytes are fetched with one funnel shift pair
//     and spread to their positions with a byte permute whose selector comes
//     from a 256-entry table indexed by the row's "common" mask;
//   * exponents come from two 8-byte palettes (low byte bit 7 = exponent
//     LSB, high byte bits 0-6 = exponent >> 1), selected by the code nibbles;
//   * rare words are scattered into a per-thread row buffer (a short loop
//     over the rare bits only) and merged with another byte permute.
// Reference decoder semantics: csrc/L_Kernel.cuh:146-250 (register fragment
// decoder) and csrc/L_Kernel.cuh:1022-1143 (tile decoder to shared memory);
// bit-exact results are checked against oracle/oracle.c:oracle_decode.
#pragma once
#include <cstdint>

#include "ptx.cuh"

namespace zs {

constexpr uint32_t kFullMask = 0xFFFFFFFFu;
constexpr int kIndexTableBytes = 256 * 16;        // per "common" mask: 4 selectors
constexpr int kCodeTableBytes = 256 * 32 * 4;     // per bitmap byte x per lane
constexpr int kRowBufferBytes = 128;              // per decoder thread

// Fill the two lookup tables. Called by all threads of the block, followed
// by a __syncthreads() before use.
__device__ __forceinline__ void build_decode_tables(uint8_t* it_bytes, uint32_t* ct, int tid,
                                                    int nthreads) {
    // Index table entry for mask `ind` (bit p set = position p is common):
    //   x, y: byte selectors picking the compact common byte for positions
    //         0-3 / 4-7 (nibble = rank of the position among common ones);
    //   z, w: merge selectors taking byte p from the decoded word (nibble p)
    //         when common, else from the rare row buffer (nibble 4+p).
    for (int ind = tid; ind < 256; ind += nthreads) {
        uint32_t sel[2] = {0, 0}, mix[2] = {0, 0};
        int rank = 0;
        for (int p = 0; p < 8; ++p) {
            const bool common = (ind >> p) & 1;
            const int h = p >> 2, q = p & 3;
            sel[h] |= uint32_t(rank & 7) << (4 * q);
            mix[h] |= uint32_t(common ? q : 4 + q) << (4 * q);
            rank += common;
        }
        reinterpret_cast<uint4*>(it_bytes)[ind] = make_uint4(sel[0], sel[1], mix[0], mix[1]);
    }
    // Code table: bit p of a bitmap byte -> bit 0 of nibble p, replicated per
    // lane (entry m of lane l at word m*32 + l).
    for (int i = tid; i < 256 * 32; i += nthreads) {
        const uint32_t m = uint32_t(i) >> 5;
        uint32_t v = 0;
        for (int p = 0; p < 8; ++p) v |= ((m >> p) & 1u) << (4 * p);
        ct[i] = v;
    }
}

// Per-thread constants of the row decoder.
struct RowDecoder {
    const uint32_t* ct;  // code table + lane
    const uint4* it;     // index table
    uint8_t* rb;         // this thread's 128-byte row buffer
    uint32_t sw;         // row-buffer chunk swizzle (lane & 15)
    uint32_t selr;       // byte-permute selector: byte (r & 3) of a, zeros elsewhere
    int bm_word;         // u32 index of this row's bitmap word inside one plane
    int band;            // 16-row band inside the tile
    uint32_t lane16;     // lane inside the 16-lane band half
    uint32_t row_elems;  // 64*rt + 8*r: elements before this row in its small-tile pair
    uint32_t lp_lo, lp_hi, hp_lo, hp_hi;  // exponent palettes, indexed by code

    // `row_in_tile` is 0..63; lane = threadIdx.x & 31 must equal row_in_tile & 31.
    __device__ __forceinline__ void init(const uint32_t* ct_base, const uint4* it_base,
                                         uint8_t* row_buffer, int lane, int row_in_tile,
                                         uint32_t start_exp) {
        const int r = row_in_tile & 7, rt = (row_in_tile >> 3) & 1;
        band = row_in_tile >> 4;
        ct = ct_base + lane;
        it = it_base;
        rb = row_buffer;
        sw = uint32_t(lane) & 15u;
        selr = uint32_t(r & 3) | 0x4440u;
        bm_word = (band * 16 + rt) * 2 + (r >> 2);
        lane16 = uint32_t(lane) & 15u;
        row_elems = uint32_t(64 * rt + 8 * r);
        // Palettes: low byte of code c is (E&1)<<7, high byte E>>1, where
        // E = (start_exp + c) mod 256; code 0 (rare) maps to zero bytes.
        uint32_t lp[2] = {0, 0}, hp[2] = {0, 0};
        for (int c = 1; c < 8; ++c) {
            const uint32_t e = (start_exp + uint32_t(c)) & 255u;
            lp[c >> 2] |= ((e & 1u) << 7) << (8 * (c & 3));
            hp[c >> 2] |= (e >> 1) << (8 * (c & 3));
        }
        lp_lo = lp[0], lp_hi = lp[1], hp_lo = hp[0], hp_hi = hp[1];
    }

    // Decode this thread's row of one 64x64 tile. `plane` points at the
    // tile's bitmap1 (bitmap2/3 follow at +512/+1024 bytes), `medium` at its
    // four (common, rare) band offsets, `common`/`rare` at its payloads.
    // cap_c / cap_r bound every payload index (bytes / words). All 32 lanes
    // of the warp must call this together.
    __device__ __forceinline__ void decode(const uint32_t* plane, const int* medium,
                                           const uint8_t* common, const uint16_t* rare,
                                           uint32_t cap_c, uint32_t cap_r,
                                           uint32_t (&out)[32]) const {
        uint32_t code[8], ind[8];
        uint32_t k0 = 0, k1 = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t* w = plane + bm_word + 4 * j;
            const uint32_t m1 = __byte_perm(w[0], 0, selr);
            const uint32_t m2 = __byte_perm(w[128], 0, selr);
            const uint32_t m3 = __byte_perm(w[256], 0, selr);
            code[j] = ct[m1 << 5] + 2u * ct[m2 << 5] + 4u * ct[m3 << 5];
            ind[j] = m1 | m2 | m3;
            const uint32_t cnt = __popc(ind[j]);
            if (j < 4) k0 |= cnt << (8 * j);
            else k1 |= cnt << (8 * (j - 4));
        }
        // Inclusive 16-lane scan of the byte-packed row counts (each pair of
        // small tiles holds at most 128 common elements, so bytes never carry).
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
        const uint32_t cb = min(uint32_t(max(medium[band * 2], 0)), cap_c);
        const uint32_t rbase = min(uint32_t(max(medium[band * 2 + 1], 0)), cap_r);
        uint32_t off[8];
        uint32_t run = cb;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t ex = j < 4 ? ex0 : ex1, tot = j < 4 ? tot0 : tot1;
            off[j] = run + ((ex >> (8 * (j & 3))) & 255u);
            run += (tot >> (8 * (j & 3))) & 255u;
        }
        // Rare words of segment j start at rbase + (elements before the row in
        // the band) - (common elements before it).
        const uint32_t rconst = rbase + cb + row_elems;
        const uint32_t rcap = cap_r ? cap_r - 1 : 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t co = min(off[j], cap_c);
            const uint32_t* aw = reinterpret_cast<const uint32_t*>(common + (co & ~3u));
            const uint32_t w0 = aw[0], w1 = aw[1], w2 = aw[2];
            const uint32_t q0 = __funnelshift_r(w0, w1, co << 3);
            const uint32_t q1 = __funnelshift_r(w1, w2, co << 3);
            const uint4 t = it[ind[j]];
            uint32_t rm = ~ind[j] & 0xFFu;
            uint32_t ro = rconst + 128u * j - off[j];
            uint8_t* rlo = rb + ((uint32_t(j) ^ sw) << 3);
            uint8_t* rhi = rb + ((uint32_t(8 + j) ^ sw) << 3);
            while (rm) {
                const uint32_t c = __ffs(rm) - 1;
                rm &= rm - 1;
                const uint32_t word = rare[min(ro, rcap)];
                ++ro;
                rlo[c] = uint8_t(word);
                rhi[c] = uint8_t(word >> 8);
            }
            const uint2 rl = *reinterpret_cast<const uint2*>(rlo);
            const uint2 rh = *reinterpret_cast<const uint2*>(rhi);
            const uint32_t cj = code[j];
            {
                const uint32_t pe = __byte_perm(q0, q1, t.x);
                uint32_t a = (pe & 0x7F7F7F7Fu) | __byte_perm(lp_lo, lp_hi, cj);
                uint32_t b = (pe & 0x80808080u) | __byte_perm(hp_lo, hp_hi, cj);
                a = __byte_perm(a, rl.x, t.z);
                b = __byte_perm(b, rh.x, t.z);
                out[4 * j] = __byte_perm(a, b, 0x5140);
                out[4 * j + 1] = __byte_perm(a, b, 0x7362);
            }
            {
                const uint32_t pe = __byte_perm(q0, q1, t.y);
                const uint32_t ch = cj >> 16;
                uint32_t a = (pe & 0x7F7F7F7Fu) | __byte_perm(lp_lo, lp_hi, ch);
                uint32_t b = (pe & 0x80808080u) | __byte_perm(hp_lo, hp_hi, ch);
                a = __byte_perm(a, rl.y, t.w);
                b = __byte_perm(b, rh.y, t.w);
                out[4 * j + 2] = __byte_perm(a, b, 0x5140);
                out[4 * j + 3] = __byte_perm(a, b, 0x7362);
            }
        }
    }
};

}  // namespace zs
