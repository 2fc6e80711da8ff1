// TCA-TBE small-tile decoder of the fused GEMM: one thread rebuilds one 8x8
// small tile (8 rows x 8 BF16) straight into the A tile, where it is one
// core matrix of the tensor cores' unswizzled K-major layout (zipgemm.cuh).
//
// Why a small tile per thread: inside a 64x64 tile the payload streams are
// ordered band, column block j, row half, row, column (csrc/HostPacker.h:
// 110-150), so a small tile's common bytes and rare words are each one
// contiguous run. A thread takes each row's offset in the run from a masked
// population count of the small tile's bitmap OR, needs one
// 16-lane scan per step (the small tiles of a band, in stream order) instead
// of one per row, loads each bitmap plane as one 64-bit word, and patches its
// rares from a plain running index.
//
// Lane mapping (warp q of a decoder group = 16-row band q of both tiles of
// the row block): lane = tau*16 + rt*8 + j, i.e. tile tau, row half rt,
// column block j. The thread writes the core matrix of A rows 32q + 16tau +
// 8rt .. +7 and K chunk j: 128 contiguous bytes, row r at 16r and element
// (r, c) at 2 * (8r + c), so its row stores take immediate offsets and a rare
// element's address is its bit position times two. The 8 lanes of one store
// phase write the 8 K chunks of one 8-row group, 2064 bytes apart: distinct
// banks.
//
// Per row (8 elements): the three bitmap bytes (byte r of each plane word)
// index a lookup table replicated per lane that spreads them to nibbles;
// OR-ing gives the "common" flags, whose multiply by 0x11111110 is each
// position's rank among the row's common elements: the byte-permute selector
// that spreads the compact payload (one funnel-shift pair of the run); the
// exponent comes from an 8-byte palette of rotated exponents indexed by the
// code nibbles, one permute serving both byte planes. Rare elements are
// patched after the rows are stored, one 16-bit store each.
// Reference decoder semantics: csrc/L_Kernel.cuh:146-250; bit-exact results
// are checked against oracle/oracle.c:oracle_decode.
#pragma once
#include <cstdint>

#include "decode.cuh"
#include "ptx.cuh"
#include "zipgemm.cuh"

namespace zs {

struct TileDecoder {
    uint32_t ct;        // shared address of the code table + (lane % kTableCopies) * 4
    uint32_t word;      // byte offset of this small tile's word in a tile's bitmap plane
    uint32_t band8;     // byte offset of band q's (common, rare) pair in a tile's band offsets
    uint32_t aoff;      // offset of this thread's core matrix in an A tile
    uint32_t ord64;     // 64 * (2j + rt): elements before this small tile in its band
    uint32_t j, rt;

    __device__ __forceinline__ void init(uint32_t tables_smem, int lane, int q) {
        const uint32_t tau = uint32_t(lane) >> 4;
        rt = (uint32_t(lane) >> 3) & 1u;
        j = uint32_t(lane) & 7u;
        ct = tables_smem + uint32_t(lane % kTableCopies) * 4u;
        word = (uint32_t(q) * 16u + 2u * j + rt) * 8u;
        band8 = uint32_t(q) * 8u;
        // 8-row group (32q + 16tau + 8rt) / 8 along M, K chunk j.
        aoff = (4u * uint32_t(q) + 2u * tau + rt) * kAGroup + j * kACoreK;
        ord64 = 64u * (2u * j + rt);
    }

    // Decode this thread's small tile of the tile whose slot data sits at
    // `plane` (bitmap plane 1; planes 2 and 3 follow at plane_stride),
    // `medium` (the tile's four band offset pairs), `common` / `rare` (the
    // tile's payload runs), and write it into the A tile at `atile`. All 32
    // lanes call this together. cap_c / cap_r (bytes / words) bound the
    // offsets read from the packed data. A thread whose tile does not exist
    // (ragged last row block) passes valid = false and writes zeros.
    // `kc` holds the multipliers and the exponent palette (a DecodeConsts in
    // the kernel's parameter bank).
    template <class Consts>
    __device__ __forceinline__ void decode_store(const Consts& kc, uint32_t plane,
                                                 uint32_t plane_stride,
                                                 uint32_t medium, uint32_t common, uint32_t rare,
                                                 uint32_t cap_c, uint32_t cap_r, uint32_t atile,
                                                 bool valid) const {
        const uint2 p1 = ptx::lds_u64(plane + word);
        const uint2 p2 = ptx::lds_u64(plane + plane_stride + word);
        const uint2 p3 = ptx::lds_u64(plane + 2u * plane_stride + word);
        const uint32_t ind_lo = p1.x | p2.x | p3.x, ind_hi = p1.y | p2.y | p3.y;
        const uint32_t nc = valid ? uint32_t(__popc(ind_lo) + __popc(ind_hi)) : 0u;
        // Commons before this small tile in its band, in stream order (j, rt):
        // pair sums over column blocks j' < j, plus the row half 0 tile of
        // column block j when rt = 1.
        const uint32_t other = __shfl_xor_sync(kFullMask, nc, 8);
        uint32_t pair = nc + other, incl = pair;
#pragma unroll
        for (uint32_t d = 1; d < 8; d <<= 1) {
            const uint32_t v = __shfl_up_sync(kFullMask, incl, d, 8);
            if (j >= d) incl += v;
        }
        const uint32_t before = incl - pair + (rt ? other : 0u);
        // Trip counts of the rare patch loops below: the most rare elements
        // any lane of the warp has in rows 0-3 and in rows 4-7 (a missing
        // tile counts none). Every lane takes part, before the return below.
        const uint32_t n_lo =
            32u - uint32_t(__reduce_min_sync(kFullMask, valid ? uint32_t(__popc(ind_lo)) : 32u));
        const uint32_t n_hi =
            32u - uint32_t(__reduce_min_sync(kFullMask, valid ? uint32_t(__popc(ind_hi)) : 32u));
        const int2 med = ptx::lds_s64(medium + band8);
        const uint32_t cofs = min(uint32_t(max(med.x, 0)) + before, cap_c);
        const uint32_t rofs = min(uint32_t(max(med.y, 0)) + ord64 - before, cap_r);
        // Row r's payload starts after the commons of rows 0 .. r-1: one
        // masked population count per row, so no row waits for the previous.
        const uint32_t co0 = common + cofs, co4 = co0 + uint32_t(__popc(ind_lo));
        const uint32_t a_s = atile + aoff;
        if (!valid) {  // only in a ragged last row block: zero rows, no patches
#pragma unroll
            for (int r = 0; r < 8; ++r) ptx::sts128(a_s + uint32_t(r) * 16u, make_uint4(0u, 0u, 0u, 0u));
            return;
        }
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            const uint32_t co =
                (r & 3) == 0 ? (r ? co4 : co0)
                             : (r < 4 ? co0 : co4) +
                                   uint32_t(__popc((r < 4 ? ind_lo : ind_hi) &
                                                   ((1u << (8 * (r & 3))) - 1u)));
            const uint32_t sel = 0x4440u | uint32_t(r & 3);
            const uint32_t m1 = __byte_perm(r < 4 ? p1.x : p1.y, 0, sel);
            const uint32_t m2 = __byte_perm(r < 4 ? p2.x : p2.y, 0, sel);
            const uint32_t m3 = __byte_perm(r < 4 ? p3.x : p3.y, 0, sel);
            const uint32_t t1 = ptx::lds_s32(ptx::mad_lo(m1, kc.kent, ct));
            const uint32_t t2 = ptx::lds_s32(ptx::mad_lo(m2, kc.kent, ct));
            const uint32_t t3 = ptx::lds_s32(ptx::mad_lo(m3, kc.kent, ct));
            const uint32_t code = ptx::mad_lo(t3, kc.k4, ptx::mad_lo(t2, kc.k2, t1));
            const uint32_t flag = t1 | t2 | t3;
            const uint32_t aw = co & ~3u;
            const uint32_t w0 = ptx::lds_s32(aw), w1 = ptx::lds_s32(aw + 4), w2 = ptx::lds_s32(aw + 8);
            const uint32_t sh = ptx::mad_lo(co, kc.k8, 0);
            const uint32_t q0 = __funnelshift_r(w0, w1, sh);
            const uint32_t q1 = __funnelshift_r(w1, w2, sh);
            const uint32_t rank = ptx::mad_lo(flag, kc.krank, 0);
            const uint32_t rank_hi = ptx::mul_hi(rank, kc.khi);
            uint32_t out[4];
            {
                const uint32_t pe = __byte_perm(q0, q1, rank);
                const uint32_t xv = __byte_perm(kc.xp_lo, kc.xp_hi, code);
                const uint32_t a = (pe & 0x7F7F7F7Fu) | (xv & 0x80808080u);
                const uint32_t b = (pe & 0x80808080u) | (xv & 0x7F7F7F7Fu);
                out[0] = __byte_perm(a, b, 0x5140);
                out[1] = __byte_perm(a, b, 0x7362);
            }
            {
                const uint32_t pe = __byte_perm(q0, q1, rank_hi);
                const uint32_t xv = __byte_perm(kc.xp_lo, kc.xp_hi, ptx::mul_hi(code, kc.khi));
                const uint32_t a = (pe & 0x7F7F7F7Fu) | (xv & 0x80808080u);
                const uint32_t b = (pe & 0x80808080u) | (xv & 0x7F7F7F7Fu);
                out[2] = __byte_perm(a, b, 0x5140);
                out[3] = __byte_perm(a, b, 0x7362);
            }
            ptx::sts128(a_s + uint32_t(r) * 16u, make_uint4(out[0], out[1], out[2], out[3]));
        }
        // Rare elements in row order: element p = 8r + c of the small tile is
        // the next word of the tile's rare run, stored at 2p in the core
        // matrix. Rows 0-3, then rows 4-7 (64 bytes further), each a loop of
        // the warp's uniform trip count in which a lane patches its lowest
        // remaining rare bit (a lane with none left reads a word it does not
        // store). The run is read from its clamped start without a per-word
        // clamp: at most 65 words, which stay inside the slot ring and its
        // pad.
        uint32_t ra = rare + 2u * rofs;
        uint32_t rm = ~ind_lo;
        for (uint32_t i = 0; i < n_lo; ++i) {
            const bool has = rm != 0u;
            const uint32_t p = uint32_t(__ffs(rm) - 1);
            rm &= rm - 1u;
            const uint32_t wv = ptx::lds_u16(ra);
            if (has) ptx::sts16(a_s + 2u * p, wv);
            ra += has ? 2u : 0u;
        }
        rm = ~ind_hi;
        const uint32_t a_h = a_s + 64u;
        for (uint32_t i = 0; i < n_hi; ++i) {
            const bool has = rm != 0u;
            const uint32_t p = uint32_t(__ffs(rm) - 1);
            rm &= rm - 1u;
            const uint32_t wv = ptx::lds_u16(ra);
            if (has) ptx::sts16(a_h + 2u * p, wv);
            ra += has ? 2u : 0u;
        }
    }
};

}  // namespace zs
