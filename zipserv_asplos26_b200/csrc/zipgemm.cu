// Fused TCA-TBE decompress + GEMM ("ZipGEMM") for sm_100a.
//
//   y[n, m] = sum_k W[m, k] * x[n, k],  W decoded on the fly from TCA-TBE.
//
// A CTA computes 128-row blocks of W (two vertically adjacent 64x64 global
// tiles) against a tile of up to 256 tokens over its range of 64-wide K
// slices. Warp roles (1 CTA per SM):
//   warp 0      allocates tensor memory and issues tcgen05.mma (one
//               elected lane) with both operands in shared memory (A = a
//               decoder group's tile of decoded W in the unswizzled
//               core-matrix layout, B = an x tile, 128-byte swizzled as TMA
//               writes it) and two FP32 accumulators in TMEM;
//   warp 1      keeps a ring of x slices filled with 3-D TMA loads;
//   warps 2-3   producers: fill the compressed ring's slots as soon as their
//               previous K slice was decoded, with few, large copies (an
//               SM's copy engine takes ~100 cycles per copy whatever its
//               size): one 4-D tensor load for the three bitmap planes of
//               both tile rows, one 3-D load for the band offsets, one bulk
//               copy per payload run;
//   warps 4..   NDG decoder groups of four warps. Group g decodes the CTA's
//               K slices g, g+NDG, ... (slice t from ring entry t % nslots)
//               into its A tile: warp q takes 16-row band q of both tiles,
//               each thread rebuilds one 8x8 small tile (tile_decode.cuh),
//               one core matrix of the A tile, with 16-byte stores and
//               patches its rare elements with 16-bit stores;
//   last 4      epilogue, one TMEM lane quarter each: TMEM -> BF16 -> y for
//               whole units, TMEM -> FP32 pieces for split ones.
// Split-K: the grid is persistent (one CTA per SM) and every CTA takes an
// equal contiguous range of the (row block, K slice) work items, so each
// gets the same amount of decoding whatever the shape. A row block whose K
// range is split over several CTAs is summed in FP32, in K order
// (deterministic), inside this kernel: the CTA holding its first K part
// waits a bounded time for the other parts' pieces (published through L2)
// and adds them to its TMEM accumulator; if they are late, it publishes its
// own part instead and the last part to arrive reduces. No second kernel
// runs (replaces csrc/Reduction_Kernel.cuh:16-41).
//
// Reference kernel this replaces: csrc/L_Kernel.cuh:310-915 (mma.sync,
// cp.async double buffering, per-column-warp redundant decode).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>
#include <vector>

#include "capi_internal.h"
#include "codec.h"
#include "decode.cuh"
#include "tile_decode.cuh"
#include "ptx.cuh"
#include "zipgemm.cuh"

namespace zs {

// Warpgroups: 0 = MMA issuer, x loader, two producers; 1 .. NDG = decoder
// groups; NDG + 1 = epilogue.
constexpr int gemm_threads(int ndg) { return 256 + 128 * ndg; }

// Default of how long a reducing CTA waits for the other K parts of its row
// block before it falls back to publishing its own part (the last arrival
// then reduces). On a resident grid the other parts are their CTAs' first
// segments and arrive long before; the limit only matters when those CTAs
// could not start (other work holding SMs).
constexpr uint64_t kReducerWaitNs = 50000;


// TMEM lane (= decoder thread slot) -> row inside the 128-row block.
__host__ __device__ __forceinline__ int lane_row(int slot) {
    const int band = slot >> 5, l = slot & 31;
    return (l >> 4) * 64 + band * 16 + (l & 15);
}

__device__ __forceinline__ uint32_t bar_addr(uint32_t base, int index) {
    return base + 8u * uint32_t(index);
}

// Work schedule (persistent, "stream-K"): a unit is one 128-row block x one
// N tile; its kt K slices are the work items, units in order, so the grid's
// steps = units * kt items form one sequence. CTA c owns the contiguous items
// [start(c), start(c+1)), start(c) = c * steps / grid: every CTA gets the
// same number of K slices (+-1) whatever the shape. The run of a CTA's items
// inside one unit is a segment. A segment that covers its whole unit stores
// BF16 output directly. For a unit split over CTAs c0 .. c0 + parts - 1,
// parts 1 .. are their CTAs' first segments and write FP32 partial pieces to
// the workspace, then count their arrival (one counter per (c0, TMEM lane
// quarter)); part 0 is c0's last segment. On a resident grid c0 waits,
// bounded, for the other arrivals and sums its TMEM accumulator with their
// pieces; if it gives up (or the grid is larger than the GPU) it publishes
// too and whichever part arrives last sums all pieces. Either way the sum
// runs in K order - a fixed order, so results do not depend on timing - and
// the reducer returns the counter to zero.
// The items are dealt out in groups of S consecutive K slices of one unit
// (the host schedule uses S = 1; the kernel accepts any S dividing K/64),
// so a CTA's range always holds whole groups and each compressed slot
// carries one group: CTA c owns groups [c * G / grid, (c + 1) * G / grid),
// G = steps / S.
__device__ __forceinline__ int sched_start(int c, int grid, int groups, int S) {
    return S * int(int64_t(c) * groups / grid);
}
__device__ __forceinline__ int sched_owner(int item, int grid, int groups, int S) {
    return int((int64_t(item / S + 1) * grid - 1) / groups);
}
__device__ __forceinline__ int step_start(int c, const GemmParams& p) {
    return sched_start(c, p.grid, p.groups, p.S);
}
__device__ __forceinline__ int step_owner(int item, const GemmParams& p) {
    return sched_owner(item, p.grid, p.groups, p.S);
}

// ----------------------------------------------------------------------
// Fused all-reduce of the output (row-parallel layers over tp_world GPUs).
// When a CTA holds the final FP32 value of a (unit, TMEM lane quarter) - a
// whole unit, or a split unit it reduced - it stores the quarter's chunks
// into every rank's receive buffer (peer stores over NVLink). After its last
// segment it waits (bounded) for every rank's values of the units it holds,
// sums them in rank order and stores BF16. Every rank runs the same schedule
// on its K shard, so every rank computes every unit; the sum order is fixed,
// so all ranks store identical outputs.
// Each value travels as one 64-bit word (launch epoch << 32 | FP32 bits),
// written and read whole: a reader knows a value has arrived when its word
// carries this launch's epoch, so no fence or separate flag is needed (a
// system-scope fence before a flag cost several microseconds per launch).
// Buffers are double-buffered by the epoch's parity: a rank can be at most
// one launch ahead of another (it cannot finish a launch without every
// rank's values), so the buffer it writes is never the one a slower rank
// still reads, and a word left from two launches ago carries another epoch.
//   receive buffer: [2][world][units][4 quarters][chunks][8][32 lanes][2] u64
// A chunk is a lane's 16 columns; columns 2i, 2i+1 sit in the chunk's i-th
// 512-byte run, so every warp-wide 16-byte store or load covers 512
// contiguous bytes (whole 128-byte lines across NVLink).
__device__ __forceinline__ size_t tp_recv_index(const GemmParams& p, uint32_t par, int src,
                                                int unit, int q, int c, int lane) {
    return ((((size_t(par) * p.tp_world + src) * p.units + unit) * 4 + q) * size_t(p.bn / 16) +
            c) * 512u + size_t(lane) * 2u;
}
// This launch's epoch (read after the previous launch completed: every rank
// counts its fused launches alike; never 0, the buffers' initial contents).
__device__ __forceinline__ uint32_t tp_epoch(const GemmParams& p) {
    const uint32_t e = *reinterpret_cast<volatile uint32_t*>(p.tp_state) + 1u;
    return e ? e : 1u;
}
__device__ __forceinline__ uint64_t tp_word(uint32_t epoch, float v) {
    return (uint64_t(epoch) << 32) | __float_as_uint(v);
}
__device__ __forceinline__ void tp_put(const GemmParams& p, uint32_t epoch, int unit, int q, int c,
                                       int lane, const float (&acc)[16]) {
    for (int r = 0; r < p.tp_world; ++r) {
        uint64_t* dst = p.tp_recv[r] + tp_recv_index(p, epoch & 1u, p.tp_rank, unit, q, c, lane);
#pragma unroll
        for (int i = 0; i < 8; ++i)
            ptx::st_volatile_v2u64(dst + 64 * i, tp_word(epoch, acc[2 * i]),
                                   tp_word(epoch, acc[2 * i + 1]));
    }
}
// Wait (bounded) for every rank's values of (unit, q), sum them in rank
// order and store BF16. Called once the CTA has sent all its units, so the
// wait overlaps the other ranks' remaining work rather than this one's.
__device__ __noinline__ void tp_collect(const GemmParams& p, uint32_t epoch, int unit, int q,
                                        int lane, int nb, int mrow, bool row_ok) {
    const uint32_t par = epoch & 1u;
    const uint64_t* mine = p.tp_recv[p.tp_rank];
    bool ok = true;
    for (int c = 0; c < p.bn / 16; ++c) {
        float acc[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = 0.f;
        for (int src = 0; src < p.tp_world; ++src) {
            const uint64_t* from = mine + tp_recv_index(p, par, src, unit, q, c, lane);
            float v[16];
            uint64_t t0 = 0;
            for (uint32_t it = 0;; ++it) {
                uint32_t mismatch = 0;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    uint64_t a0, a1;
                    ptx::ld_volatile_v2u64(from + 64 * i, a0, a1);
                    mismatch |= (uint32_t(a0 >> 32) ^ epoch) | (uint32_t(a1 >> 32) ^ epoch);
                    v[2 * i] = __uint_as_float(uint32_t(a0));
                    v[2 * i + 1] = __uint_as_float(uint32_t(a1));
                }
                if (!mismatch || !ok) break;
                if ((it & 15) == 15) {
                    const uint64_t now = ptx::global_timer_ns();
                    if (!t0) t0 = now;
                    else if (now - t0 > 2000000000ull) {
                        atomicOr(&g_device_flags, 1u);
                        ok = false;
                    }
                    __nanosleep(64);
                }
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[j] += v[j];
        }
        if (!row_ok || !ok) continue;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int nn = nb * p.bn + 16 * c + j;
            if (nn < p.n)
                p.y[size_t(nn) * p.m + mrow] = __bfloat16_as_ushort(__float2bfloat16_rn(acc[j]));
        }
    }
}

// One 16-column chunk of a resident reducer's row block: its own K part
// from TMEM plus the other parts' published pieces, added in K order (two
// whole pieces per L2 round trip), converted and stored. Run by the epilogue
// warp of a TMEM lane quarter and, since the reducer's segment is its CTA's
// last, by the idle decoder warps of the same quarter, each on its share of
// the chunks. `tbase` is the quarter's lanes of the segment's accumulator.
struct ChunkReduce {
    float* ws_partials;
    uint16_t* y;
    int m, n, bn, pieces;
    uint32_t tbase;
    int c0, parts, nb, mrow, lane;
    size_t piece0;  // the quarter's first piece
    bool row_ok, dok, wok;
    const GemmParams* gp;  // fused all-reduce: chunks go to the ranks instead of y
    uint32_t epoch;
    int unit, q;

    __device__ __forceinline__ void run(int c) const {
        uint32_t v[16];
        ptx::tmem_ld_32x32b_x16(tbase + 16u * uint32_t(c), v);
        ptx::tmem_wait_ld();
        float acc[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = dok ? __uint_as_float(v[j]) : 0.f;
        // Part pp >= 1 is CTA c0 + pp's first segment (partial slot 0).
        auto piece = [&](int pp) {
            return ws_partials +
                   ((size_t(c0 + pp) * 2) * size_t(pieces) + piece0 + size_t(c)) * 512u +
                   size_t(lane) * 16u;
        };
        for (int pp = 1; wok && pp < parts; pp += 2) {
            const bool two = pp + 1 < parts;
            const float* s0 = piece(pp);
            const float* s1 = two ? piece(pp + 1) : s0;
            float4 x[4], y[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) x[i] = ptx::ldg_cg_f4(s0 + 4 * i);
#pragma unroll
            for (int i = 0; i < 4; ++i) y[i] = ptx::ldg_cg_f4(s1 + 4 * i);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                acc[4 * i] += x[i].x, acc[4 * i + 1] += x[i].y;
                acc[4 * i + 2] += x[i].z, acc[4 * i + 3] += x[i].w;
            }
            if (two) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    acc[4 * i] += y[i].x, acc[4 * i + 1] += y[i].y;
                    acc[4 * i + 2] += y[i].z, acc[4 * i + 3] += y[i].w;
                }
            }
        }
        if (gp->tp_world > 1) {
            tp_put(*gp, epoch, unit, q, c, lane, acc);
            return;
        }
        if (!row_ok) return;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int nn = nb * bn + 16 * c + j;
            if (nn < n)
                y[size_t(nn) * m + mrow] = __bfloat16_as_ushort(__float2bfloat16_rn(acc[j]));
        }
    }
};

// A decoder warp's share of its CTA's last-segment reduction (kept out of
// line so the decoder loop's register allocation is not affected). Runs
// only when the quarter's epilogue warp saw every other part arrive in time.
__device__ __noinline__ void help_reduce(const GemmParams* gp, float* ws_partials, uint16_t* y,
                                         int m, int n, int bn, int pieces, uint32_t tmem_cols,
                                         int grid, int groups, int S, uint32_t tmem, uint32_t bar_d,
                                         int unit, int s, int rbs, int kt, int cta, int g, int q,
                                         int lane, int stride) {
    const int b = s & 1, chunks = bn / 16, ubeg = unit * kt;
    const bool dok = ptx::mbar_wait(bar_d + 8u * uint32_t(b), uint32_t(s >> 1) & 1u);
    ptx::tc_fence_after();
    ptx::wait_prerequisites();  // output writes, as in the epilogue
    const int last_owner = sched_owner(ubeg + kt - 1, grid, groups, S);
    const int parts = last_owner - cta + 1;
    const int mrow = (unit % rbs) * 128 + lane_row(32 * q + lane);
    const uint32_t epoch = gp->tp_world > 1 ? tp_epoch(*gp) : 0u;
    const ChunkReduce cr{ws_partials, y, m, n, bn, pieces,
                         tmem + (uint32_t(32 * q) << 16) + uint32_t(b) * tmem_cols,
                         cta, parts, unit / rbs, mrow, lane, size_t(q) * size_t(chunks),
                         mrow < m, dok, true, gp, epoch, unit, q};
    for (int c = g + 1; c < chunks; c += stride) cr.run(c);
    // Chunks sent to other GPUs: the named barrier below orders them before
    // the epilogue warp's system-scope release of the flags.
    ptx::tc_fence_before();
}

// Warp roles: warp 0 allocates TMEM and issues the MMAs; warp 1 keeps the x
// ring filled; warps 2-3 fill the decoder groups' compressed slots; warps
// 4 .. 4 + 4*NDG - 1 form NDG decoder groups (local step t, item
// start(c) + t, is decoded by group t % NDG from ring entry (t / S) %
// nslots); the last four warps drain the accumulators (epilogue), one TMEM
// lane quarter each.
template <int NDG>
__global__ void __launch_bounds__(256 + 128 * NDG, 1)
    zipgemm_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ PlaneMaps pm,
                   const __grid_constant__ CUtensorMap mmap, const __grid_constant__ GemmParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t sbase = ptx::smem_addr(smem);
    const uint32_t bar_full = sbase;                         // [nslots] slot landed
    const uint32_t bar_free = sbase + 8 * kMaxStages;         // [nslots] slot read by its groups
    const uint32_t bar_afull = bar_free + 8 * kMaxStages;     // [na] A tile written
    const uint32_t bar_aempty = bar_afull + 8 * kMaxATiles;  // [na] A tile read by MMAs
    const uint32_t bar_xfull = bar_aempty + 8 * kMaxATiles;   // [kMaxX]
    const uint32_t bar_xempty = bar_xfull + 8 * kMaxX;
    const uint32_t bar_d = bar_xempty + 8 * kMaxX;             // [2] accumulator complete
    const uint32_t bar_tempty = bar_d + 16;                    // [2] accumulator drained
    const uint32_t bar_tab = bar_tempty + 16;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + (bar_tab - sbase) + 8);
    // Per TMEM lane quarter: 1 when a reducing CTA's other K parts arrived in
    // time (written by the quarter's epilogue warp, read by its decoder warps).
    const uint32_t verdict = sbase + 512;
    const uint32_t tables = sbase + kBarrierBytes;
    constexpr int kEpiWarp = 4 + 4 * NDG;

    const int cta = int(blockIdx.x);
    const int kt = p.kt, rbs = p.row_blocks;
    const int t_begin = step_start(cta, p), t_end = step_start(cta + 1, p);
    const int nsteps = t_end - t_begin;
    const int unit0 = t_begin / kt;
    const int nseg = nsteps > 0 ? (t_end - 1) / kt - unit0 + 1 : 0;
    const uint32_t cap_c = p.cap_c, cap_r = p.cap_r;
    const SlotLayout L = p.slot;

    // The next kernel in the stream may start launching now; it waits for
    // this grid's completion before it reads anything this grid writes.
    ptx::launch_dependents();
    // Prologue, overlapped across warps: warp 0 allocates TMEM while warp 1
    // initialises the barriers (one lane per barrier) and starts the table
    // copy, and the producers fetch their first chunk of payload offsets.
    //
    // Payload offsets: lane l of producer pi holds, for chunk c, the `global`
    // entries of its slot pi + 2 * (32c + l): K tiles k .. k + S of both tile
    // rows (the start of each of the slot's tiles and the end of the last);
    // the next chunk is fetched a whole chunk ahead, so the producers never
    // wait on these global loads.
    const int2* goffs = reinterpret_cast<const int2*>(p.global);
    const int nslot_items = nsteps / p.S;  // slots this CTA fills (its groups)
    auto fetch_offsets = [&](int pi, int c, int2 (&v)[6]) {
#pragma unroll
        for (int i = 0; i < 6; ++i) v[i] = make_int2(0, 0);
        const int sl = pi + 2 * (32 * c + lane);
        if (sl < nslot_items) {
            const int item = t_begin + sl * p.S, unit = item / kt, k = item - unit * kt;
            const int tr = 2 * (unit % rbs);
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                if (tr + r >= p.row_tiles) break;
                const size_t at = size_t(tr + r) * kt + k;
                v[3 * r] = goffs[at];
                v[3 * r + 1] = goffs[at + 1];
                v[3 * r + 2] = p.S == 2 ? goffs[at + 2] : v[3 * r + 1];
            }
        }
    };
    int2 first_offs[6];
    if (warp == 2 || warp == 3) fetch_offsets(warp - 2, 0, first_offs);
    if (warp == 0) {
        ptx::tmem_alloc(ptx::smem_addr(tmem_slot), 2 * p.tmem_cols);
        ptx::tmem_relinquish();
    } else if (warp == 1) {
        if (lane < p.nslots) {
            ptx::mbar_init(bar_addr(bar_full, lane), 1);
            ptx::mbar_init(bar_addr(bar_free, lane), 4u * uint32_t(p.S));  // its S steps' warps
        }
        if (lane < kMaxX) {
            ptx::mbar_init(bar_addr(bar_xfull, lane), 1);
            ptx::mbar_init(bar_addr(bar_xempty, lane), 1);
        }
        // With one x slot per A tile, x slot i lands on A tile i's barrier
        // (the x loader's arrival plus its bytes), so each step's MMAs wait
        // on one barrier.
        if (lane < kMaxATiles) {
            ptx::mbar_init(bar_addr(bar_afull, lane), p.nx == p.na ? 5u : 4u);  // group (+ x)
            ptx::mbar_init(bar_addr(bar_aempty, lane), 1);                       // MMA commit
        }
        if (lane < 2) {
            ptx::mbar_init(bar_addr(bar_d, lane), 1);
            ptx::mbar_init(bar_addr(bar_tempty, lane), 4);  // the epilogue warps
        }
        if (lane == 0) ptx::mbar_init(bar_tab, 1);
        ptx::fence_mbar_init();
        if (lane == 0) {
            ptx::prefetch_tensormap(&xmap);
            ptx::prefetch_tensormap(&mmap);
            for (int i = 0; i < pm.count; ++i) ptx::prefetch_tensormap(&pm.map[i]);
            // Decode lookup tables: one bulk copy from the library's constant table.
            ptx::mbar_arrive_expect_tx(bar_tab, kTableBytes);
            ptx::bulk_g2s(tables, &g_decode_tables, kTableBytes, bar_tab, ptx::policy_evict_last());
        }
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------ MMA issuer
        // Step t: A tile a = t % na (written by group t % NDG), B = x slot
        // t % nx (with nx == na the same index: one barrier says both
        // landed and one commit frees both). Segment s accumulates into TMEM
        // buffer s & 1; its first MMA overwrites, and it waits until the
        // epilogue of segment s - 2 has drained that buffer. The whole warp
        // runs the loop in uniform control flow; one elected lane issues
        // each step's four MMAs and commit. This warp paces the CTA, so the
        // loop is kept short: descriptors advance as 32-bit halves (the
        // start-address field holds address >> 4, a tile of B bytes adds
        // B >> 4) and common steps take a single barrier wait.
        const uint32_t idesc = ptx::idesc_bf16_m128(uint32_t(p.bn));
        const int nx = p.nx, na = p.na;
        const bool xmerged = nx == na;
        const uint64_t xdesc0 = ptx::smem_desc_sw128(sbase + p.off_x);
        const uint64_t adesc0 = ptx::smem_desc_kmajor(sbase + p.off_a, kACoreK, kAGroup);
        const uint32_t x_lo0 = uint32_t(xdesc0), x_hi = uint32_t(xdesc0 >> 32);
        const uint32_t a_lo0 = uint32_t(adesc0), a_hi = uint32_t(adesc0 >> 32);
        const uint32_t xstep = p.x_bytes >> 4, astep = kATileBytes >> 4;
        const uint32_t tcols = p.tmem_cols;
        int xs = 0, a = 0, s = 0, k = t_begin - unit0 * kt;
        uint32_t xph = 0, aph = 0, x_lo = x_lo0, a_lo = a_lo0;
        for (int t = 0; t < nsteps; ++t) {
            const bool first = t == 0 || k == 0, last = t == nsteps - 1 || k == kt - 1;
            bool ok = true;
            if (first && s >= 2)
                ok = ptx::mbar_wait(bar_addr(bar_tempty, s & 1), uint32_t((s >> 1) - 1) & 1u);
            if (!xmerged) ok = ptx::mbar_wait(bar_addr(bar_xfull, xs), xph) && ok;
            ok = ptx::mbar_wait(bar_addr(bar_afull, a), aph) && ok;
            if (!__all_sync(kFullMask, ok)) break;
            ptx::tc_fence_after();
            ptx::mma_bf16_slice_elect<2 * kACoreK / 16>(tmem + uint32_t(s & 1) * tcols, a_lo, a_hi, x_lo, x_hi, idesc,
                                      first ? 0u : 1u, bar_addr(bar_aempty, a));
            if (!xmerged) ptx::mma_commit_elect(bar_addr(bar_xempty, xs));
            if (last) ptx::mma_commit_elect(bar_addr(bar_d, s & 1));  // segment complete
            if (++xs == nx) xs = 0, xph ^= 1u, x_lo = x_lo0;
            else x_lo += xstep;
            if (++a == na) a = 0, aph ^= 1u, a_lo = a_lo0;
            else a_lo += astep;
            if (++k == kt) k = 0;
            if (last) ++s;
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------ x loader
        // Step t's x tile goes to x slot t % nx once the MMAs of step t - nx
        // have finished reading that slot. x may be written by the previous
        // kernel in the stream: wait for it first.
        if (lane == 0) {
            ptx::wait_prerequisites();
            const uint64_t pol_x = ptx::policy_evict_last();
            const int nx = p.nx;
            // One x slot per A tile: x lands on the A tile's barrier and the
            // A tile's commit frees it.
            const bool xmerged = nx == p.na;
            const uint32_t freed = xmerged ? bar_aempty : bar_xempty;
            const uint32_t landed = xmerged ? bar_afull : bar_xfull;
            int issued = 0, k = t_begin - unit0 * kt, xs = 0;
            int ntok = (unit0 / rbs) * p.bn, rb = unit0 % rbs;  // token offset of the unit
            uint32_t fph = 0;  // parity of the `freed` completion awaited next
            for (int t = 0; t < nsteps; ++t) {
                if (t >= nx && !ptx::mbar_wait(bar_addr(freed, xs), fph)) break;
                ptx::mbar_arrive_expect_tx(bar_addr(landed, xs), p.x_bytes);
                ptx::tma_load_3d(sbase + p.off_x + uint32_t(xs) * p.x_bytes, &xmap, 0, ntok, k,
                                 bar_addr(landed, xs), pol_x);
                issued = t + 1;
                if (++xs == nx) {
                    xs = 0;
                    if (t >= nx) fph ^= 1u;
                }
                if (++k == kt) {
                    k = 0;
                    if (++rb == rbs) rb = 0, ntok += p.bn;
                }
            }
            // Never leave copies in flight: wait for the last loads to land.
            for (int t = max(0, issued - nx); t < issued; ++t)
                ptx::mbar_wait(bar_addr(landed, t % nx), (t / nx) & 1);
        }
        __syncwarp();
    } else if (warp < 4) {
        // ------------------------------------------------------ producers
        // A slot holds one group of S consecutive K slices (both tile rows of
        // the block): producer pi fills the CTA's slots pi, pi + 2, ... (slot
        // v goes to ring entry v % nslots) once the decoder groups of its
        // previous contents released it. Per slot: one 4-D tensor load for
        // the three bitmap planes of the S x 2 tiles, one 3-D load for their
        // band offsets, one bulk copy per payload stream and tile row (the S
        // tiles of a tile row are consecutive in the packed streams), and the
        // tile-relative payload starts written into the slot header. An SM
        // takes ~100 cycles per copy whatever its size (S > 1 would halve the
        // copies per K slice; it measured no faster, so the host uses S = 1).
        // The packed weight is never written by other kernels: no
        // prerequisite wait.
        const int pi = warp - 2;
        const uint64_t pol_w = ptx::policy_evict_first();
        const int S = p.S, nslots = p.nslots;
        int kc = t_begin - unit0 * kt + pi * S, rb = unit0 % rbs;  // position of slot pi
        while (kc >= kt) {
            kc -= kt;
            if (++rb == rbs) rb = 0;
        }
        int2 chunk[6], ahead[6];
#pragma unroll
        for (int i = 0; i < 6; ++i) chunk[i] = first_offs[i];
        bool ok = true;
        int last = -1;  // last slot issued
        for (int v = pi, i = 0; v < nslot_items; v += 2, ++i) {
            const int ci = i & 31;
            if (ci == 0) {
                if (i > 0) {
#pragma unroll
                    for (int j = 0; j < 6; ++j) chunk[j] = ahead[j];
                }
                fetch_offsets(pi, (i >> 5) + 1, ahead);
            }
            const int sidx = v % nslots, use = v / nslots;
            int2 e[6];
#pragma unroll
            for (int j = 0; j < 6; ++j)
                e[j].x = __shfl_sync(kFullMask, chunk[j].x, ci),
                e[j].y = __shfl_sync(kFullMask, chunk[j].y, ci);
            const uint32_t slot = sbase + p.off_slots + uint32_t(sidx) * L.bytes;
            // Everything the fill needs is computed before waiting for the
            // slot, so only the stores and copies follow the wait (the
            // decoders compete for issue slots; a late fill stalls them).
            const int tr0 = 2 * rb;
            const bool has1 = tr0 + 1 < p.row_tiles;
            // Slot header: payload starts of tile j of tile row r inside the
            // row's runs, clamped to the capacities (decoders stay in bounds
            // whatever the offsets say).
            int2 h = make_int2(0, 0);
            if (lane < 2 * S) {
                const int r = lane / S, j = lane - r * S;
                const int2 st = r ? e[3] : e[0];
                const int2 tj = j ? (r ? e[4] : e[1]) : st;
                h = make_int2(min(max(tj.x - st.x, 0), int(uint32_t(j) * cap_c)),
                              min(max(tj.y - st.y, 0), int(uint32_t(j) * cap_r)));
            }
            uint32_t clen[2], rlen[2];
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const int2 st = e[3 * r], en = e[3 * r + 2];
                const bool live = r == 0 || has1;
                // Payload copies need 16-byte aligned sources, which the
                // offsets of valid packed data always give.
                clen[r] = live && (st.x & 15) == 0
                              ? min(uint32_t(max(en.x - st.x, 0)), uint32_t(S) * cap_c) & ~15u
                              : 0u;
                rlen[r] = live && (st.y & 7) == 0
                              ? (min(uint32_t(max(en.y - st.y, 0)), uint32_t(S) * cap_r) * 2u) & ~15u
                              : 0u;
            }
            const uint32_t full = bar_addr(bar_full, sidx);
            const uint32_t expect =
                p.plane_box_bytes + 64u * uint32_t(S) + clen[0] + clen[1] + rlen[0] + rlen[1];
            if (use >= 1 && lane == 0) ok = ptx::mbar_wait(bar_addr(bar_free, sidx), (use - 1) & 1);
            ok = __shfl_sync(kFullMask, ok, 0) != 0;
            if (!ok) break;
            if (lane < 2 * S) ptx::sts64(slot + L.hdr + uint32_t(lane) * 8u, h);
            // The header stores of lanes 0 .. 2S-1 are ordered before lane 0's
            // arrival (release), which the decoders acquire.
            __syncwarp();
            if (lane == 0) {
                ptx::mbar_arrive_expect_tx(full, expect);
                // Largest copies first: the slot is ready when its last byte lands.
                if (clen[0]) ptx::bulk_g2s(slot + L.common0, p.sm + e[0].x, clen[0], full, pol_w);
                if (clen[1]) ptx::bulk_g2s(slot + L.common1, p.sm + e[3].x, clen[1], full, pol_w);
                if (pm.count == 1) {
                    ptx::tma_load_4d(slot, &pm.map[0], 0, kc, tr0, 0, full, pol_w);
                } else {
#pragma unroll
                    for (int pl = 0; pl < 3; ++pl)
                        ptx::tma_load_3d(slot + uint32_t(pl) * L.plane_stride, &pm.map[pl], 0, kc,
                                         tr0, full, pol_w);
                }
                if (rlen[0]) ptx::bulk_g2s(slot + L.rare0, p.rare + e[0].y, rlen[0], full, pol_w);
                if (rlen[1]) ptx::bulk_g2s(slot + L.rare1, p.rare + e[3].y, rlen[1], full, pol_w);
                ptx::tma_load_3d(slot + L.med, &mmap, 0, kc, tr0, full, pol_w);
            }
            last = v;
            for (kc += 2 * S; kc >= kt;) {
                kc -= kt;
                if (++rb == rbs) rb = 0;
            }
        }
        // Never leave copies in flight: wait (bounded) for this producer's
        // slots that are the last use of their ring entry (with an odd ring
        // the producers alternate on an entry, and waiting on an earlier use
        // after a later one landed would target a phase already passed).
        if (lane == 0) {
            const int end = ok ? nslot_items : last + 1;
            for (int v = max(0, end - nslots); v < end; ++v)
                if ((v & 1) == pi) ptx::mbar_wait(bar_addr(bar_full, v % nslots), (v / nslots) & 1);
        }
        __syncwarp();
    } else if (warp < kEpiWarp) {
        // ------------------------------------------------------ decoders
        const int dw = warp - 4, g = dw >> 2;
        const int q = warp & 3;  // TMEM lane quarter of this warp = band it decodes
        const int tau = lane >> 4;
        TileDecoder dec;
        dec.init(tables, lane, q);
        const uint32_t abase = sbase + p.off_a;
        const int na = p.na;  // >= NDG
        bool ok = ptx::mbar_wait(bar_tab, 0);

        // Position of the group's step t, advanced without divisions.
        int k = t_begin - unit0 * kt + g, rb = unit0 % rbs;
        while (k >= kt) {
            k -= kt;
            if (++rb == rbs) rb = 0;
        }
        int a = g, ause = 0;  // A tile t % na and its use t / na
        // Slot v = t / S, slice j = t % S, ring entry v % nslots and its use
        // v / nslots, all advanced without divisions.
        const int S = p.S, nslots = p.nslots;
        int j = g % S, sidx = (g / S) % nslots, use = (g / S) / nslots;
        // Per step the group moves NDG slices on: NDG / S slots plus NDG % S
        // slices (one more slot when the slice index wraps); NDG <= nslots,
        // so the ring index wraps at most once.
        const int dslot = NDG / S, dj = NDG % S;
        for (int t = g; t < nsteps; t += NDG) {
            const bool valid = tau == 0 || 2 * rb + 1 < p.row_tiles;
            const uint32_t slot = ptx::launder(sbase + p.off_slots + uint32_t(sidx) * L.bytes);
            ok = ok && ptx::mbar_wait(bar_addr(bar_full, sidx), use & 1);
            // A tile a = t % na is free once the MMAs of step t - na finished.
            if (ause > 0) ok = ok && ptx::mbar_wait(bar_addr(bar_aempty, a), (ause - 1) & 1);
            if (!__all_sync(kFullMask, ok)) break;
            const uint32_t tile = uint32_t(tau * p.S + j);  // the tile's index in the slot
            const int2 h = ptx::lds_s64(slot + L.hdr + tile * 8u);
            dec.decode_store(p.dk, slot + tile * L.plane1, L.plane_stride, slot + L.med + tile * 32u,
                             slot + (tau ? L.common1 : L.common0) + uint32_t(h.x),
                             slot + (tau ? L.rare1 : L.rare0) + 2u * uint32_t(h.y), cap_c, cap_r,
                             abase + uint32_t(a) * kATileBytes, valid);
            // Generic-proxy stores must be visible to the tensor cores.
            ptx::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                ptx::mbar_arrive(bar_addr(bar_free, sidx));  // slot fully read
                ptx::mbar_arrive(bar_addr(bar_afull, a));
            }
            if ((a += NDG) >= na) a -= na, ++ause;
            int adv = dslot;
            if ((j += dj) >= S) j -= S, ++adv;
            if ((sidx += adv) >= nslots) sidx -= nslots, ++use;
            for (k += NDG; k >= kt;) {
                k -= kt;
                if (++rb == rbs) rb = 0;
            }
        }
        // If the CTA's last segment is a row block it reduces (resident
        // grids), help the epilogue warp of lane quarter q with it: group g
        // takes chunks g + 1, g + 2 + NDG, ... . Every warp of the quarter
        // meets twice at the quarter's named barrier: once for the epilogue
        // warp's verdict on the other parts (all arrived in time, or the
        // reduction falls back to the last arrival), once when done.
        if (p.resident && nseg > 0 && p.bn > 16) {
            const int s = nseg - 1, unit = unit0 + s, ubeg = unit * kt;
            const bool whole = t_begin <= ubeg && ubeg + kt <= t_end;
            if (!whole && cta == step_owner(ubeg, p)) {
                const int chunks = p.bn / 16;
                ptx::named_barrier_sync(1u + uint32_t(q), 32u * (1u + NDG));
                const bool fast = ptx::lds_s32(verdict + 4u * uint32_t(q)) != 0;
                if (fast && g + 1 < chunks)
                    help_reduce(&p, p.ws_partials, p.y, p.m, p.n, p.bn, p.pieces, p.tmem_cols,
                                p.grid, p.groups, p.S, tmem, bar_d, unit, s, rbs, kt, cta, g, q,
                                lane, 1 + NDG);
                ptx::named_barrier_sync(1u + uint32_t(q), 32u * (1u + NDG));
            }
        }
    } else {
        // ------------------------------------------------------ epilogue
        // Segment s (unit unit0 + s) is in accumulator s & 1. Whole units:
        // TMEM -> BF16 -> y. Partial units: TMEM -> this CTA's FP32 partial
        // pieces, release the accumulator, count the arrivals; the last
        // arrival of a piece sums its partials in K order and stores it.
        const int q = warp & 3;  // TMEM lane quarter
        const int chunks = p.bn / 16;
        const int row = 32 * q + lane;  // TMEM lane = slot in the unit's 128-row tile
        // Output and workspace writes must not race the kernels this one
        // depends on (they may still read those buffers).
        ptx::wait_prerequisites();
        const bool tp = p.tp_world > 1;
        const uint32_t epoch = tp ? tp_epoch(p) : 0u;
        // Fused all-reduce: segments whose final value this CTA published
        // (collected after the loop; at most 64 segments per CTA, see the
        // host launcher).
        uint64_t owned = 0;
        auto store_row = [&](int nb, int c, int mrow, const float (&acc)[16]) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int n = nb * p.bn + 16 * c + j;
                if (n < p.n)
                    p.y[size_t(n) * p.m + mrow] = __bfloat16_as_ushort(__float2bfloat16_rn(acc[j]));
            }
        };
        for (int s = 0; s < nseg; ++s) {
            const int b = s & 1;
            const bool dok = ptx::mbar_wait(bar_addr(bar_d, b), uint32_t(s >> 1) & 1u);
            ptx::tc_fence_after();
            const int unit = unit0 + s, rb = unit % rbs, nb = unit / rbs;
            const int ubeg = unit * kt;
            const bool whole = t_begin <= ubeg && ubeg + kt <= t_end;
            const int mrow = rb * 128 + lane_row(row);
            const bool row_ok = mrow < p.m;
            const uint32_t tbase = tmem + (uint32_t(32 * q) << 16) + uint32_t(b) * p.tmem_cols;
            if (whole) {
                for (int c = 0; c < chunks; ++c) {
                    uint32_t v[16];
                    ptx::tmem_ld_32x32b_x16(tbase + 16u * c, v);
                    ptx::tmem_wait_ld();
                    float acc[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) acc[j] = dok ? __uint_as_float(v[j]) : 0.f;
                    if (tp) tp_put(p, epoch, unit, q, c, lane, acc);
                    else if (row_ok) store_row(nb, c, mrow, acc);
                }
                ptx::tc_fence_before();
                __syncwarp();
                if (lane == 0) ptx::mbar_arrive(bar_addr(bar_tempty, b));
                if (tp) owned |= 1ull << (s & 63);
                continue;
            }
            // Partial segments are a CTA's first or last: slot `which`.
            const int which = s > 0 ? 1 : 0;
            const size_t piece0 = size_t(q) * size_t(chunks);  // this quarter's pieces
            const int c0 = step_owner(ubeg, p);
            const int parts = step_owner(ubeg + kt - 1, p) - c0 + 1;
            // One arrival counter per (first CTA of the unit, lane quarter):
            // a CTA is the first part of at most one split unit (its last
            // segment), so grid x 4 counters serve any shape.
            uint32_t* ctr = p.ws_counters + size_t(c0) * 4u + size_t(q);
            if (p.resident && cta == c0) {
                // This CTA holds the unit's first K part, the last one it
                // computes. The other parts are their CTAs' first segments,
                // so on a resident grid they publish early: wait (briefly)
                // for them and reduce with this part straight from TMEM. If
                // they are late (their CTAs could not start because other
                // work holds SMs), publish this part like the others instead:
                // the last arrival reduces, so no CTA depends on another one
                // being resident.
                bool fast = true;
                if (lane == 0)
                    fast = ptx::wait_global_geq(ctr, uint32_t(parts - 1), p.reducer_wait_ns, false);
                fast = __shfl_sync(kFullMask, fast, 0);
                if (chunks > 1) {  // tell the quarter's decoder warps
                    if (lane == 0) ptx::sts32(verdict + 4u * uint32_t(q), fast ? 1u : 0u);
                    ptx::named_barrier_sync(1u + uint32_t(q), 32u * (1u + NDG));
                }
                if (fast) {
                    // Chunks 0, 1 + NDG, ...; the quarter's decoder warps take
                    // the others (this is the CTA's last segment, they are idle).
                    const ChunkReduce cr{p.ws_partials, p.y, p.m, p.n, p.bn, p.pieces, tbase, c0,
                                         parts, nb, mrow, lane, piece0, row_ok, dok, true,
                                         &p, epoch, unit, q};
                    // With one chunk (N tile 16) the epilogue warp works alone.
                    const int stride = chunks > 1 ? 1 + NDG : 1;
                    for (int c = 0; c < chunks; c += stride) cr.run(c);
                    ptx::tc_fence_before();
                    if (chunks > 1) ptx::named_barrier_sync(1u + uint32_t(q), 32u * (1u + NDG));
                    if (tp) owned |= 1ull << (s & 63);
                    __syncwarp();
                    if (lane == 0) {
                        ptx::mbar_arrive(bar_addr(bar_tempty, b));
                        *reinterpret_cast<volatile uint32_t*>(ctr) = 0u;  // ready for reuse
                    }
                    continue;
                }
                if (chunks > 1) ptx::named_barrier_sync(1u + uint32_t(q), 32u * (1u + NDG));
            }
            // Publish this part's FP32 pieces of the quarter.
            float* mine = p.ws_partials +
                          ((size_t(cta) * 2 + size_t(which)) * size_t(p.pieces) + piece0) * 512u +
                          size_t(lane) * 16u;
            for (int c = 0; c < chunks; ++c) {
                uint32_t v[16];
                ptx::tmem_ld_32x32b_x16(tbase + 16u * c, v);
                ptx::tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; j += 4)
                    ptx::stg_cg_f4(mine + size_t(c) * 512u + j,
                                   dok ? make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]),
                                                     __uint_as_float(v[j + 2]),
                                                     __uint_as_float(v[j + 3]))
                                       : make_float4(0.f, 0.f, 0.f, 0.f));
            }
            ptx::tc_fence_before();
            // The warp barrier orders every lane's partial stores before
            // lane 0's release below, which publishes them GPU-wide.
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(bar_addr(bar_tempty, b));  // TMEM read
            // Count this arrival. On a resident grid the first part's CTA is
            // normally waiting (it never adds), so no writer is last; when it
            // gave up waiting, or the grid is not resident, the last arrival
            // sums every part in K order, stores, and resets the counter.
            uint32_t prior = 0;
            if (lane == 0) prior = ptx::atom_acq_rel_add(ctr, 1u);
            if (__shfl_sync(kFullMask, prior, 0) != uint32_t(parts - 1)) continue;
            __threadfence();  // every lane sees every part's pieces
            for (int c = 0; c < chunks; ++c) {
                float acc[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) acc[j] = 0.f;
                for (int pp = 0; pp < parts; ++pp) {
                    const int cp = c0 + pp;
                    // Part pp is CTA c0 + pp's first segment (slot 0), except
                    // the first part when the unit starts after that CTA's
                    // first segment (slot 1).
                    const int wh = (pp == 0 && step_start(cp, p) < ubeg) ? 1 : 0;
                    const float* src = p.ws_partials +
                                       ((size_t(cp) * 2 + size_t(wh)) * size_t(p.pieces) +
                                        piece0 + size_t(c)) * 512u + size_t(lane) * 16u;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float4 v = ptx::ldg_cg_f4(src + 4 * i);
                        acc[4 * i] += v.x, acc[4 * i + 1] += v.y;
                        acc[4 * i + 2] += v.z, acc[4 * i + 3] += v.w;
                    }
                }
                if (tp) tp_put(p, epoch, unit, q, c, lane, acc);
                else if (row_ok) store_row(nb, c, mrow, acc);
            }
            __syncwarp();
            if (lane == 0) *reinterpret_cast<volatile uint32_t*>(ctr) = 0u;  // ready for reuse
            if (tp) owned |= 1ull << (s & 63);
        }
        for (uint64_t todo = owned; todo; todo &= todo - 1) {
            const int s = __ffsll(static_cast<long long>(todo)) - 1;
            const int unit = unit0 + s, rb = unit % rbs;
            const int mrow = rb * 128 + lane_row(row);
            tp_collect(p, epoch, unit, q, lane, unit / rbs, mrow, mrow < p.m);
        }
    }

    __syncthreads();
    if (warp == 0) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, 2 * p.tmem_cols);
    }
    // Fused all-reduce: the last CTA to finish advances this rank's epoch
    // (every CTA read it in its epilogue, before this point).
    if (p.tp_world > 1 && tid == 0) {
        __threadfence();
        if (atomicAdd(p.tp_state + 1, 1u) == uint32_t(p.grid - 1)) {
            p.tp_state[1] = 0u;
            p.tp_state[0] = tp_epoch(p);
        }
    }
}

// ------------------------------------------------------------------ host

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<EncodeTiledFn>(f);
    }();
    return fn;
}

// Filled once per device; `sms` is published last (release), so a thread
// that reads it nonzero (acquire) also sees smem_optin.
struct DeviceInfo {
    std::atomic<int> sms{0};
    int smem_optin = 0;
    std::atomic<bool> gemm_attr{false};
};
constexpr int kMaxDevices = 64;
DeviceInfo g_devices[kMaxDevices];
std::mutex g_device_mutex;

DeviceInfo& device_info(int device) {
    DeviceInfo& d = g_devices[device];
    if (!d.sms.load(std::memory_order_acquire)) {
        std::lock_guard<std::mutex> lock(g_device_mutex);
        if (!d.sms.load(std::memory_order_relaxed)) {
            int smem = 0, sms = 0;
            cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
            d.smem_optin = smem;
            d.sms.store(sms, std::memory_order_release);
        }
    }
    return d;
}

uint32_t round_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

struct GemmLayout {
    uint32_t off_a, off_x, off_slots, x_bytes, total;
    SlotLayout slot;
    int nx, nslots;
};

// Shared memory: barriers | lookup tables | A tiles (na 16.1 KB 128 x 64
// BF16 tiles) | x ring (1024-aligned, nx slots of bn*128
// bytes) | compressed slots (2 * ndg / S, each S K slices: two K slices'
// worth per decoder group) | pad. The x ring gets one slot per A tile when
// they fit (then an x slot is freed by the same commit as its A tile), else
// as many as fit.
GemmLayout gemm_layout(int ndg, int na, int bn, uint32_t plane_pitch, uint32_t cap_c,
                       uint32_t cap_r, int smem_limit, int S) {
    GemmLayout l{};
    l.off_a = round_up(kBarrierBytes + kTableBytes, 1024);
    l.off_x = round_up(l.off_a + uint32_t(na) * kATileBytes, 1024);  // x tiles: 128-byte swizzle
    l.x_bytes = uint32_t(bn) * 128;
    l.slot = gemm_slot_layout(plane_pitch, cap_c, cap_r, S);
    // At least two K slices of compressed data per decoder group; the x ring
    // then takes one slot per A tile if it fits (two at least), and what is
    // left goes to more compressed slots (a deeper ring hides the refill
    // latency: a slot is refilled only after its last reader released it).
    const int min_slots = 2 * ndg / S;
    const uint32_t base = l.off_x + kRingPadBytes;
    const auto fits = [&](int nx, int ns) {
        return base + uint32_t(nx) * l.x_bytes + uint32_t(ns) * l.slot.bytes <=
               uint32_t(smem_limit);
    };
    l.nx = 0;
    for (int nx = std::min(kMaxX, na); nx >= 2 && !l.nx; --nx)
        if (fits(nx, min_slots)) l.nx = nx;
    l.nslots = min_slots;
    while (l.nx && l.nslots < kMaxStages && fits(l.nx, l.nslots + 1)) ++l.nslots;
    l.off_slots = l.off_x + uint32_t(l.nx) * l.x_bytes;
    l.total = l.off_slots + uint32_t(l.nslots) * l.slot.bytes + kRingPadBytes;
    return l;
}

}  // namespace

int device_sm_count(int device) { return device_info(device).sms; }

SlotLayout gemm_slot_layout(uint32_t plane_pitch, uint32_t cap_c, uint32_t cap_r, int S) {
    // S K slices of two tile rows: 2S tiles, tile (row r, slice j) at index
    // r*S + j. A bitmap plane's tile occupies plane_pitch bytes: the tensor
    // load's box is wider than the 64-word tile (the words past it
    // zero-filled), which puts consecutive tiles off each other modulo 128
    // bytes, so lanes decoding different tiles read different banks (528:
    // 16 bytes off; 576: 64 bytes off, with every plane 128-byte aligned as
    // separate tensor loads require). Then the tiles' band offsets (32 B
    // each), a header of tile-relative payload starts ([2][S] int2, written
    // by the producer), and per tile row one common and one rare run of its S
    // tiles. The row-1 common run starts 32 bytes further modulo 128: a
    // warp's lanes read the small tiles of one band of both tiles, whose
    // runs sit ~62 bytes apart, so within a tile they spread over the banks
    // in two interleaved combs ~half a bank row apart; a 32-byte shift puts
    // the other tile's lanes between them (64 would put them on the same
    // banks). Modelled on N(0, 0.02) weights: 3.2 instead of 4.3 shared
    // wavefronts per payload load.
    SlotLayout s{};
    const uint32_t us = uint32_t(S);
    s.plane1 = plane_pitch;
    s.plane_stride = 2u * us * plane_pitch;
    s.med = round_up(3u * s.plane_stride, 128);  // [2S][32 B]
    s.hdr = s.med + 64u * us;                    // [2S] int2
    s.common0 = round_up(s.hdr + 16u * us, 128);
    s.common1 = s.common0 + us * cap_c + 32;  // cap_c is a multiple of 128
    s.rare0 = round_up(s.common1 + us * cap_c, 16);
    s.rare1 = s.rare0 + us * cap_r * 2;
    s.bytes = round_up(s.rare1 + us * cap_r * 2, 128);
    return s;
}

SlotLayout decompress_slot_layout(int half, uint32_t cap_c, uint32_t cap_r) {
    SlotLayout s{};
    const uint32_t h = uint32_t(half);
    s.plane1 = 512u * h;           // second half of each plane
    s.plane_stride = 2u * 512u * h;
    s.med = 3u * s.plane_stride;   // [2*half][32 B]
    s.hdr = s.med + 2u * h * 32u;
    s.common0 = round_up(s.hdr + 2u * kMaxGroup * 8u, 128);
    s.common1 = s.common0 + h * cap_c + 64;
    s.rare0 = round_up(s.common1 + h * cap_c, 16);  // one run for the whole chunk
    s.rare1 = s.rare0;
    s.bytes = round_up(s.rare0 + 2u * h * cap_r * 2, 128);
    return s;
}

static bool encode_map(CUtensorMap* map, CUtensorMapDataType type, const void* base,
                       cuuint32_t rank, const cuuint64_t* dims, const cuuint64_t* strides,
                       const cuuint32_t* box, CUtensorMapSwizzle swizzle) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    return fn(map, type, rank, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_tensor_map_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                          uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer) {
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    return encode_map(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, 2, dims, strides, box,
                      CU_TENSOR_MAP_SWIZZLE_128B);
}

bool encode_plane_maps(PlaneMaps* maps, const void* b1, const void* b2, const void* b3,
                       uint64_t inner, uint64_t outer, uint32_t box_words, uint32_t box_inner,
                       uint32_t box_outer) {
    // A plane: [outer][inner] tiles of 64 u64 words (512 B); the box is
    // box_words wide (> 64: zero-filled padding after each tile).
    const cuuint64_t dims[4] = {64, inner, outer, 3};
    const cuuint32_t box[4] = {box_words, box_inner, box_outer, 3};
    const auto a1 = reinterpret_cast<uintptr_t>(b1), a2 = reinterpret_cast<uintptr_t>(b2),
               a3 = reinterpret_cast<uintptr_t>(b3);
    if (a2 > a1 && a2 - a1 == a3 - a2 && (a2 - a1) % 16 == 0 && a2 - a1 < (uint64_t(1) << 40)) {
        const cuuint64_t strides[3] = {512, inner * 512, a2 - a1};
        maps->count = 1;
        return encode_map(&maps->map[0], CU_TENSOR_MAP_DATA_TYPE_UINT64, b1, 4, dims, strides,
                          box, CU_TENSOR_MAP_SWIZZLE_NONE);
    }
    const cuuint64_t strides[2] = {512, inner * 512};
    const void* planes[3] = {b1, b2, b3};
    maps->count = 3;
    for (int i = 0; i < 3; ++i)
        if (!encode_map(&maps->map[i], CU_TENSOR_MAP_DATA_TYPE_UINT64, planes[i], 3, dims,
                        strides, box, CU_TENSOR_MAP_SWIZZLE_NONE))
            return false;
    return true;
}

static int tile_n(int n) { return n > 256 ? 256 : std::max(16, (n + 15) / 16 * 16); }

static cudaError_t ensure_gemm_attributes(int device) {
    DeviceInfo& d = device_info(device);
    if (d.gemm_attr) return cudaSuccess;
    cudaError_t e = cudaSuccess;
    for (auto fn : {zipgemm_kernel<4>, zipgemm_kernel<3>, zipgemm_kernel<2>}) {
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     d.smem_optin);
    }
    if (e == cudaSuccess) d.gemm_attr = true;
    else {
        char msg[160];
        snprintf(msg, sizeof(msg), "zipgemm: kernel attributes (shared memory %d) rejected: %s",
                 d.smem_optin, cudaGetErrorString(e));
        zs_set_error(msg);
    }
    return e;
}

// The persistent schedule of one launch (see the kernel's work schedule).
struct Schedule {
    int bn, row_blocks, units, steps, S, groups, grid, pieces;
    bool partial;  // some CTA range splits a unit: the fixup workspace is used
};

static Schedule make_schedule(int m, int n, int k, int kparts, int sms) {
    Schedule s{};
    const int kt = k / 64;
    s.bn = tile_n(n);
    s.row_blocks = (m / 64 + 1) / 2;
    s.units = s.row_blocks * ((n + s.bn - 1) / s.bn);
    s.steps = s.units * kt;
    // K slices per slot. Two slices per slot (half the copies per slice)
    // measured no faster on B200 than one (the fills are limited by how fast
    // data lands, not by copy issue), and a slot shared by two decoder
    // groups is released later; so one.
    s.S = 1;
    s.groups = s.steps / s.S;
    const int64_t want = kparts > 0 ? int64_t(s.units) * kparts : int64_t(std::max(1, sms));
    s.grid = int(std::max<int64_t>(1, std::min<int64_t>(want, s.groups)));
    s.pieces = s.bn / 4;
    s.partial = false;
    for (int c = 1; c < s.grid && !s.partial; ++c)
        if ((int64_t(s.S) * (int64_t(c) * s.groups / s.grid)) % kt) s.partial = true;
    return s;
}

// Fixup scratch of a schedule: FP32 partial tiles (any contents; at most two
// partial segments per CTA, its first and last) and one arrival counter per
// (CTA, TMEM lane quarter). Counters live in their own buffer, which holds
// zeros between launches (the launch that completes a unit returns its
// counter to zero), so launches of different shapes can share both buffers.
static size_t schedule_partial_bytes(const Schedule& s) {
    return s.partial ? size_t(s.grid) * 2u * size_t(s.pieces) * 512u * sizeof(float) : 0;
}
static size_t schedule_counter_bytes(const Schedule& s) {
    return s.partial ? (size_t(s.grid) * 4u * 4u + 15u) / 16u * 16u : 0;
}

// Library-owned fixup scratch, one pair of buffers per (device, stream):
// launches on one stream are ordered, so they can share it. The first launch
// that needs scratch on a stream allocates enough for every shape of the
// default schedule (one CTA per SM, N tile 256: 2 x 64 pieces of 2 KB per
// CTA, 38.8 MB on a 148-SM GPU), so later shapes never allocate. Only an
// explicit K partition with more CTAs than SMs can need more; buffers that
// are outgrown are kept (never freed: launches already queued or captured
// in a graph may still use them), so no launch ever waits for the stream.
// An allocation while the stream is being captured switches this thread to
// relaxed capture mode for the cudaMalloc (it enqueues nothing); the
// counters' zero-fill is then captured with the launch, so the first launch
// on the stream outside capture enqueues it once more. A graph keeps using
// the scratch of the stream it was captured on: replaying it while other
// work uses that stream's scratch (on any stream) races, as with any
// library workspace captured in a graph.
struct WorkspaceEntry {
    int device;
    cudaStream_t stream;
    void* partials;
    size_t partial_bytes;
    void* counters;
    size_t counter_bytes;
    bool zero_pending;  // counters zero-filled only inside a captured graph so far
};
std::vector<WorkspaceEntry> g_workspaces;
std::vector<void*> g_retired_workspaces;
std::mutex g_workspace_mutex;

static cudaError_t relaxed_malloc(void** ptr, size_t bytes) {
    cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
    cudaError_t e = cudaThreadExchangeStreamCaptureMode(&mode);
    if (e != cudaSuccess) return e;
    const cudaError_t a = cudaMalloc(ptr, bytes);
    e = cudaThreadExchangeStreamCaptureMode(&mode);  // restores the caller's mode
    return a != cudaSuccess ? a : e;
}

static cudaError_t library_workspace(int device, int sms, cudaStream_t stream,
                                     size_t partial_bytes, size_t counter_bytes,
                                     void** partials, void** counters) {
    std::lock_guard<std::mutex> lock(g_workspace_mutex);
    WorkspaceEntry* entry = nullptr;
    for (WorkspaceEntry& e : g_workspaces)
        if (e.device == device && e.stream == stream) entry = &e;
    if (!entry) {
        g_workspaces.push_back({device, stream, nullptr, 0, nullptr, 0, false});
        entry = &g_workspaces.back();
    }
    const size_t full_p = size_t(sms) * 2u * 64u * 512u * sizeof(float);
    const size_t full_c = (size_t(sms) * 16u + 15u) / 16u * 16u;
    cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
    cudaError_t e = cudaStreamIsCapturing(stream, &capture);
    if (e != cudaSuccess) return e;
    const bool capturing = capture != cudaStreamCaptureStatusNone;
    if (entry->partial_bytes < partial_bytes) {
        const size_t bytes = std::max(partial_bytes, full_p);
        void* fresh = nullptr;
        if ((e = relaxed_malloc(&fresh, bytes)) != cudaSuccess) {
            zs_set_error("zipgemm: could not allocate K-range scratch");
            return e;
        }
        if (entry->partials) g_retired_workspaces.push_back(entry->partials);
        entry->partials = fresh, entry->partial_bytes = bytes;
    }
    if (entry->counter_bytes < counter_bytes) {
        const size_t bytes = std::max(counter_bytes, full_c);
        void* fresh = nullptr;
        if ((e = relaxed_malloc(&fresh, bytes)) != cudaSuccess) {
            zs_set_error("zipgemm: could not allocate K-range counters");
            return e;
        }
        if ((e = cudaMemsetAsync(fresh, 0, bytes, stream)) != cudaSuccess) {
            g_retired_workspaces.push_back(fresh);
            return e;
        }
        if (entry->counters) g_retired_workspaces.push_back(entry->counters);
        entry->counters = fresh, entry->counter_bytes = bytes;
        entry->zero_pending = capturing;
    } else if (entry->zero_pending && !capturing) {
        if ((e = cudaMemsetAsync(entry->counters, 0, entry->counter_bytes, stream)) != cudaSuccess)
            return e;
        entry->zero_pending = false;
    }
    *partials = entry->partials;
    *counters = entry->counters;
    return cudaSuccess;
}

std::atomic<uint64_t> g_reducer_wait_ns{kReducerWaitNs};

uint64_t set_reducer_wait_ns(uint64_t ns) { return g_reducer_wait_ns.exchange(ns); }

void allreduce_exchange_bytes(int m, int n, int world, size_t* recv_bytes, size_t* flag_bytes) {
    *recv_bytes = *flag_bytes = 0;
    if (!valid_matrix(m, 64) || n <= 0 || world < 2 || world > kMaxTp) return;
    const Schedule s = make_schedule(m, n, 64, 0, 1);  // units and N tile do not depend on K
    *recv_bytes = size_t(2) * world * s.units * s.bn * 128u * sizeof(uint64_t);
    *flag_bytes = 16;  // reserved: values carry their own epoch
}

int plan_kparts(int m, int n, int k, int device) {
    if (!valid_matrix(m, k) || n <= 0) return -1;
    const Schedule s = make_schedule(m, n, k, 0, device_info(device).sms);
    return std::max(1, s.grid / s.units);
}

void gemm_workspace_bytes(int m, int n, int k, int kparts, int device, size_t* partial_bytes,
                          size_t* counter_bytes) {
    *partial_bytes = *counter_bytes = 0;
    if (!valid_matrix(m, k) || n <= 0) return;
    const Schedule s = make_schedule(m, n, k, kparts, device_info(device).sms);
    *partial_bytes = schedule_partial_bytes(s);
    *counter_bytes = schedule_counter_bytes(s);
}

cudaError_t launch_zipgemm(cudaStream_t stream, const void* sm, const void* rare, const void* b1,
                           const void* b2, const void* b3, const void* medium, const void* global,
                           int max_common, int max_rare, int start_exp, const void* x, void* y,
                           int m, int n, int k, int kparts, const GemmScratch* scratch,
                           const TpExchange* tp) {
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return e;
    if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
    DeviceInfo& d = device_info(device);
    if ((e = ensure_gemm_attributes(device)) != cudaSuccess) return e;
    const int kt = k / 64;
    const Schedule sched = make_schedule(m, n, k, std::max(0, kparts), d.sms);

    GemmParams p{};
    p.sm = static_cast<const uint8_t*>(sm);
    p.rare = static_cast<const uint16_t*>(rare);
    p.global = static_cast<const int*>(global);
    p.y = static_cast<uint16_t*>(y);
    p.m = m, p.n = n, p.k = k, p.kt = kt, p.row_tiles = m / 64;
    p.row_blocks = sched.row_blocks, p.units = sched.units, p.steps = sched.steps;
    p.S = sched.S, p.groups = sched.groups;
    p.grid = sched.grid, p.pieces = sched.pieces;
    // One CTA per SM (the shared-memory footprint allows no more): with at
    // most one CTA per SM every CTA of the grid normally runs at the same
    // time, and a row block's first part may wait (briefly) for the others.
    // Nothing depends on it: a reducer that waits in vain falls back to the
    // last-arrival reduction.
    p.resident = sched.grid <= d.sms ? 1 : 0;
    p.reducer_wait_ns = g_reducer_wait_ns.load(std::memory_order_relaxed);
    if (tp && tp->world > 1) {
        // A CTA keeps the segments it must collect in a 64-bit mask.
        const int per_cta = (sched.steps + sched.grid - 1) / sched.grid;
        if (per_cta / kt + 2 > 64) {
            zs_set_error("zipserv_mm_allreduce: more than 64 output segments per CTA (K/64 too "
                         "small for this M and N)");
            return cudaErrorInvalidValue;
        }
        p.tp_world = tp->world, p.tp_rank = tp->rank;
        for (int r = 0; r < tp->world; ++r) {
            p.tp_recv[r] = static_cast<uint64_t*>(tp->recv[r]);
        }
        p.tp_state = static_cast<uint32_t*>(tp->state);
    }
    p.bn = sched.bn;
    if (sched.partial) {
        const size_t need_p = schedule_partial_bytes(sched), need_c = schedule_counter_bytes(sched);
        void *partials = nullptr, *counters = nullptr;
        if (scratch) {
            if (!scratch->partials || !scratch->counters || scratch->partial_bytes < need_p ||
                scratch->counter_bytes < need_c ||
                ((reinterpret_cast<uintptr_t>(scratch->partials) |
                  reinterpret_cast<uintptr_t>(scratch->counters)) & 15u)) {
                zs_set_error("zipgemm: caller scratch missing, too small or not 16-byte aligned");
                return cudaErrorInvalidValue;
            }
            partials = scratch->partials, counters = scratch->counters;
        } else if ((e = library_workspace(device, d.sms, stream, need_p, need_c, &partials,
                                          &counters)) != cudaSuccess) {
            return e;
        }
        p.ws_counters = static_cast<uint32_t*>(counters);
        p.ws_partials = static_cast<float*>(partials);
    }
    p.cap_c = common_capacity(max_common);
    p.cap_r = uint32_t(max_rare);
    p.start_exp = uint32_t(start_exp) & 255u;
    {
        // Exponent palette: byte c = exponent start_exp + c rotated right by
        // one bit (bit 7 = its bit 0, bits 0-6 = its bits 1-7).
        uint32_t xp[2] = {0, 0};
        for (int c = 1; c < 8; ++c) {
            const uint32_t e = (p.start_exp + uint32_t(c)) & 255u;
            xp[c >> 2] |= (((e & 1u) << 7) | (e >> 1)) << (8 * (c & 3));
        }
        p.dk = DecodeConsts{2u, 4u, 8u, uint32_t(kTableCopies) * 4u, 0x11111110u, 0x10000u,
                            xp[0], xp[1]};
    }
    // Bitmap tensor maps. Equally spaced planes (one allocation, as the
    // runtime lays them out) load with one 4-D copy into a 528-byte pitch;
    // otherwise three copies need 128-byte aligned planes: pitch 576. 512
    // (no bank offset) if the driver rejects a box wider than the tile.
    PlaneMaps pm;
    const auto a1 = reinterpret_cast<uintptr_t>(b1), a2 = reinterpret_cast<uintptr_t>(b2),
               a3 = reinterpret_cast<uintptr_t>(b3);
    const bool spaced = a2 > a1 && a2 - a1 == a3 - a2 && (a2 - a1) % 16 == 0 &&
                        a2 - a1 < (uint64_t(1) << 40);  // the test encode_plane_maps makes
    uint32_t pitch = spaced ? 528 : 576;
    const uint32_t S = uint32_t(sched.S);
    if (!encode_plane_maps(&pm, b1, b2, b3, uint64_t(kt), uint64_t(m / 64), pitch / 8, S, 2)) {
        pitch = 512;
        if (!encode_plane_maps(&pm, b1, b2, b3, uint64_t(kt), uint64_t(m / 64), 64, S, 2)) {
            zs_set_error("zipgemm: bitmap tensor maps rejected (bitmaps must be 16-byte aligned)");
            return cudaErrorInvalidValue;
        }
    }
    p.plane_box_bytes = 3u * 2u * S * pitch;
    // Band offsets as [row tiles][k tiles][4 u64]: one box = both tile rows.
    CUtensorMap mmap;
    {
        const cuuint64_t dims[3] = {4, uint64_t(kt), uint64_t(m / 64)};
        const cuuint64_t strides[2] = {32, uint64_t(kt) * 32};
        const cuuint32_t box[3] = {4, S, 2};
        if (!encode_map(&mmap, CU_TENSOR_MAP_DATA_TYPE_UINT64, medium, 3, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_NONE)) {
            zs_set_error("zipgemm: band-offset tensor map rejected (must be 16-byte aligned)");
            return cudaErrorInvalidValue;
        }
    }
    // (decoder groups, A tiles per group), best first (measured): four
    // groups with one A tile each (more decode throughput, some stalls on
    // the previous slice's MMAs), then fewer groups with double-buffered A
    // tiles. The x ring needs at least two slots.
    struct Choice {
        int ndg, na;
    };
    constexpr Choice kChoices[] = {{4, 4}, {3, 6}, {2, 4}, {2, 2}};
    int ndg = 0;
    GemmLayout l{};
    for (const Choice& c : kChoices) {
        l = gemm_layout(c.ndg, c.na, p.bn, pitch, p.cap_c, p.cap_r, d.smem_optin, sched.S);
        if (l.nx >= 2) {
            ndg = c.ndg;
            p.na = c.na;
            break;
        }
    }
    if (!ndg) {
        zs_set_error("zipgemm: packed payload capacity leaves no room for the shared-memory rings");
        return cudaErrorInvalidConfiguration;
    }
    p.nx = l.nx;
    p.nslots = l.nslots;
    p.off_a = l.off_a, p.off_x = l.off_x;
    p.off_slots = l.off_slots, p.x_bytes = l.x_bytes, p.slot = l.slot;
    // TMEM holds two FP32 accumulators of bn columns (consecutive segments
    // alternate, so one can drain while the next accumulates).
    uint32_t cols = 32;
    while (cols < uint32_t(p.bn)) cols <<= 1;
    p.tmem_cols = cols;

    // x viewed as [K/64][N][64]: one box = one K slice of bn tokens, a
    // 128-byte-swizzled bn x 64 tile.
    CUtensorMap xmap;
    const cuuint64_t dims[3] = {64, uint64_t(n), uint64_t(kt)};
    const cuuint64_t strides[2] = {uint64_t(k) * 2, 128};
    const cuuint32_t box[3] = {64, uint32_t(p.bn), 1};
    if (!encode_map(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, 3, dims, strides, box,
                    CU_TENSOR_MAP_SWIZZLE_128B)) {
        zs_set_error("zipgemm: activation tensor map rejected (x must be 16-byte aligned)");
        return cudaErrorInvalidValue;
    }

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(sched.grid), 1, 1);
    cfg.blockDim = dim3(gemm_threads(ndg), 1, 1);
    cfg.dynamicSmemBytes = l.total;
    cfg.stream = stream;
    // Programmatic dependent launch: the prologue and the first weight
    // copies overlap the previous kernel's tail; x is read and the output
    // written only after it completes (griddepcontrol.wait in the kernel).
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = ndg == 4   ? cudaLaunchKernelEx(&cfg, zipgemm_kernel<4>, xmap, pm, mmap, p)
        : ndg == 3 ? cudaLaunchKernelEx(&cfg, zipgemm_kernel<3>, xmap, pm, mmap, p)
                   : cudaLaunchKernelEx(&cfg, zipgemm_kernel<2>, xmap, pm, mmap, p);
    if (e != cudaSuccess) {
        char msg[220];
        snprintf(msg, sizeof(msg),
                 "zipgemm launch (grid %u, %u B shared, %d decoder groups, %d x slots, bn %d): %s",
                 cfg.gridDim.x, l.total, ndg, l.nx, p.bn, cudaGetErrorString(e));
        zs_set_error(msg);
    }
    return e;
}

}  // namespace zs
