// Standalone TCA-TBE decompression to a dense row-major BF16 matrix in HBM,
// for large-N (prefill) calls that decode once and then run a dense GEMM.
//
// Persistent grid, one CTA per SM. The CTA walks chunks of 2*half
// consecutive global tiles (row-major tile order) with stride gridDim.x; the
// packed streams of a chunk are contiguous, so a chunk arrives with five
// copies whatever its length. Warp roles:
//   warp 0, warps after the decoders
//              producers (chunks rotate between them): bulk async copies
//              of each chunk's bitmaps, band offsets and payloads into a
//              ring of shared-memory slots;
//   warps 1..16 four decoder groups (four warps each, one chunk per group
//              at a time); pair j of a chunk is tile j of each half, and warp
//              w decodes 16-row band w%4 of both tiles of the pair, a thread
//              rebuilding one 64-element row with the shared row decoder.
//              The warp writes its rows into a 32x64 staging tile in the
//              128-byte-swizzled layout and one lane stores each 16-row half
//              to HBM with a TMA tensor store (full 128-byte lines); the next
//              pair is decoded while the store drains and only its staging
//              waits for the store to have read the tile.
// Sixteen decoder warps (four per SM sub-partition) hide the decoder's
// instruction latencies; fewer leave the issue slots half idle.
// Reference kernel this replaces: csrc/L_Kernel.cuh:1147-1278 (one tile per
// CTA, load -> sync -> decode -> sync -> 16-byte stores, no overlap).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>

#include <cstdio>

#include "capi_internal.h"
#include "codec.h"
#include "decode.cuh"
#include "ptx.cuh"
#include "zipgemm.cuh"

namespace zs {

constexpr int kDecGroups = 4;
constexpr int kDecProducers = 3;
constexpr int kDecThreads = 32 * kDecProducers + 128 * kDecGroups;
constexpr int kDecStages = 12;  // ring slots at most; fewer when payload capacities are large
constexpr uint32_t kOutTileBytes = 32 * 128;  // one warp's 32 rows x 64 BF16

__global__ void __launch_bounds__(kDecThreads, 1)
    decompress_kernel(const __grid_constant__ CUtensorMap omap,
                      const __grid_constant__ PlaneMaps pm, const DecompressParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t sbase = ptx::smem_addr(smem);
    const uint32_t bar_full = sbase, bar_empty = sbase + 8 * kDecStages;
    const uint32_t bar_tab = sbase + 16 * kDecStages;
    const uint32_t tables = sbase + kBarrierBytes;
    const uint32_t cap_c = p.cap_c, cap_r = p.cap_r;
    const int H = p.half, C = 2 * p.half;
    const SlotLayout L = p.slot;
    const int nlocal = p.chunks > int(blockIdx.x)
                           ? (p.chunks - int(blockIdx.x) + int(gridDim.x) - 1) / int(gridDim.x)
                           : 0;

    if (tid == 0) {
        for (int s = 0; s < kDecStages; ++s) {
            ptx::mbar_init(bar_full + 8 * s, 1);
            ptx::mbar_init(bar_empty + 8 * s, 4);
        }
        ptx::mbar_init(bar_tab, 1);
        ptx::fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
        ptx::prefetch_tensormap(&omap);
        for (int i = 0; i < pm.count; ++i) ptx::prefetch_tensormap(&pm.map[i]);
        ptx::mbar_arrive_expect_tx(bar_tab, kTableBytes);
        ptx::bulk_g2s(tables, &g_decode_tables, kTableBytes, bar_tab, ptx::policy_evict_last());
    }

    if (warp == 0 || warp > 4 * kDecGroups) {
        // ------------------------------------------------------ producers
        // Per chunk: one tensor load for the bitmap planes (tiles past the end
        // arrive zero-filled), one bulk copy of the band offsets, one of each
        // half's common payload and one of the chunk's rare payload.
        // This producer's chunks: pi, pi + kDecProducers, ...
        const int pi = warp == 0 ? 0 : warp - 4 * kDecGroups;
        const uint64_t pol = ptx::policy_evict_first();
        const int2* goffs = reinterpret_cast<const int2*>(p.global);
        const uint32_t plane_bytes = 3u * 512u * uint32_t(C);
        // Lane i holds offset entry i (tile t0 + i, i <= C) of the chunk in
        // flight; the next chunk's entries are loaded one iteration early.
        auto load = [&](int it) {
            const int t = (int(blockIdx.x) + it * int(gridDim.x)) * C + lane;
            return (it < nlocal && lane <= C) ? goffs[min(t, p.tiles)] : make_int2(0, 0);
        };
        int2 next = load(pi);
        bool ok = true;
        int last = -1;  // last chunk issued
        for (int it = pi; it < nlocal; it += kDecProducers) {
            const int2 cur = next;
            next = load(it + kDecProducers);
            const int s = it % p.nstages;
            if (it >= p.nstages && lane == 0)
                ok = ptx::mbar_wait(bar_empty + 8 * s, ((it / p.nstages) - 1) & 1);
            ok = __shfl_sync(kFullMask, ok, 0) != 0;
            if (!ok) break;
            const int t0 = (int(blockIdx.x) + it * int(gridDim.x)) * C;
            const uint32_t slot = sbase + p.off_slots + uint32_t(s) * L.bytes;
            const uint32_t full = bar_full + 8 * s;
            const int n = min(C, p.tiles - t0);  // tiles in this chunk
            const int nt0 = min(H, n), nt1 = n - nt0;
            int2 st[2], en[2];
            st[0].x = __shfl_sync(kFullMask, cur.x, 0), st[0].y = __shfl_sync(kFullMask, cur.y, 0);
            en[0].x = __shfl_sync(kFullMask, cur.x, nt0);
            st[1].x = en[0].x;
            en[1].x = __shfl_sync(kFullMask, cur.x, n);
            en[1].y = __shfl_sync(kFullMask, cur.y, n);
            // Payload copies need 16-byte aligned sources; offsets of valid
            // packed data always are.
            const uint32_t clen0 =
                (st[0].x & 15) == 0 ? min(uint32_t(max(en[0].x - st[0].x, 0)), uint32_t(H) * cap_c) & ~15u : 0u;
            const uint32_t clen1 = nt1 && (st[1].x & 15) == 0
                                       ? min(uint32_t(max(en[1].x - st[1].x, 0)), uint32_t(H) * cap_c) & ~15u
                                       : 0u;
            const uint32_t rlen =
                (st[0].y & 7) == 0
                    ? (min(uint32_t(max(en[1].y - st[0].y, 0)), uint32_t(C) * cap_r) * 2u) & ~15u
                    : 0u;
            // Per-tile payload starts (common: within its half's run; rare:
            // within the chunk's run), clamped so tile i reads inside its
            // region whatever the offsets say; missing tiles get zero starts.
            if (lane < C) {
                const int tau = lane >= H, i = lane - tau * H;
                int2 h = make_int2(0, 0);
                if (lane < n)
                    h = make_int2(min(max(cur.x - st[tau].x, 0), int(uint32_t(i) * cap_c)),
                                  min(max(cur.y - st[0].y, 0), int(uint32_t(lane) * cap_r)));
                reinterpret_cast<int2*>(smem + p.off_slots + uint32_t(s) * L.bytes +
                                        L.hdr)[tau * kMaxGroup + i] = h;
            }
            __syncwarp();
            if (lane == 0)
                ptx::mbar_arrive_expect_tx(full, plane_bytes + 32u * uint32_t(n) + clen0 + clen1 + rlen);
            __syncwarp();
            ptx::load_planes(slot, L.plane_stride, pm.map, pm.count, t0, 0, full, pol, lane);
            if (lane == 3)
                ptx::bulk_g2s(slot + L.med, p.medium + size_t(t0) * 8, 32u * uint32_t(n), full, pol);
            if (lane == 4 && clen0) ptx::bulk_g2s(slot + L.common0, p.sm + st[0].x, clen0, full, pol);
            if (lane == 5 && clen1) ptx::bulk_g2s(slot + L.common1, p.sm + st[1].x, clen1, full, pol);
            if (lane == 6 && rlen) ptx::bulk_g2s(slot + L.rare0, p.rare + st[0].y, rlen, full, pol);
            last = it;
        }
        // Never leave copies in flight: wait for this producer's chunks that
        // are the last use of their slot (earlier uses were consumed before
        // their slot was refilled; a later use, possibly another producer's,
        // would advance the barrier past the awaited phase).
        if (lane == 0)
            for (int it = last; it >= 0 && it >= nlocal - p.nstages; it -= kDecProducers)
                ptx::mbar_wait(bar_full + 8 * (it % p.nstages), (it / p.nstages) & 1);
        __syncwarp();
    } else {
        // ------------------------------------------------------ decoders
        // Group g takes chunks g, g + kDecGroups, ...; within a chunk, pair j
        // is tile j of each half (lanes 0-15: half 0, lanes 16-31: half 1).
        const int dw = warp - 1, g = dw >> 2, q = dw & 3;
        const int tau = lane >> 4;
        RowDecoder dec;
        dec.init(tables, lane, q, p.start_exp);
        const uint32_t obuf = sbase + p.off_out + uint32_t(dw) * kOutTileBytes;
        uint32_t out[32];
        RareState rs;
        bool ok = ptx::mbar_wait(bar_tab, 0);
        for (int it = g; it < nlocal; it += kDecGroups) {
            const int s = it % p.nstages;
            ok = ok && ptx::mbar_wait(bar_full + 8 * s, (it / p.nstages) & 1);
            if (!__all_sync(kFullMask, ok)) break;
            const int t0 = (int(blockIdx.x) + it * int(gridDim.x)) * C;
            const int n0 = min(H, p.tiles - t0), n1 = max(0, min(H, p.tiles - t0 - H));
            const uint32_t slot = ptx::launder(sbase + p.off_slots + uint32_t(s) * L.bytes);
            const uint32_t plane = slot + uint32_t(tau) * L.plane1;
            const uint32_t med = slot + L.med + uint32_t(tau * H) * 32u;
            const uint32_t com = slot + (tau ? L.common1 : L.common0);
            for (int j = 0; j < n0; ++j) {
                const int2 hdr = ptx::lds_s64(slot + L.hdr + uint32_t(tau * kMaxGroup + j) * 8u);
                dec.decode(plane + 512u * uint32_t(j), L.plane_stride, med + 32u * uint32_t(j),
                           com + uint32_t(hdr.x), cap_c, cap_r, out, rs);
                // Stage the warp's 32 rows: row `lane`, 16-byte chunk c at
                // position c ^ (row & 7) (the TMA 128-byte swizzle); rare
                // elements are patched in place. A missing second tile is
                // staged but never stored.
                const uint32_t buf = obuf;
                if (lane == 0) ptx::bulk_wait_read<0>();  // previous pair's store has read it
                __syncwarp();
                dec.store(buf + uint32_t(lane) * 128u, uint32_t(lane & 7) << 4, out, rs,
                          slot + L.rare0 + 2u * uint32_t(hdr.y), cap_r, tau == 1 && j >= n1);
                ptx::fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    const int ta = t0 + j, tb = t0 + H + j;
                    ptx::tma_store_2d(&omap, (ta % p.kt) * 64, (ta / p.kt) * 64 + 16 * q, buf);
                    if (j < n1)
                        ptx::tma_store_2d(&omap, (tb % p.kt) * 64, (tb / p.kt) * 64 + 16 * q,
                                          buf + 16 * 128);
                    ptx::bulk_commit();
                }
            }
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(bar_empty + 8 * s);
        }
        if (lane == 0) ptx::bulk_wait<0>();
        __syncwarp();
    }
}

namespace {
uint32_t round_up_u(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }
std::atomic<int> g_dec_smem_set[64];  // shared-memory attribute set on a device
}  // namespace

cudaError_t launch_decompress(cudaStream_t stream, const void* sm, const void* rare,
                              const void* b1, const void* b2, const void* b3,
                              const void* medium, const void* global, int max_common,
                              int max_rare, int start_exp, void* out, int m, int k) {
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return e;
    if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
    int smem_optin = 0;
    cudaDeviceGetAttribute(&smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    DecompressParams p{};
    p.sm = static_cast<const uint8_t*>(sm);
    p.rare = static_cast<const uint16_t*>(rare);
    p.medium = static_cast<const int*>(medium);
    p.global = static_cast<const int*>(global);
    p.m = m, p.k = k, p.kt = k / 64;
    p.tiles = (m / 64) * (k / 64);
    p.cap_c = common_capacity(max_common);
    p.cap_r = uint32_t(max_rare);
    p.start_exp = uint32_t(start_exp) & 255u;
    p.off_out = round_up_u(kBarrierBytes + kTableBytes, 1024);
    p.off_slots = p.off_out + 4 * kDecGroups * kOutTileBytes;
    const uint32_t used = p.off_slots + kRingPadBytes;
    const uint32_t avail = uint32_t(smem_optin) > used ? uint32_t(smem_optin) - used : 0;
    // Largest half (tiles per copy run) that still leaves two slots per
    // decoder group (one being decoded, one landing), else fewer. Chunk i
    // uses slot i % nstages whatever group decodes it.
    p.nstages = 0;
    for (int min_slots : {2 * kDecGroups, kDecGroups + 2, 2}) {
        for (int half : {4, 2, 1}) {
            const SlotLayout l = decompress_slot_layout(half, p.cap_c, p.cap_r);
            const int n = std::min<int>(kDecStages, int(avail / l.bytes));
            if (n >= min_slots) {
                p.half = half, p.slot = l, p.nstages = n;
                break;
            }
        }
        if (p.nstages) break;
    }
    if (p.nstages < 2) {
        zs_set_error("decompress: packed payload capacity leaves room for fewer than two stages");
        return cudaErrorInvalidConfiguration;
    }
    p.chunks = (p.tiles + 2 * p.half - 1) / (2 * p.half);
    const uint32_t total = p.off_slots + uint32_t(p.nstages) * p.slot.bytes + kRingPadBytes;
    if (!g_dec_smem_set[device]) {
        e = cudaFuncSetAttribute(decompress_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 smem_optin);
        if (e != cudaSuccess) {
            char msg[160];
            snprintf(msg, sizeof(msg), "decompress: shared memory limit %d rejected: %s",
                     smem_optin, cudaGetErrorString(e));
            zs_set_error(msg);
            return e;
        }
        g_dec_smem_set[device] = 1;
    }
    CUtensorMap omap;
    if (!encode_tensor_map_2d(&omap, out, uint64_t(k), uint64_t(m), uint64_t(k) * 2, 64, 16)) {
        zs_set_error("decompress: output tensor map rejected (output must be 16-byte aligned)");
        return cudaErrorInvalidValue;
    }
    PlaneMaps pm;
    if (!encode_plane_maps(&pm, b1, b2, b3, uint64_t(p.tiles), 1, 64, uint32_t(2 * p.half), 1)) {
        zs_set_error("decompress: bitmap tensor maps rejected (bitmaps must be 16-byte aligned)");
        return cudaErrorInvalidValue;
    }
    p.plane_maps = pm.count;
    const int sms = device_sm_count(device);
    const int grid = std::max(1, std::min(p.chunks, sms));
    decompress_kernel<<<grid, kDecThreads, total, stream>>>(omap, pm, p);
    e = cudaGetLastError();
    if (e != cudaSuccess) {
        char msg[200];
        snprintf(msg, sizeof(msg),
                 "decompress launch (grid %d, %d threads, %u B shared, %d slots x %d tiles): %s",
                 grid, kDecThreads, total, p.nstages, 2 * p.half, cudaGetErrorString(e));
        zs_set_error(msg);
    }
    return e;
}

}  // namespace zs
