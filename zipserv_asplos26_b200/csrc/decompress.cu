// Standalone TCA-TBE decompression to a dense row-major BF16 matrix in HBM,
// for large-N (prefill) calls that decode once and then run a dense GEMM.
//
// Persistent grid, one CTA per SM. The CTA walks chunks of 2*half
// consecutive global tiles (row-major tile order) with stride gridDim.x; the
// packed streams of a chunk are contiguous, so each half of it arrives with
// six bulk copies whatever its length. Warp roles:
//   warp 0     producer: bulk async copies of each chunk's bitmaps, band
//              offsets and payloads into a ring of shared-memory slots;
//   warps 1..8 two decoder groups (four warps each, one chunk per group at
//              a time); pair j of a chunk is tile j of each half, and warp w
//              decodes 16-row band w%4 of both tiles of the pair, a thread
//              rebuilding one 64-element row with the shared row decoder.
//              The warp writes its rows into a 32x64 staging tile in the
//              128-byte-swizzled layout and one lane stores each 16-row half
//              to HBM with a TMA tensor store (full 128-byte lines,
//              double-buffered so decoding overlaps the store).
// Reference kernel this replaces: csrc/L_Kernel.cuh:1147-1278 (one tile per
// CTA, load -> sync -> decode -> sync -> 16-byte stores, no overlap).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include <cstdio>

#include "capi_internal.h"
#include "codec.h"
#include "decode.cuh"
#include "ptx.cuh"
#include "zipgemm.cuh"

namespace zs {

constexpr int kDecGroups = 2;
constexpr int kDecThreads = 32 + 128 * kDecGroups;
constexpr int kDecStages = 8;  // ring slots at most; fewer when payload capacities are large
constexpr uint32_t kOutTileBytes = 32 * 128;  // one warp's 32 rows x 64 BF16

__global__ void __launch_bounds__(kDecThreads, 1)
    decompress_kernel(const __grid_constant__ CUtensorMap omap, const DecompressParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t sbase = ptx::smem_addr(smem);
    const uint32_t bar_full = sbase, bar_empty = sbase + 8 * kDecStages;
    const uint32_t bar_tab = sbase + 16 * kDecStages;
    const uint32_t tables = sbase + kBarrierBytes;
    const uint32_t cap_c = p.cap_c, cap_r = p.cap_r;
    const int H = p.half, C = 2 * p.half;
    const uint32_t pstride = 512u * uint32_t(H);
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
        ptx::mbar_arrive_expect_tx(bar_tab, kTableBytes);
        ptx::bulk_g2s(tables, &g_decode_tables, kTableBytes, bar_tab, ptx::policy_evict_last());
    }

    if (warp == 0) {
        // ------------------------------------------------------ producer
        const uint64_t pol = ptx::policy_evict_first();
        const int2* goffs = reinterpret_cast<const int2*>(p.global);
        // Lane i holds offset entry i (tiles t0 + i, i <= C) of the chunk in
        // flight; the next chunk's entries are loaded one iteration early.
        auto load = [&](int it) {
            const int t = (int(blockIdx.x) + it * int(gridDim.x)) * C + lane;
            return (it < nlocal && lane <= C) ? goffs[min(t, p.tiles)] : make_int2(0, 0);
        };
        int2 next = load(0);
        bool ok = true;
        int issued = 0;
        for (int it = 0; it < nlocal; ++it) {
            const int2 cur = next;
            next = load(it + 1);
            const int s = it % p.nstages;
            if (it >= p.nstages && lane == 0)
                ok = ptx::mbar_wait(bar_empty + 8 * s, ((it / p.nstages) - 1) & 1);
            ok = __shfl_sync(kFullMask, ok, 0) != 0;
            if (!ok) break;
            const int t0 = (int(blockIdx.x) + it * int(gridDim.x)) * C;
            const uint32_t slot = sbase + p.off_slots + uint32_t(s) * p.slot.bytes;
            const uint32_t full = bar_full + 8 * s;
            int nt[2];
            nt[0] = min(H, p.tiles - t0);
            nt[1] = max(0, min(H, p.tiles - t0 - H));
            uint32_t clen[2] = {0, 0}, rlen[2] = {0, 0};
            int2 g0[2];
            uint32_t bytes = 0;
            for (int tau = 0; tau < 2; ++tau) {
                g0[tau].x = __shfl_sync(kFullMask, cur.x, tau * H);
                g0[tau].y = __shfl_sync(kFullMask, cur.y, tau * H);
                const int ex = __shfl_sync(kFullMask, cur.x, tau * H + nt[tau]);
                const int ey = __shfl_sync(kFullMask, cur.y, tau * H + nt[tau]);
                // Payload copies need 16-byte aligned sources; offsets of
                // valid packed data always are.
                if (nt[tau] && (g0[tau].x & 15) == 0)
                    clen[tau] = min(uint32_t(max(ex - g0[tau].x, 0)), uint32_t(H) * cap_c) & ~15u;
                if (nt[tau] && (g0[tau].y & 7) == 0)
                    rlen[tau] =
                        (min(uint32_t(max(ey - g0[tau].y, 0)), uint32_t(H) * cap_r) * 2u) & ~15u;
                bytes += 3u * 512u * uint32_t(nt[tau]) + 32u * uint32_t(nt[tau]) + clen[tau] +
                         rlen[tau];
            }
            // Per-tile payload starts relative to the half's run, clamped so
            // tile i reads inside its region whatever the offsets say; tiles
            // missing at the end of the matrix get zero starts.
            if (lane < C) {
                const int tau = lane >= H, i = lane - tau * H;
                int2 h = make_int2(0, 0);
                if (i < nt[tau])
                    h = make_int2(min(max(cur.x - g0[tau].x, 0), int(uint32_t(i) * cap_c)),
                                  min(max(cur.y - g0[tau].y, 0), int(uint32_t(i) * cap_r)));
                reinterpret_cast<int2*>(smem + p.off_slots + uint32_t(s) * p.slot.bytes +
                                        p.slot.hdr)[tau * kMaxGroup + i] = h;
            }
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive_expect_tx(full, bytes);
            __syncwarp();
            if (lane < 12) {
                const int tau = lane / 6, c = lane % 6;
                const size_t t = size_t(t0 + tau * H);
                if (nt[tau]) {
                    if (c < 3) {
                        const uint64_t* src = c == 0 ? p.b1 : c == 1 ? p.b2 : p.b3;
                        ptx::bulk_g2s(slot + (tau ? p.slot.plane1 : 0u) + uint32_t(c) * pstride,
                                      src + t * 64, 512u * uint32_t(nt[tau]), full, pol);
                    } else if (c == 3) {
                        ptx::bulk_g2s(slot + p.slot.med + uint32_t(tau) * 32u * H, p.medium + t * 8,
                                      32u * uint32_t(nt[tau]), full, pol);
                    } else if (c == 4) {
                        if (clen[tau])
                            ptx::bulk_g2s(slot + (tau ? p.slot.common1 : p.slot.common0),
                                          p.sm + g0[tau].x, clen[tau], full, pol);
                    } else if (rlen[tau]) {
                        ptx::bulk_g2s(slot + (tau ? p.slot.rare1 : p.slot.rare0), p.rare + g0[tau].y,
                                      rlen[tau], full, pol);
                    }
                }
            }
            ++issued;
        }
        if (lane == 0)
            for (int it = max(0, issued - p.nstages); it < issued; ++it)
                ptx::mbar_wait(bar_full + 8 * (it % p.nstages), (it / p.nstages) & 1);
        __syncwarp();
    } else {
        // ------------------------------------------------------ decoders
        // Group g takes chunks g, g + kDecGroups, ...; within a chunk, pair j
        // is tile j of each half (lanes 0-15: half 0, lanes 16-31: half 1).
        const int dw = warp - 1, g = dw >> 2, q = dw & 3;
        const int tau = lane >> 4;
        RowDecoder<8 * 128 * kDecGroups> dec;
        dec.init(tables, sbase + p.off_rb + uint32_t(dw * 32 + lane) * 8u, lane, q, p.start_exp);
        const uint32_t obuf = sbase + p.off_out + uint32_t(dw) * 2 * kOutTileBytes;
        uint32_t out[32];
        int nstore = 0;
        bool ok = ptx::mbar_wait(bar_tab, 0);
        for (int it = g; it < nlocal; it += kDecGroups) {
            const int s = it % p.nstages;
            ok = ok && ptx::mbar_wait(bar_full + 8 * s, (it / p.nstages) & 1);
            if (!__all_sync(kFullMask, ok)) break;
            const int t0 = (int(blockIdx.x) + it * int(gridDim.x)) * C;
            const int n0 = min(H, p.tiles - t0), n1 = max(0, min(H, p.tiles - t0 - H));
            const uint32_t slot = ptx::launder(sbase + p.off_slots + uint32_t(s) * p.slot.bytes);
            const uint32_t plane = slot + (tau ? p.slot.plane1 : 0u);
            const uint32_t med = slot + p.slot.med + uint32_t(tau) * 32u * H;
            const uint32_t com = slot + (tau ? p.slot.common1 : p.slot.common0);
            const uint32_t rar = slot + (tau ? p.slot.rare1 : p.slot.rare0);
            for (int j = 0; j < n0; ++j) {
                const int2 hdr = ptx::lds_s64(slot + p.slot.hdr + uint32_t(tau * kMaxGroup + j) * 8u);
                dec.decode(plane + 512u * uint32_t(j), pstride, med + 32u * uint32_t(j),
                           com + uint32_t(hdr.x), rar + 2u * uint32_t(hdr.y), cap_c, cap_r, out);
                // Stage the warp's 32 rows: row `lane`, 16-byte chunk c at
                // position c ^ (row & 7) (the TMA 128-byte swizzle).
                const uint32_t buf = obuf + uint32_t(nstore & 1) * kOutTileBytes;
                if (lane == 0) ptx::bulk_wait_read<1>();
                __syncwarp();
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    ptx::sts128(buf + uint32_t(lane) * 128 + ((uint32_t(c) ^ (lane & 7)) << 4),
                                make_uint4(out[4 * c], out[4 * c + 1], out[4 * c + 2], out[4 * c + 3]));
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
                ++nstore;
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
int g_dec_smem_set[64];
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
    p.b1 = static_cast<const uint64_t*>(b1);
    p.b2 = static_cast<const uint64_t*>(b2);
    p.b3 = static_cast<const uint64_t*>(b3);
    p.medium = static_cast<const int*>(medium);
    p.global = static_cast<const int*>(global);
    p.m = m, p.k = k, p.kt = k / 64;
    p.tiles = (m / 64) * (k / 64);
    p.cap_c = common_capacity(max_common);
    p.cap_r = uint32_t(max_rare);
    p.start_exp = uint32_t(start_exp) & 255u;
    p.off_rb = kBarrierBytes + kTableBytes;
    p.off_out = round_up_u(p.off_rb + 128 * kDecGroups * kRowBufferBytes, 1024);
    p.off_slots = p.off_out + 4 * kDecGroups * 2 * kOutTileBytes;
    const uint32_t used = p.off_slots + kRingPadBytes;
    const uint32_t avail = uint32_t(smem_optin) > used ? uint32_t(smem_optin) - used : 0;
    // Largest half (tiles per copy run) that still leaves four slots, else
    // two; the slot count is a multiple of the group count so each group
    // owns the slots it consumes.
    p.nstages = 0;
    for (int min_slots : {4, 2}) {
        for (int half : {4, 2, 1}) {
            const SlotLayout l = slot_layout(half, p.cap_c, p.cap_r);
            const int n = std::min<int>(kDecStages, int(avail / l.bytes)) / kDecGroups * kDecGroups;
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
    const int sms = device_sm_count(device);
    const int grid = std::max(1, std::min(p.chunks, sms));
    decompress_kernel<<<grid, kDecThreads, total, stream>>>(omap, p);
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
