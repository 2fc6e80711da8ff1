// Standalone TCA-TBE decompression to a dense row-major BF16 matrix in HBM,
// for large-N (prefill) calls that decode once and then run a dense GEMM.
//
// Persistent grid, one CTA per SM. The CTA walks pairs of global tiles
// (2p, 2p+1 in row-major tile order) with stride gridDim.x. Warp roles:
//   warp 0     producer: bulk async copies of each pair's bitmaps, band
//              offsets and payloads into a ring of shared-memory slots;
//   warps 1..8 two decoder groups (four warps each, one pair per group at a
//              time); a thread rebuilds one 64-element row with the shared
//              row decoder, writes it into a per-warp 32x64 staging tile in
//              the 128-byte-swizzled layout, and one lane per warp stores the
//              tile to HBM with a TMA tensor store (full 128-byte lines,
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
constexpr uint32_t kPairMedium = 3072;
constexpr uint32_t kPairCommon = 3136;

__global__ void __launch_bounds__(kDecThreads, 1)
    decompress_kernel(const __grid_constant__ CUtensorMap omap, const DecompressParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t sbase = ptx::smem_addr(smem);
    const uint32_t bar_full = sbase, bar_empty = sbase + 8 * kDecStages;
    const uint32_t cap_c = p.cap_c, cap_r = p.cap_r;
    const int nlocal = p.pairs > int(blockIdx.x)
                           ? (p.pairs - int(blockIdx.x) + int(gridDim.x) - 1) / int(gridDim.x)
                           : 0;

    if (tid == 0) {
        for (int s = 0; s < kDecStages; ++s) {
            ptx::mbar_init(bar_full + 8 * s, 1);
            ptx::mbar_init(bar_empty + 8 * s, 4);
        }
        ptx::fence_mbar_init();
        ptx::prefetch_tensormap(&omap);
    }
    uint8_t* it_tab = smem + kBarrierBytes;
    uint32_t* ct_tab = reinterpret_cast<uint32_t*>(smem + kBarrierBytes + kIndexTableBytes);
    build_decode_tables(it_tab, ct_tab, tid, blockDim.x);
    __syncthreads();

    if (warp == 0) {
        const uint64_t pol = ptx::policy_evict_first();
        bool ok = true;
        int issued = 0;
        int2 pre_g[3];  // lane j: global offsets of tiles 2p, 2p+1 and the next, pair p = it0 + j
        for (int it = 0; it < nlocal && ok; ++it) {
            const int j = it & 31;
            if (j == 0) {
                // Each lane prefetches the offsets of one of the next 32 pairs.
                const int pi = int(blockIdx.x) + (it + lane) * int(gridDim.x);
                pre_g[0] = pre_g[1] = pre_g[2] = make_int2(0, 0);
                if (pi < p.pairs) {
                    const int t0 = 2 * pi;
                    const int2* g = reinterpret_cast<const int2*>(p.global);
                    pre_g[0] = g[t0];
                    pre_g[1] = g[t0 + 1];
                    pre_g[2] = t0 + 2 <= p.tiles ? g[t0 + 2] : pre_g[1];
                }
            }
            int2 gv[3];
#pragma unroll
            for (int e = 0; e < 3; ++e) {
                gv[e].x = __shfl_sync(kFullMask, pre_g[e].x, j);
                gv[e].y = __shfl_sync(kFullMask, pre_g[e].y, j);
            }
            if (lane == 0) {
                const int s = it % p.nstages;
                if (it >= p.nstages)
                    ok = ptx::mbar_wait(bar_empty + 8 * s, ((it / p.nstages) - 1) & 1);
                if (ok) {
                    const int pi = int(blockIdx.x) + it * int(gridDim.x);
                    const int t0 = 2 * pi;
                    const int ntiles = t0 + 1 < p.tiles ? 2 : 1;
                    const uint32_t slot = sbase + p.off_slots + uint32_t(s) * p.slot_bytes;
                    const uint32_t full = bar_full + 8 * s;
                    uint32_t clen[2] = {0, 0}, rlen[2] = {0, 0}, bytes = 0;
                    for (int tau = 0; tau < ntiles; ++tau) {
                        const int dc = gv[tau + 1].x - gv[tau].x, dr = gv[tau + 1].y - gv[tau].y;
                        if ((gv[tau].x & 15) == 0) clen[tau] = min(uint32_t(max(dc, 0)), cap_c) & ~15u;
                        if ((gv[tau].y & 7) == 0)
                            rlen[tau] = (min(uint32_t(max(dr, 0)), cap_r) * 2u) & ~15u;
                        bytes += 3 * 512 + 32 + clen[tau] + rlen[tau];
                    }
                    ptx::mbar_arrive_expect_tx(full, bytes);
                    for (int tau = 0; tau < ntiles; ++tau) {
                        const size_t t = size_t(t0 + tau);
                        ptx::bulk_g2s(slot + tau * 1536, p.b1 + t * 64, 512, full, pol);
                        ptx::bulk_g2s(slot + tau * 1536 + 512, p.b2 + t * 64, 512, full, pol);
                        ptx::bulk_g2s(slot + tau * 1536 + 1024, p.b3 + t * 64, 512, full, pol);
                        ptx::bulk_g2s(slot + kPairMedium + tau * 32, p.medium + t * 8, 32, full, pol);
                        if (clen[tau])
                            ptx::bulk_g2s(slot + kPairCommon + tau * cap_c, p.sm + gv[tau].x,
                                          clen[tau], full, pol);
                        if (rlen[tau])
                            ptx::bulk_g2s(slot + kPairCommon + 2 * cap_c + tau * 2 * cap_r,
                                          p.rare + gv[tau].y, rlen[tau], full, pol);
                    }
                    ++issued;
                }
            }
            ok = __shfl_sync(kFullMask, ok, 0) != 0;
        }
        if (lane == 0)
            for (int it = max(0, issued - p.nstages); it < issued; ++it)
                ptx::mbar_wait(bar_full + 8 * (it % p.nstages), (it / p.nstages) & 1);
        __syncwarp();
    } else {
        const int dw = warp - 1, g = dw >> 2, q = dw & 3;
        const int tau = q >> 1;
        uint8_t* rb = smem + p.off_rb + uint32_t(dw * 32 + lane) * kRowBufferBytes;
        RowDecoder dec;
        dec.init(ct_tab, reinterpret_cast<const uint4*>(it_tab), rb, lane, 32 * (q & 1) + lane,
                 p.start_exp);
        const uint32_t obuf = sbase + p.off_out + uint32_t(dw) * 2 * kOutTileBytes;
        uint32_t out[32];
        int nstore = 0;
        for (int it = g; it < nlocal; it += kDecGroups) {
            const int s = it % p.nstages;
            const bool ok = ptx::mbar_wait(bar_full + 8 * s, (it / p.nstages) & 1);
            if (!__all_sync(kFullMask, ok)) break;
            const int pi = int(blockIdx.x) + it * int(gridDim.x);
            const int t = 2 * pi + tau;
            const bool valid = t < p.tiles;
            const uint8_t* slot = smem + p.off_slots + uint32_t(s) * p.slot_bytes;
            if (valid)
                dec.decode(reinterpret_cast<const uint32_t*>(slot + tau * 1536),
                           reinterpret_cast<const int*>(slot + kPairMedium + tau * 32),
                           slot + kPairCommon + tau * cap_c,
                           reinterpret_cast<const uint16_t*>(slot + kPairCommon + 2 * cap_c +
                                                             tau * 2 * cap_r),
                           cap_c, cap_r, out);
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(bar_empty + 8 * s);
            if (!valid) continue;
            // Stage this warp's 32x64 block: row `lane`, 16-byte chunk c at
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
                ptx::tma_store_2d(&omap, (t % p.kt) * 64, (t / p.kt) * 64 + 32 * (q & 1), buf);
                ptx::bulk_commit();
            }
            ++nstore;
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
    p.pairs = (p.tiles + 1) / 2;
    p.cap_c = round_up_u(uint32_t(max_common), 16);
    p.cap_r = uint32_t(max_rare);
    p.start_exp = uint32_t(start_exp) & 255u;
    p.off_rb = kBarrierBytes + kIndexTableBytes + kCodeTableBytes;
    p.off_out = round_up_u(p.off_rb + 128 * kDecGroups * kRowBufferBytes, 1024);
    p.off_slots = p.off_out + 4 * kDecGroups * 2 * kOutTileBytes;
    p.slot_bytes = round_up_u(kPairCommon + 2 * p.cap_c + 4 * p.cap_r + 64, 128);
    const uint32_t avail = uint32_t(smem_optin) > p.off_slots ? uint32_t(smem_optin) - p.off_slots : 0;
    p.nstages = std::min<int>(kDecStages, int(avail / p.slot_bytes));
    if (p.nstages < 2) {
        zs_set_error("decompress: packed payload capacity leaves room for fewer than two stages");
        return cudaErrorInvalidConfiguration;
    }
    const uint32_t total = p.off_slots + uint32_t(p.nstages) * p.slot_bytes;
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
    if (!encode_tensor_map_2d(&omap, out, uint64_t(k), uint64_t(m), uint64_t(k) * 2, 64, 32))
        return cudaErrorInvalidValue;
    const int sms = device_sm_count(device);
    const int grid = std::max(1, std::min(p.pairs, sms));
    decompress_kernel<<<grid, kDecThreads, total, stream>>>(omap, p);
    e = cudaGetLastError();
    if (e != cudaSuccess) {
        char msg[200];
        snprintf(msg, sizeof(msg), "decompress launch (grid %d, %d threads, %u B shared, %d stages): %s",
                 grid, kDecThreads, total, p.nstages, cudaGetErrorString(e));
        zs_set_error(msg);
    }
    return e;
}

}  // namespace zs
