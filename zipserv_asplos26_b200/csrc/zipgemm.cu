// Fused TCA-TBE decompress + GEMM ("ZipGEMM") for sm_100a.
//
//   y[n, m] = sum_k W[m, k] * x[n, k],  W decoded on the fly from TCA-TBE.
//
// One CTA computes a 128-row block of W (two vertically adjacent 64x64 global
// tiles) against a tile of up to 256 tokens over a contiguous range of 64-wide
// K slices. The K slices stream through a ring of shared-memory slots, each
// holding `group` consecutive slices: for consecutive tiles of one tile row
// every stream (bitmap planes, band offsets, common and rare payloads) is
// contiguous in global memory, so a slot takes one bulk copy per stream and
// tile row plus one 3-D TMA load of the x tiles - 13 copies per slot instead
// of 12 per slice (a copy costs about 100 cycles to issue, whatever its size).
// Warp roles (1 CTA per SM):
//   warp 0      producer: issues a slot's copies from several lanes, all
//               completing on the slot's mbarrier;
//   warp 1      allocates tensor memory and issues tcgen05.mma (one thread):
//               A = decoded W slice read from TMEM, B = x tile from shared
//               memory (128-byte swizzle), D = FP32 accumulator in TMEM;
//   warps 2..   NDG decoder groups of four warps; group g decodes slots g,
//               g+NDG, ... Warp w serves TMEM lanes 32*(w%4).. and decodes
//               16-row band w%4 of both tiles (row = tile*64 + 16*band + i,
//               TMEM lane = 32*band + 16*tile + i). Each thread rebuilds one W
//               row (64 BF16) per slice and stores it with tcgen05.st into one
//               of the group's TMEM A buffers, so decoded weights never touch
//               shared memory.
// Split-K: the CTAs of a thread-block cluster (1..16) share one row block and
// split its K slices. Each writes its FP32 accumulator tile to its own shared
// memory; after a cluster barrier every CTA reduces a disjoint part of the
// tile by reading all partners' tiles through distributed shared memory in
// rank order (deterministic), converts to BF16 and stores. No global
// workspace and no second kernel (replaces csrc/Reduction_Kernel.cuh:16-41).
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
#include <mutex>

#include "capi_internal.h"
#include "codec.h"
#include "decode.cuh"
#include "ptx.cuh"
#include "zipgemm.cuh"

namespace zs {

constexpr int kGemmThreads4 = 64 + 128 * 4;
constexpr int kGemmThreads2 = 64 + 128 * 2;

// TMEM lane (= decoder thread slot) -> row inside the 128-row block.
__host__ __device__ __forceinline__ int lane_row(int slot) {
    const int band = slot >> 5, l = slot & 31;
    return (l >> 4) * 64 + band * 16 + (l & 15);
}

__device__ __forceinline__ uint32_t bar_addr(uint32_t base, int index) {
    return base + 8u * uint32_t(index);
}

// Cache the (common, rare) offsets of `cnt` consecutive tiles of both tile
// rows, starting at K slice `kt`, in shared memory ([2][kOffsetChunk + 1]).
__device__ __forceinline__ void fetch_offsets(int2* goff, const int* global, int tr0, bool has1,
                                              int kt_total, int kt, int cnt, int lane) {
    for (int e = lane; e < 2 * cnt; e += 32) {
        const int tr = e / cnt, i = e % cnt;
        int2 v = make_int2(0, 0);
        if (tr == 0 || has1)
            v = reinterpret_cast<const int2*>(global)[size_t(tr0 + tr) * kt_total + kt + i];
        goff[tr * (kOffsetChunk + 1) + i] = v;
    }
}

// NDG decoder groups. The ring size is a multiple of NDG so each group owns
// the slots it consumes (slot = stage % ring) and its A buffers, and never
// waits on a barrier more than one phase ahead of what it observed.
template <int NDG>
__global__ void __launch_bounds__(64 + 128 * NDG, 1)
    zipgemm_kernel(const __grid_constant__ CUtensorMap xmap, const GemmParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t sbase = ptx::smem_addr(smem);
    const uint32_t bar_full = sbase;
    const uint32_t bar_empty = sbase + 8 * kMaxStages;
    const uint32_t bar_afull = sbase + 16 * kMaxStages;
    const uint32_t bar_aempty = bar_afull + 8 * kMaxABuffers;
    const uint32_t bar_d = bar_aempty + 8 * kMaxABuffers;
    const uint32_t bar_tab = bar_d + 8;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + (bar_tab - sbase) + 8);
    const uint32_t tables = sbase + kBarrierBytes;

    const int S = p.kparts;
    const int G = p.group;
    const int rank = int(blockIdx.x) % S;  // == %cluster_ctarank: clusters span S consecutive x
    const int mblk = int(blockIdx.x) / S, nblk = int(blockIdx.y);
    const int kt0 = int(int64_t(p.kt) * rank / S), kt1 = int(int64_t(p.kt) * (rank + 1) / S);
    const int nk = kt1 - kt0;
    const int nsup = (nk + G - 1) / G;  // slots this CTA streams
    const int tr0 = 2 * mblk;
    const bool has1 = tr0 + 1 < p.row_tiles;
    const uint32_t cap_c = p.cap_c, cap_r = p.cap_r;
    const uint32_t pstride = 512u * uint32_t(G);
    int2* goff = reinterpret_cast<int2*>(smem + p.off_goff);

    if (tid == 0) {
        for (int s = 0; s < kMaxStages; ++s) {
            ptx::mbar_init(bar_addr(bar_full, s), 1);
            ptx::mbar_init(bar_addr(bar_empty, s), 4 + 1);  // one decoder group + MMA commit
        }
        for (int i = 0; i < kMaxABuffers; ++i) {
            ptx::mbar_init(bar_addr(bar_afull, i), 4);
            ptx::mbar_init(bar_addr(bar_aempty, i), 1);
        }
        ptx::mbar_init(bar_d, 1);
        ptx::mbar_init(bar_tab, 1);
        ptx::fence_mbar_init();
    }
    // The first chunk of tile offsets is fetched right away, so its latency
    // overlaps the rest of the set-up.
    if (warp == 0) fetch_offsets(goff, p.global, tr0, has1, p.kt, kt0, min(kOffsetChunk, nk) + 1, lane);
    if (warp == 1) {
        ptx::tmem_alloc(ptx::smem_addr(tmem_slot), p.tmem_cols);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    if (tid == 0) {
        ptx::prefetch_tensormap(&xmap);
        // Decode lookup tables: one bulk copy from the library's constant table.
        ptx::mbar_arrive_expect_tx(bar_tab, kTableBytes);
        ptx::bulk_g2s(tables, &g_decode_tables, kTableBytes, bar_tab, ptx::policy_evict_last());
    }
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------ producer
        const uint64_t pol_w = ptx::policy_evict_first();
        const uint64_t pol_x = ptx::policy_evict_last();
        const int ntiles = has1 ? 2 : 1;
        bool ok = true;
        int issued = 0;
        for (int is = 0; is < nsup; ++is) {
            const int s = is % p.nstages;
            const int kb = is * G;             // first local K slice of the slot
            const int gn = min(G, nk - kb);    // slices in this slot
            const int ci = kb % kOffsetChunk;  // its index in the offset cache (G divides the chunk)
            if (kb > 0 && ci == 0) {
                fetch_offsets(goff, p.global, tr0, has1, p.kt, kt0 + kb,
                              min(kOffsetChunk, nk - kb) + 1, lane);
                __syncwarp();
            }
            if (is >= p.nstages && lane == 0)
                ok = ptx::mbar_wait(bar_addr(bar_empty, s), ((is / p.nstages) - 1) & 1);
            ok = __shfl_sync(kFullMask, ok, 0) != 0;
            if (!ok) break;
            const uint32_t slot = sbase + p.off_slots + uint32_t(s) * p.slot.bytes;
            const uint32_t full = bar_addr(bar_full, s);
            // Payload runs of the slot's slices. Copies need 16-byte aligned
            // sources; offsets of valid packed data always are.
            uint32_t clen[2] = {0, 0}, rlen[2] = {0, 0};
            int2 g0[2] = {make_int2(0, 0), make_int2(0, 0)};
            for (int tau = 0; tau < ntiles; ++tau) {
                const int2* row = goff + tau * (kOffsetChunk + 1) + ci;
                g0[tau] = row[0];
                const int dc = row[gn].x - g0[tau].x, dr = row[gn].y - g0[tau].y;
                if ((g0[tau].x & 15) == 0)
                    clen[tau] = min(uint32_t(max(dc, 0)), uint32_t(G) * cap_c) & ~15u;
                if ((g0[tau].y & 7) == 0)
                    rlen[tau] = (min(uint32_t(max(dr, 0)), uint32_t(G) * cap_r) * 2u) & ~15u;
            }
            if (lane == 0) {
                // Per-slice payload starts within the slot's regions, clamped
                // so slice g reads inside its region whatever the offsets say.
                int2* hdr = reinterpret_cast<int2*>(smem + p.off_slots + uint32_t(s) * p.slot.bytes +
                                                    p.slot.hdr);
                // A missing second tile row decodes (discarded) zero offsets.
                uint32_t bytes = p.x_bytes;
                for (int tau = 0; tau < 2; ++tau) {
                    const int2* row = goff + tau * (kOffsetChunk + 1) + ci;
                    for (int g = 0; g < gn; ++g) {
                        const int dc = row[g].x - g0[tau].x, dr = row[g].y - g0[tau].y;
                        hdr[tau * kMaxGroup + g] =
                            tau < ntiles ? make_int2(min(max(dc, 0), int(uint32_t(g) * cap_c)),
                                                     min(max(dr, 0), int(uint32_t(g) * cap_r)))
                                         : make_int2(0, 0);
                    }
                    if (tau < ntiles)
                        bytes += 3u * 512u * uint32_t(gn) + 32u * uint32_t(gn) + clen[tau] +
                                 rlen[tau];
                }
                ptx::mbar_arrive_expect_tx(full, bytes);
            }
            __syncwarp();
            // Copies spread over lanes: tile row tau uses lanes 6*tau + {0..5}.
            if (lane < 6 * ntiles) {
                const int tau = lane / 6, c = lane % 6;
                const size_t t = size_t(tr0 + tau) * p.kt + kt0 + kb;
                if (c < 3) {
                    const uint64_t* src = c == 0 ? p.b1 : c == 1 ? p.b2 : p.b3;
                    ptx::bulk_g2s(slot + (tau ? p.slot.plane1 : 0u) + uint32_t(c) * pstride,
                                  src + t * 64, 512u * uint32_t(gn), full, pol_w);
                } else if (c == 3) {
                    ptx::bulk_g2s(slot + p.slot.med + uint32_t(tau) * 32u * G, p.medium + t * 8,
                                  32u * uint32_t(gn), full, pol_w);
                } else if (c == 4) {
                    if (clen[tau])
                        ptx::bulk_g2s(slot + (tau ? p.slot.common1 : p.slot.common0), p.sm + g0[tau].x,
                                      clen[tau], full, pol_w);
                } else if (rlen[tau]) {
                    ptx::bulk_g2s(slot + (tau ? p.slot.rare1 : p.slot.rare0), p.rare + g0[tau].y,
                                  rlen[tau], full, pol_w);
                }
            } else if (lane == 31) {
                // x tiles of the slot's K slices: one 3-D box (64 x bn x G);
                // slices past the end of K arrive zero-filled and are unused.
                ptx::tma_load_3d(sbase + p.off_x + uint32_t(s) * p.x_bytes, &xmap, 0,
                                 nblk * p.bn, kt0 + kb, full, pol_x);
            }
            ++issued;
        }
        // Never leave copies in flight: wait for every issued slot to land.
        if (lane == 0)
            for (int is = max(0, issued - p.nstages); is < issued; ++is)
                ptx::mbar_wait(bar_addr(bar_full, is % p.nstages), (is / p.nstages) & 1);
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc = ptx::idesc_bf16_m128(uint32_t(p.bn));
            bool ok = true;
            for (int is = 0; is < nsup && ok; ++is) {
                const int s = is % p.nstages, grp = is % NDG, use = is / NDG;
                const int gn = min(G, nk - is * G);
                if (!ptx::mbar_wait(bar_addr(bar_full, s), (is / p.nstages) & 1)) break;
                const uint32_t xslot = sbase + p.off_x + uint32_t(s) * p.x_bytes;
                for (int gi = 0; gi < gn; ++gi) {
                    const int a = grp * G + gi;
                    if (!ptx::mbar_wait(bar_addr(bar_afull, a), use & 1)) {
                        ok = false;
                        break;
                    }
                    ptx::tc_fence_after();
                    const uint64_t bdesc =
                        ptx::smem_desc_sw128(xslot + uint32_t(gi * p.bn) * 128u);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        ptx::mma_bf16_ts(tmem, tmem + p.a_col0 + 32u * a + 8u * kk, bdesc + 2u * kk,
                                         idesc, (is | gi | kk) != 0);
                    ptx::mma_commit(bar_addr(bar_aempty, a));
                }
                ptx::mma_commit(bar_addr(bar_empty, s));
            }
            ptx::mma_commit(bar_d);  // fires once every issued MMA has finished
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------ decoders
        const int dw = warp - 2, g = dw >> 2, q = warp & 3;
        const int tau = lane >> 4;
        const bool valid = tau == 0 || has1;
        RowDecoder<8 * 128 * NDG> dec;
        dec.init(tables, sbase + p.off_rb + uint32_t(dw * 32 + lane) * 8u, lane, q, p.start_exp);
        const uint32_t trow = tmem + (uint32_t(32 * q) << 16) + p.a_col0;
        uint32_t out[32];
        bool ok = ptx::mbar_wait(bar_tab, 0);
        for (int is = g; is < nsup; is += NDG) {
            const int s = is % p.nstages, use = is / NDG;
            const int gn = min(G, nk - is * G);
            ok = ok && ptx::mbar_wait(bar_addr(bar_full, s), (is / p.nstages) & 1);
            if (!__all_sync(kFullMask, ok)) break;
            const uint32_t slot = ptx::launder(sbase + p.off_slots + uint32_t(s) * p.slot.bytes);
            const uint32_t plane = slot + (tau ? p.slot.plane1 : 0u);
            const uint32_t med = slot + p.slot.med + uint32_t(tau) * 32u * G;
            const uint32_t com = slot + (tau ? p.slot.common1 : p.slot.common0);
            const uint32_t rar = slot + (tau ? p.slot.rare1 : p.slot.rare0);
            for (int gi = 0; gi < gn; ++gi) {
                const int a = g * G + gi;
                if (use > 0) ok = ptx::mbar_wait(bar_addr(bar_aempty, a), (use - 1) & 1);
                if (!__all_sync(kFullMask, ok)) break;
                const int2 hdr = ptx::lds_s64(slot + p.slot.hdr + uint32_t(tau * kMaxGroup + gi) * 8u);
                dec.decode(plane + 512u * uint32_t(gi), pstride, med + 32u * uint32_t(gi),
                           com + uint32_t(hdr.x), rar + 2u * uint32_t(hdr.y), cap_c, cap_r, out);
                if (!valid) {
#pragma unroll
                    for (int w = 0; w < 32; ++w) out[w] = 0;
                }
                __syncwarp();
                ptx::tmem_st_32x32b_x32(trow + 32u * a, out);
                ptx::tmem_wait_st();
                ptx::tc_fence_before();
                __syncwarp();
                if (lane == 0) ptx::mbar_arrive(bar_addr(bar_afull, a));
            }
            if (!__all_sync(kFullMask, ok)) break;
            if (lane == 0) ptx::mbar_arrive(bar_addr(bar_empty, s));
        }
    }

    // ---------------------------------------------------------- epilogue
    float* red = reinterpret_cast<float*>(smem + p.off_x);  // [bn][128] FP32 when S > 1
    if (warp >= 2) {
        const int dw = warp - 2, g = dw >> 2, q = warp & 3;
        const bool dok = ptx::mbar_wait(bar_d, 0);
        ptx::tc_fence_after();
        const int row = 32 * q + lane;  // TMEM lane = slot in the reduction tile
        const int mrow = mblk * 128 + lane_row(row);
        const bool row_ok = mrow < p.m;
        for (int c = g; c < p.bn / 16; c += NDG) {
            uint32_t v[16];
            ptx::tmem_ld_32x32b_x16(tmem + (uint32_t(32 * q) << 16) + 16u * c, v);
            ptx::tmem_wait_ld();
            if (nk == 0 || !dok) {
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = 0;
            }
            if (S == 1) {
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int n = nblk * p.bn + 16 * c + j;
                    if (n < p.n && row_ok)
                        p.y[size_t(n) * p.m + mrow] =
                            __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(v[j])));
                }
            } else {
#pragma unroll
                for (int j = 0; j < 16; ++j) red[(16 * c + j) * 128 + row] = __uint_as_float(v[j]);
            }
        }
        ptx::tc_fence_before();
    }
    if (S > 1) {
        ptx::cluster_sync();
        const int groups = p.bn * 32;  // float4 = 4 consecutive rows of one token
        const int g0 = int(int64_t(groups) * rank / S), g1 = int(int64_t(groups) * (rank + 1) / S);
        const uint32_t red_addr = ptx::smem_addr(red);
        for (int gi = g0 + tid; gi < g1; gi += blockDim.x) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int src = 0; src < S; ++src) {
                const float4 v = ptx::ld_cluster_f4(ptx::map_to_rank(red_addr + 16u * gi, src));
                acc.x += v.x, acc.y += v.y, acc.z += v.z, acc.w += v.w;
            }
            const int n = nblk * p.bn + (gi >> 5);
            const int mrow = mblk * 128 + lane_row((gi & 31) * 4);  // 4 slots = 4 consecutive rows
            if (n < p.n && mrow < p.m) {
                uint2 packed;
                packed.x = uint32_t(__bfloat16_as_ushort(__float2bfloat16_rn(acc.x))) |
                           (uint32_t(__bfloat16_as_ushort(__float2bfloat16_rn(acc.y))) << 16);
                packed.y = uint32_t(__bfloat16_as_ushort(__float2bfloat16_rn(acc.z))) |
                           (uint32_t(__bfloat16_as_ushort(__float2bfloat16_rn(acc.w))) << 16);
                *reinterpret_cast<uint2*>(p.y + size_t(n) * p.m + mrow) = packed;
            }
        }
        ptx::cluster_sync();  // partners may still read this CTA's tile until here
    }
    __syncthreads();
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, p.tmem_cols);
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

struct DeviceInfo {
    int sms = 0;
    int smem_optin = 0;
    bool gemm_attr = false;
    int active_clusters[17] = {};  // by cluster size, at the GEMM's shared memory budget
};
constexpr int kMaxDevices = 64;
DeviceInfo g_devices[kMaxDevices];
std::mutex g_device_mutex;

DeviceInfo& device_info(int device) {
    DeviceInfo& d = g_devices[device];
    if (!d.sms) {
        std::lock_guard<std::mutex> lock(g_device_mutex);
        if (!d.sms) {
            int smem = 0, sms = 0;
            cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
            d.smem_optin = smem;
            d.sms = sms;
        }
    }
    return d;
}

uint32_t round_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

struct GemmLayout {
    uint32_t off_rb, off_goff, off_x, off_slots, x_bytes, total;
    SlotLayout slot;
    int nstages;
};

// Shared memory: barriers | lookup tables | row buffers | offset cache |
// x ring (1024-aligned, group*bn*128 bytes per slot) | compressed ring | pad.
GemmLayout gemm_layout(int ndg, int group, int bn, uint32_t cap_c, uint32_t cap_r,
                       int smem_limit) {
    GemmLayout l{};
    l.off_rb = kBarrierBytes + kTableBytes;
    l.off_goff = l.off_rb + uint32_t(128 * ndg) * kRowBufferBytes;
    l.off_x = round_up(l.off_goff + 2 * (kOffsetChunk + 1) * 8, 1024);
    l.x_bytes = uint32_t(group * bn) * 128;
    l.slot = slot_layout(group, cap_c, cap_r);
    const uint32_t per_stage = l.x_bytes + l.slot.bytes;
    const uint32_t used = l.off_x + kRingPadBytes;
    const uint32_t avail = uint32_t(smem_limit) > used ? uint32_t(smem_limit) - used : 0;
    l.nstages = std::min<int>(kMaxStages, int(avail / per_stage)) / ndg * ndg;
    l.off_slots = l.off_x + uint32_t(l.nstages) * l.x_bytes;
    l.total = l.off_slots + uint32_t(l.nstages) * l.slot.bytes + kRingPadBytes;
    return l;
}

}  // namespace

int device_sm_count(int device) { return device_info(device).sms; }

SlotLayout slot_layout(int group, uint32_t cap_c, uint32_t cap_r) {
    SlotLayout s{};
    const uint32_t g = uint32_t(group);
    const uint32_t planes = 3u * 512u * g;
    s.plane1 = planes + 64;
    s.med = s.plane1 + planes;
    s.hdr = s.med + 2u * 32u * g;
    s.common0 = round_up(s.hdr + 2u * kMaxGroup * 8u, 128);
    s.common1 = s.common0 + g * cap_c + 64;  // cap_c is a multiple of 128
    s.rare0 = round_up(s.common1 + g * cap_c, 16);
    s.rare1 = s.rare0 + g * cap_r * 2;
    s.bytes = round_up(s.rare1 + g * cap_r * 2, 128);
    return s;
}

static bool encode_map(CUtensorMap* map, const void* base, cuuint32_t rank,
                       const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims,
              strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_tensor_map_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                          uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer) {
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    return encode_map(map, base, 2, dims, strides, box);
}

static int tile_n(int n) { return n > 256 ? 256 : std::max(16, (n + 15) / 16 * 16); }

static int active_clusters(int device, int size, uint32_t smem) {
    DeviceInfo& d = device_info(device);
    if (size <= 0 || size > 16) return 0;
    if (d.active_clusters[size]) return d.active_clusters[size];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(size * 64, 1, 1);
    cfg.blockDim = dim3(kGemmThreads4, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = size;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, zipgemm_kernel<4>, &cfg) != cudaSuccess ||
        clusters <= 0) {
        cudaGetLastError();
        clusters = std::max(1, d.sms / size);
    }
    d.active_clusters[size] = clusters;
    return clusters;
}

static cudaError_t ensure_gemm_attributes(int device) {
    DeviceInfo& d = device_info(device);
    if (d.gemm_attr) return cudaSuccess;
    cudaError_t e = cudaSuccess;
    for (auto fn : {zipgemm_kernel<4>, zipgemm_kernel<2>}) {
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     d.smem_optin);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
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

int plan_kparts(int m, int n, int k, int device) {
    if (!valid_matrix(m, k) || n <= 0) return -1;
    DeviceInfo& d = device_info(device);
    if (ensure_gemm_attributes(device) != cudaSuccess) return 1;
    const int kt = k / 64;
    const int units = ((m / 64 + 1) / 2) * ((n + 255) / 256);
    const int max_s = std::min(kt, 16);
    int best = 1;
    double best_cost = 1e300;
    for (int s = 1; s <= max_s; ++s) {
        const int slots = active_clusters(device, s, uint32_t(d.smem_optin)) * s;
        if (slots <= 0) continue;
        const int ctas = units * s;
        const int waves = (ctas + slots - 1) / slots;
        // Per CTA: its K slices plus a fixed start-up/reduction overhead
        // (about four slices); a partially filled wave still costs a wave.
        const double per_cta = double((kt + s - 1) / s) + 4.0 + (s > 1 ? 1.0 : 0.0);
        const double cost = waves * per_cta * (s > 8 ? 1.03 : 1.0);
        if (cost < best_cost - 1e-9) best_cost = cost, best = s;
    }
    return best;
}

cudaError_t launch_zipgemm(cudaStream_t stream, const void* sm, const void* rare, const void* b1,
                           const void* b2, const void* b3, const void* medium, const void* global,
                           int max_common, int max_rare, int start_exp, const void* x, void* y,
                           int m, int n, int k, int kparts) {
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return e;
    if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
    DeviceInfo& d = device_info(device);
    if ((e = ensure_gemm_attributes(device)) != cudaSuccess) return e;
    const int kt = k / 64;
    if (kparts <= 0) kparts = plan_kparts(m, n, k, device);
    kparts = std::max(1, std::min({kparts, kt, 16}));

    GemmParams p{};
    p.sm = static_cast<const uint8_t*>(sm);
    p.rare = static_cast<const uint16_t*>(rare);
    p.b1 = static_cast<const uint64_t*>(b1);
    p.b2 = static_cast<const uint64_t*>(b2);
    p.b3 = static_cast<const uint64_t*>(b3);
    p.medium = static_cast<const int*>(medium);
    p.global = static_cast<const int*>(global);
    p.y = static_cast<uint16_t*>(y);
    p.m = m, p.n = n, p.k = k, p.kt = kt, p.row_tiles = m / 64;
    p.kparts = kparts;
    p.bn = tile_n(n);
    p.cap_c = common_capacity(max_common);
    p.cap_r = uint32_t(max_rare);
    p.start_exp = uint32_t(start_exp) & 255u;
    // (decoder groups, K slices per slot), most parallel first. Four groups
    // need a ring of at least four slots, two groups of two.
    struct Choice {
        int ndg, group;
    };
    constexpr Choice kChoices[] = {{4, 2}, {2, 4}, {2, 2}, {2, 1}};
    int ndg = 0;
    GemmLayout l{};
    for (const Choice& c : kChoices) {
        l = gemm_layout(c.ndg, c.group, p.bn, p.cap_c, p.cap_r, d.smem_optin);
        if (l.nstages >= c.ndg && c.ndg * c.group <= kMaxABuffers) {
            ndg = c.ndg;
            p.group = c.group;
            break;
        }
    }
    if (!ndg) {
        zs_set_error("zipgemm: packed payload capacity leaves no room for a two-slot ring");
        return cudaErrorInvalidConfiguration;
    }
    // Split-K reduction reuses the rings: they must hold a bn x 128 FP32 tile.
    if (kparts > 1 && uint32_t(p.bn) * 128 * 4 > l.total - kRingPadBytes - l.off_x)
        kparts = p.kparts = 1;
    p.nstages = l.nstages;
    p.off_rb = l.off_rb, p.off_goff = l.off_goff, p.off_x = l.off_x;
    p.off_slots = l.off_slots, p.x_bytes = l.x_bytes, p.slot = l.slot;
    p.a_col0 = uint32_t(std::max(p.bn, 32));
    uint32_t cols = 32;
    while (cols < p.a_col0 + 32u * uint32_t(ndg * p.group)) cols <<= 1;
    p.tmem_cols = cols;

    // x viewed as [K/64][N][64]: one box = `group` consecutive K slices of
    // bn tokens, each slice a 128-byte-swizzled bn x 64 tile.
    CUtensorMap xmap;
    const cuuint64_t dims[3] = {64, uint64_t(n), uint64_t(kt)};
    const cuuint64_t strides[2] = {uint64_t(k) * 2, 128};
    const cuuint32_t box[3] = {64, uint32_t(p.bn), uint32_t(p.group)};
    if (!encode_map(&xmap, x, 3, dims, strides, box)) {
        zs_set_error("zipgemm: activation tensor map rejected (x must be 16-byte aligned)");
        return cudaErrorInvalidValue;
    }

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(((m / 64 + 1) / 2) * kparts), unsigned((n + p.bn - 1) / p.bn), 1);
    cfg.blockDim = dim3(ndg == 4 ? kGemmThreads4 : kGemmThreads2, 1, 1);
    cfg.dynamicSmemBytes = l.total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = unsigned(kparts);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = ndg == 4 ? cudaLaunchKernelEx(&cfg, zipgemm_kernel<4>, xmap, p)
                 : cudaLaunchKernelEx(&cfg, zipgemm_kernel<2>, xmap, p);
    if (e != cudaSuccess) {
        char msg[220];
        snprintf(msg, sizeof(msg),
                 "zipgemm launch (grid %u x %u, cluster %d, %u B shared, %d slots x %d slices, "
                 "bn %d): %s",
                 cfg.gridDim.x, cfg.gridDim.y, kparts, l.total, l.nstages, p.group, p.bn,
                 cudaGetErrorString(e));
        zs_set_error(msg);
    }
    return e;
}

}  // namespace zs
