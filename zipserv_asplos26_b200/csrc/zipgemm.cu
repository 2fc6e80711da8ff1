// Fused TCA-TBE decompress + GEMM ("ZipGEMM") for sm_100a.
//
//   y[n, m] = sum_k W[m, k] * x[n, k],  W decoded on the fly from TCA-TBE.
//
// One CTA computes a 128-row block of W (two vertically adjacent 64x64 global
// tiles) against a tile of up to 256 tokens over a contiguous range of 64-wide
// K slices. Warp roles (1 CTA per SM):
//   warp 0      allocates tensor memory; lane 0 issues tcgen05.mma with
//               both operands in shared memory (A = a decoder group's tile
//               of decoded W, B = an x tile, both 128-byte swizzled) and the
//               FP32 accumulator in TMEM;
//   warps 1..   NDG decoder groups of four warps. Group g decodes K slices
//               g, g+NDG, ... from two compressed slots it owns: while it
//               decodes one, the other is filling. Warp w decodes 16-row
//               band w%4 of both tiles (row = tile*64 + 16*band + i, tile
//               row = 32*band + 16*tile + i); each thread rebuilds one W row
//               (64 BF16) per slice in registers, writes it into the group's
//               A tile with eight 16-byte stores and patches its rare
//               elements with 16-bit stores;
//   next warp   keeps an x ring of nx slices filled with 3-D TMA loads;
//   last two    producers: fill the groups' slots as soon as a group releases
//               one, with few, large copies (an SM's copy engine takes ~100
//               cycles per copy whatever its size): one 4-D tensor load for
//               the three bitmap planes of both tile rows, one 3-D load for
//               the band offsets, one bulk copy per payload run.
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

constexpr int gemm_threads(int ndg) { return 128 + 128 * ndg; }

// TMEM lane (= decoder thread slot) -> row inside the 128-row block.
__host__ __device__ __forceinline__ int lane_row(int slot) {
    const int band = slot >> 5, l = slot & 31;
    return (l >> 4) * 64 + band * 16 + (l & 15);
}

__device__ __forceinline__ uint32_t bar_addr(uint32_t base, int index) {
    return base + 8u * uint32_t(index);
}

// Warp roles: warp 0 allocates TMEM and its lane 0 issues the MMAs; warps
// 1 .. 4*NDG form NDG decoder groups; warp 4*NDG+1 keeps the x ring filled;
// the last two warps fill the decoder groups' compressed slots. Group g decodes K slices
// g, g + NDG, ... and owns two compressed slots: while it decodes slice u
// from one, the other is being filled with its next slice. A group issues
// its own copies after a group barrier (no dedicated producer warp), lane 0
// of each of its four warps taking a share, so copy issue is spread over the
// four SM sub-partitions.
template <int NDG>
__global__ void __launch_bounds__(128 + 128 * NDG, 1)
    zipgemm_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ PlaneMaps pm,
                   const __grid_constant__ CUtensorMap mmap, const GemmParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t sbase = ptx::smem_addr(smem);
    const uint32_t bar_full = sbase;                         // [2 * NDG] slot landed
    const uint32_t bar_free = sbase + 8 * kMaxStages;         // [2 * NDG] slot read by its group
    const uint32_t bar_afull = bar_free + 8 * kMaxStages;     // [NDG] group's A tile written
    const uint32_t bar_aempty = bar_afull + 8 * kMaxATiles;  // [abuf*NDG] A tile read by MMAs
    const uint32_t bar_xfull = bar_aempty + 8 * kMaxATiles;   // [kMaxX]
    const uint32_t bar_xempty = bar_xfull + 8 * kMaxX;
    const uint32_t bar_d = bar_xempty + 8 * kMaxX;
    const uint32_t bar_tab = bar_d + 8;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + (bar_tab - sbase) + 8);
    const uint32_t tables = sbase + kBarrierBytes;

    const int S = p.kparts;
    const int rank = int(blockIdx.x) % S;  // == %cluster_ctarank: clusters span S consecutive x
    const int mblk = int(blockIdx.x) / S, nblk = int(blockIdx.y);
    const int kt0 = int(int64_t(p.kt) * rank / S), kt1 = int(int64_t(p.kt) * (rank + 1) / S);
    const int nk = kt1 - kt0;
    const int tr0 = 2 * mblk;
    const bool has1 = tr0 + 1 < p.row_tiles;
    const uint32_t cap_c = p.cap_c, cap_r = p.cap_r;
    const SlotLayout L = p.slot;

    if (tid == 0) {
        for (int s = 0; s < 2 * NDG; ++s) {
            ptx::mbar_init(bar_addr(bar_full, s), 1);
            ptx::mbar_init(bar_addr(bar_free, s), 4);
        }
        for (int i = 0; i < kMaxX; ++i) {
            ptx::mbar_init(bar_addr(bar_xfull, i), 1);
            ptx::mbar_init(bar_addr(bar_xempty, i), 1);
        }
        for (int i = 0; i < 2 * NDG; ++i) {
            ptx::mbar_init(bar_addr(bar_afull, i), 4);   // the group's four warps
            ptx::mbar_init(bar_addr(bar_aempty, i), 1);  // MMA commit
        }
        ptx::mbar_init(bar_d, 1);
        ptx::mbar_init(bar_tab, 1);
        ptx::fence_mbar_init();
    }
    if (warp == 0) {
        ptx::tmem_alloc(ptx::smem_addr(tmem_slot), p.tmem_cols);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    if (tid == 0) {
        ptx::prefetch_tensormap(&xmap);
        ptx::prefetch_tensormap(&mmap);
        for (int i = 0; i < pm.count; ++i) ptx::prefetch_tensormap(&pm.map[i]);
        // Decode lookup tables: one bulk copy from the library's constant table.
        ptx::mbar_arrive_expect_tx(bar_tab, kTableBytes);
        ptx::bulk_g2s(tables, &g_decode_tables, kTableBytes, bar_tab, ptx::policy_evict_last());
    }
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------ MMA issuer
        // Slice k = NDG*u + g: A = group g's shared-memory tile (use u),
        // B = x slot k % nx. With nx == abuf * NDG the x slot is the A tile's index
        // and one commit frees both. The whole warp runs the loop in uniform
        // control flow (descriptors in uniform registers); one elected lane
        // issues each MMA and commit.
        {
            const uint32_t idesc = ptx::idesc_bf16_m128(uint32_t(p.bn));
            const uint32_t xbase = sbase + p.off_x, xstep = p.x_bytes;
            const uint32_t abase = sbase + p.off_a;
            const int nx = p.nx;
            const int ashift = p.abuf - 1;  // A tiles per group: 1 or 2
            const bool xmerged = nx == p.abuf * NDG;
            int xs = 0;
            uint32_t xph = 0;
            bool ok = true;
            for (int u = 0, k = 0; ok && k < nk; ++u) {
                const uint32_t aph = uint32_t(u >> ashift) & 1u;
                const int aoff = (u & ashift) * NDG;
#pragma unroll
                for (int g = 0; g < NDG; ++g) {
                    if (k >= nk) break;
                    ok = ptx::mbar_wait(bar_addr(bar_xfull, xs), xph) &&
                         ptx::mbar_wait(bar_addr(bar_afull, g + aoff), aph);
                    if (!__all_sync(kFullMask, ok)) {
                        ok = false;
                        break;
                    }
                    ptx::tc_fence_after();
                    const uint64_t bdesc = ptx::smem_desc_sw128(xbase + uint32_t(xs) * xstep);
                    const uint64_t adesc =
                        ptx::smem_desc_sw128(abase + uint32_t(g + aoff) * kATileBytes);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        ptx::mma_bf16_ss_elect(tmem, adesc + 2u * kk, bdesc + 2u * kk, idesc,
                                               (k | kk) != 0);
                    ptx::mma_commit_elect(bar_addr(bar_aempty, g + aoff));
                    if (!xmerged) ptx::mma_commit_elect(bar_addr(bar_xempty, xs));
                    if (++xs == nx) xs = 0, xph ^= 1u;
                    ++k;
                }
            }
            ptx::mma_commit_elect(bar_d);  // fires once every issued MMA has finished
        }
        __syncwarp();
    } else if (warp == 4 * NDG + 1) {
        // ------------------------------------------------------ x loader
        // Slice k's x tile goes to x slot k % nx once the MMAs of slice
        // k - nx have finished reading that slot.
        if (lane == 0) {
            const uint64_t pol_x = ptx::policy_evict_last();
            const int nx = p.nx;
            int issued = 0;
            for (int k = 0; k < nk; ++k) {
                const int xs = k % nx;
                const uint32_t freed = nx == p.abuf * NDG ? bar_aempty : bar_xempty;
                if (k >= nx && !ptx::mbar_wait(bar_addr(freed, xs), ((k / nx) - 1) & 1)) break;
                ptx::mbar_arrive_expect_tx(bar_addr(bar_xfull, xs), p.x_bytes);
                ptx::tma_load_3d(sbase + p.off_x + uint32_t(xs) * p.x_bytes, &xmap, 0,
                                 nblk * p.bn, kt0 + k, bar_addr(bar_xfull, xs), pol_x);
                issued = k + 1;
            }
            // Never leave copies in flight: wait for the last loads to land.
            for (int k = max(0, issued - nx); k < issued; ++k)
                ptx::mbar_wait(bar_addr(bar_xfull, k % nx), (k / nx) & 1);
        }
        __syncwarp();
    } else if (warp >= 4 * NDG + 2) {
        // ------------------------------------------------------ producers
        // Producer pi fills the compressed slots of slices pi, pi + 2, ...
        // (slice k goes to group k % NDG, slot 2 * group + ((k / NDG) & 1))
        // once the group has released the slot's previous contents. Per
        // slot: one 4-D tensor load for the three bitmap planes of both tile
        // rows, one 3-D load for the band offsets and one bulk copy per
        // payload run, all completing on the slot's barrier.
        const int pi = warp - (4 * NDG + 2);
        const int2* goffs = reinterpret_cast<const int2*>(p.global);
        const uint64_t pol_w = ptx::policy_evict_first();
        // Lanes 0-3 hold the (common, rare) offsets of slice k: lane 2*t + e
        // = entry e (0 start, 1 end) of tile row t.
        auto load_offsets = [&](int k) {
            int2 v = make_int2(0, 0);
            if (k < nk && lane < 4 && ((lane >> 1) == 0 || has1))
                v = goffs[size_t(tr0 + (lane >> 1)) * p.kt + kt0 + k + (lane & 1)];
            return v;
        };
        int2 o = load_offsets(pi);
        bool ok = true;
        int last = -1;  // last slice issued
        for (int k = pi; k < nk; k += 2) {
            const int2 onext = load_offsets(k + 2);
            const int g = k % NDG, u = k / NDG, sidx = g * 2 + (u & 1);
            int2 e[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
                e[i].x = __shfl_sync(kFullMask, o.x, i), e[i].y = __shfl_sync(kFullMask, o.y, i);
            if (lane == 0) {
                if (u >= 2) ok = ptx::mbar_wait(bar_addr(bar_free, sidx), ((u >> 1) - 1) & 1);
                if (ok) {
                    uint32_t clen[2], rlen[2];
#pragma unroll
                    for (int t = 0; t < 2; ++t) {
                        const int2 st = e[2 * t], en = e[2 * t + 1];
                        const bool live = t == 0 || has1;
                        // Payload copies need 16-byte aligned sources, which
                        // the offsets of valid packed data always give.
                        clen[t] = live && (st.x & 15) == 0
                                      ? min(uint32_t(max(en.x - st.x, 0)), cap_c) & ~15u
                                      : 0u;
                        rlen[t] = live && (st.y & 7) == 0
                                      ? (min(uint32_t(max(en.y - st.y, 0)), cap_r) * 2u) & ~15u
                                      : 0u;
                    }
                    const uint32_t slot = sbase + p.off_slots + uint32_t(sidx) * L.bytes;
                    const uint32_t full = bar_addr(bar_full, sidx);
                    const int kc = kt0 + k;
                    ptx::mbar_arrive_expect_tx(full, p.plane_box_bytes + 64u + clen[0] + clen[1] +
                                                         rlen[0] + rlen[1]);
                    if (pm.count == 1) {
                        ptx::tma_load_4d(slot, &pm.map[0], 0, kc, tr0, 0, full, pol_w);
                    } else {
#pragma unroll
                        for (int i = 0; i < 3; ++i)
                            ptx::tma_load_3d(slot + uint32_t(i) * L.plane_stride, &pm.map[i], 0,
                                             kc, tr0, full, pol_w);
                    }
                    ptx::tma_load_3d(slot + L.med, &mmap, 0, kc, tr0, full, pol_w);
                    if (clen[0]) ptx::bulk_g2s(slot + L.common0, p.sm + e[0].x, clen[0], full, pol_w);
                    if (clen[1]) ptx::bulk_g2s(slot + L.common1, p.sm + e[2].x, clen[1], full, pol_w);
                    if (rlen[0]) ptx::bulk_g2s(slot + L.rare0, p.rare + e[0].y, rlen[0], full, pol_w);
                    if (rlen[1]) ptx::bulk_g2s(slot + L.rare1, p.rare + e[2].y, rlen[1], full, pol_w);
                    last = k;
                }
            }
            if (!__shfl_sync(kFullMask, ok, 0)) break;
            o = onext;
        }
        // Never leave copies in flight: wait (bounded) for the last use of
        // every slot this producer filled.
        if (lane == 0)
            for (int k = max(pi, last - 2 * NDG + 2); k >= 0 && k <= last; k += 2) {
                const int g = k % NDG, u = k / NDG;
                ptx::mbar_wait(bar_addr(bar_full, g * 2 + (u & 1)), (u >> 1) & 1);
            }
        __syncwarp();
    } else {
        // ------------------------------------------------------ decoders
        const int dw = warp - 1, g = dw >> 2;
        const int q = warp & 3;  // TMEM lane quarter of this warp = band it decodes
        const int tau = lane >> 4;
        const bool valid = tau == 0 || has1;
        RowDecoder dec;
        dec.init(tables, lane, q, p.start_exp);
        // This thread's row of the group's A tile: MMA row m = 32*q + lane
        // (= accumulator lane), 128-byte swizzled.
        const uint32_t m = uint32_t(32 * q + lane);
        const uint32_t arow = sbase + p.off_a + (m >> 3) * 1024u +
                              (m & 7u) * 128u;
        const uint32_t swz = (m & 7u) << 4;
        const int nu = nk > g ? (nk - g + NDG - 1) / NDG : 0;  // slices of this group
        uint32_t out[32];
        RareState rs;
        bool ok = ptx::mbar_wait(bar_tab, 0);
        for (int u = 0; u < nu; ++u) {
            const int sidx = g * 2 + (u & 1);
            const uint32_t slot = ptx::launder(sbase + p.off_slots + uint32_t(sidx) * L.bytes);
            ok = ok && ptx::mbar_wait(bar_addr(bar_full, sidx), (u >> 1) & 1);
            if (!__all_sync(kFullMask, ok)) break;
            dec.decode(slot + uint32_t(tau) * L.plane1, L.plane_stride,
                       slot + L.med + uint32_t(tau) * 32u, slot + (tau ? L.common1 : L.common0),
                       cap_c, cap_r, out, rs);
            if (!valid) {
#pragma unroll
                for (int w = 0; w < 32; ++w) out[w] = 0;
            }
            // The A tile is free once the MMAs of the group's previous slice
            // finished reading it.
            // A tile a = g + NDG * (u % abuf), use u / abuf.
            const int ashift = p.abuf - 1;
            const int a = g + (u & ashift) * NDG, ause = u >> ashift;
            if (ause > 0) ok = ptx::mbar_wait(bar_addr(bar_aempty, a), (ause - 1) & 1);
            if (!__all_sync(kFullMask, ok)) break;
            dec.store(arow + uint32_t(a) * kATileBytes, swz, out, rs, slot + (tau ? L.rare1 : L.rare0), cap_r, !valid);
            // Generic-proxy stores must be visible to the tensor cores.
            ptx::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                ptx::mbar_arrive(bar_addr(bar_free, sidx));  // slot fully read
                ptx::mbar_arrive(bar_addr(bar_afull, a));
            }
        }
    }

    // ---------------------------------------------------------- epilogue
    float* red = reinterpret_cast<float*>(smem + p.off_a);  // [bn][128] FP32 when S > 1
    if (warp >= 1 && warp <= 4 * NDG) {
        const int g = (warp - 1) >> 2, q = warp & 3;
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
    if (warp == 0) {
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
    uint32_t off_a, off_x, off_slots, x_bytes, total;
    SlotLayout slot;
    int nx;
};

// Shared memory: barriers | lookup tables | A tiles (abuf 16 KB 128 x 64
// BF16 tiles per decoder group, 1024-aligned) | x ring (nx slots of bn*128
// bytes) | compressed slots (two per group) | pad. The x ring gets one slot
// per A tile when they fit (then an x slot is freed by the same commit as
// its A tile), else as many as fit.
GemmLayout gemm_layout(int ndg, int abuf, int bn, uint32_t plane_pitch, uint32_t cap_c,
                       uint32_t cap_r, int smem_limit) {
    GemmLayout l{};
    l.off_a = round_up(kBarrierBytes + kTableBytes, 1024);
    l.off_x = l.off_a + uint32_t(ndg * abuf) * kATileBytes;
    l.x_bytes = uint32_t(bn) * 128;
    l.slot = gemm_slot_layout(plane_pitch, cap_c, cap_r);
    const uint32_t slots = uint32_t(2 * ndg) * l.slot.bytes;
    const uint32_t used = l.off_x + slots + kRingPadBytes;
    const uint32_t avail = uint32_t(smem_limit) > used ? uint32_t(smem_limit) - used : 0;
    l.nx = std::min<int>({kMaxX, ndg * abuf, int(avail / l.x_bytes)});
    l.off_slots = l.off_x + uint32_t(l.nx) * l.x_bytes;
    l.total = l.off_slots + slots + kRingPadBytes;
    return l;
}

}  // namespace

int device_sm_count(int device) { return device_info(device).sms; }

SlotLayout gemm_slot_layout(uint32_t plane_pitch, uint32_t cap_c, uint32_t cap_r) {
    // One K slice of two tile rows. A bitmap plane's tile occupies
    // plane_pitch bytes (576: the tensor load's box is 72 words wide, the 8
    // words past the 64-word tile zero-filled, which puts tile row 1 64
    // bytes off modulo 128).
    SlotLayout s{};
    s.plane1 = plane_pitch;
    s.plane_stride = 2u * plane_pitch;
    s.med = round_up(3u * s.plane_stride, 128);  // [2][32 B]
    s.hdr = 0;                                   // unused: one slice per slot
    s.common0 = round_up(s.med + 64u, 128);
    s.common1 = s.common0 + cap_c + 64;  // cap_c is a multiple of 128
    s.rare0 = round_up(s.common1 + cap_c, 16);
    s.rare1 = s.rare0 + cap_r * 2;
    s.bytes = round_up(s.rare1 + cap_r * 2, 128);
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

static int active_clusters(int device, int size, uint32_t smem) {
    DeviceInfo& d = device_info(device);
    if (size <= 0 || size > 16) return 0;
    if (d.active_clusters[size]) return d.active_clusters[size];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(size * 64, 1, 1);
    cfg.blockDim = dim3(gemm_threads(4), 1, 1);
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
    for (auto fn : {zipgemm_kernel<4>, zipgemm_kernel<3>, zipgemm_kernel<2>}) {
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
    p.global = static_cast<const int*>(global);
    p.y = static_cast<uint16_t*>(y);
    p.m = m, p.n = n, p.k = k, p.kt = kt, p.row_tiles = m / 64;
    p.kparts = kparts;
    p.bn = tile_n(n);
    p.cap_c = common_capacity(max_common);
    p.cap_r = uint32_t(max_rare);
    p.start_exp = uint32_t(start_exp) & 255u;
    // Bitmap tensor maps: 72-word boxes (bank offset for tile row 1) when the
    // driver accepts a box wider than the tile, else 64.
    PlaneMaps pm;
    uint32_t pitch = 576;
    if (!encode_plane_maps(&pm, b1, b2, b3, uint64_t(kt), uint64_t(m / 64), 72, 1, 2)) {
        pitch = 512;
        if (!encode_plane_maps(&pm, b1, b2, b3, uint64_t(kt), uint64_t(m / 64), 64, 1, 2)) {
            zs_set_error("zipgemm: bitmap tensor maps rejected (bitmaps must be 16-byte aligned)");
            return cudaErrorInvalidValue;
        }
    }
    p.plane_box_bytes = 3u * 2u * pitch;
    // Band offsets as [row tiles][k tiles][4 u64]: one box = both tile rows.
    CUtensorMap mmap;
    {
        const cuuint64_t dims[3] = {4, uint64_t(kt), uint64_t(m / 64)};
        const cuuint64_t strides[2] = {32, uint64_t(kt) * 32};
        const cuuint32_t box[3] = {4, 1, 2};
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
        int ndg, abuf;
    };
    constexpr Choice kChoices[] = {{4, 1}, {3, 2}, {2, 2}, {2, 1}};
    int ndg = 0;
    GemmLayout l{};
    for (const Choice& c : kChoices) {
        l = gemm_layout(c.ndg, c.abuf, p.bn, pitch, p.cap_c, p.cap_r, d.smem_optin);
        if (l.nx >= 2) {
            ndg = c.ndg;
            p.abuf = c.abuf;
            break;
        }
    }
    if (!ndg) {
        zs_set_error("zipgemm: packed payload capacity leaves no room for the shared-memory rings");
        return cudaErrorInvalidConfiguration;
    }
    // Split-K reduction reuses the A tiles and rings: they must hold a
    // bn x 128 FP32 tile.
    if (kparts > 1 && uint32_t(p.bn) * 128 * 4 > l.total - kRingPadBytes - l.off_a)
        kparts = p.kparts = 1;
    p.nx = l.nx;
    p.off_a = l.off_a, p.off_x = l.off_x;
    p.off_slots = l.off_slots, p.x_bytes = l.x_bytes, p.slot = l.slot;
    // TMEM holds only the FP32 accumulator (bn columns).
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
    cfg.gridDim = dim3(unsigned(((m / 64 + 1) / 2) * kparts), unsigned((n + p.bn - 1) / p.bn), 1);
    cfg.blockDim = dim3(gemm_threads(ndg), 1, 1);
    cfg.dynamicSmemBytes = l.total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = unsigned(kparts);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = ndg == 4   ? cudaLaunchKernelEx(&cfg, zipgemm_kernel<4>, xmap, pm, mmap, p)
        : ndg == 3 ? cudaLaunchKernelEx(&cfg, zipgemm_kernel<3>, xmap, pm, mmap, p)
                   : cudaLaunchKernelEx(&cfg, zipgemm_kernel<2>, xmap, pm, mmap, p);
    if (e != cudaSuccess) {
        char msg[220];
        snprintf(msg, sizeof(msg),
                 "zipgemm launch (grid %u x %u, cluster %d, %u B shared, %d decoder groups, "
                 "%d x slots, bn %d): %s",
                 cfg.gridDim.x, cfg.gridDim.y, kparts, l.total, ndg, l.nx, p.bn,
                 cudaGetErrorString(e));
        zs_set_error(msg);
    }
    return e;
}

}  // namespace zs
