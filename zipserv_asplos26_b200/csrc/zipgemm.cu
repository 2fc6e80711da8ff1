// Fused TCA-TBE decompress + GEMM ("ZipGEMM") for sm_100a.
//
//   y[n, m] = sum_k W[m, k] * x[n, k],  W decoded on the fly from TCA-TBE.
//
// One CTA computes a 128-row block of W (two vertically adjacent 64x64 global
// tiles) against a tile of up to 256 tokens over a contiguous range of 64-wide
// K slices. Warp roles (1 CTA per SM):
//   warp 0      producer: 1-D bulk async copies of each K slice's bitmaps,
//               band offsets and common/rare payloads into a ring of shared
//               memory slots, plus a 2-D TMA load of the x tile (128-byte
//               swizzle), all completing on one mbarrier per slot;
//   warp 1      allocates tensor memory and issues tcgen05.mma (one thread):
//               A = decoded W slice read from TMEM, B = x tile from shared
//               memory, D = FP32 accumulator in TMEM;
//   warps 2..9  two decoder groups of four warps; group g decodes slices
//               g, g+2, ... Each thread rebuilds one W row (64 BF16) and
//               stores it with tcgen05.st into a TMEM A buffer, so decoded
//               weights never touch shared memory.
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
#include <cstring>
#include <mutex>

#include <cstdio>

#include "capi_internal.h"
#include "codec.h"
#include "decode.cuh"
#include "ptx.cuh"
#include "zipgemm.cuh"

namespace zs {

constexpr int kDecoderGroups = 2;
constexpr int kGemmThreads = 64 + 128 * kDecoderGroups;

// Slot layout for one K slice of a 128-row block (two tiles tau = 0, 1):
//   [0, 3072)        bitmap planes b1|b2|b3 (512 B each) of tile 0 then tile 1
//   [3072, 3136)     band offsets (32 B) of tile 0 then tile 1
//   [3136, ...)      common payload of tile 0, tile 1 (cap_c bytes each)
//   [..., ...)       rare payload of tile 0, tile 1 (2*cap_r bytes each)
constexpr uint32_t kSlotMedium = 3072;
constexpr uint32_t kSlotCommon = 3136;

__device__ __forceinline__ uint32_t bar_addr(uint32_t base, int index) {
    return base + 8u * uint32_t(index);
}

template <int NDG>
__global__ void __launch_bounds__(64 + 128 * NDG, 1)
    zipgemm_kernel(const __grid_constant__ CUtensorMap xmap, const GemmParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t sbase = ptx::smem_addr(smem);
    const uint32_t bar_full = sbase;
    const uint32_t bar_empty = sbase + 8 * kMaxStages;
    const uint32_t bar_afull = sbase + 16 * kMaxStages;
    const uint32_t bar_aempty = bar_afull + 8 * kAStages;
    const uint32_t bar_d = bar_aempty + 8 * kAStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + (bar_d - sbase) + 8);

    const int S = p.kparts;
    const int rank = int(blockIdx.x) % S;  // == %cluster_ctarank: clusters span S consecutive x
    const int mblk = int(blockIdx.x) / S, nblk = int(blockIdx.y);
    const int kt0 = int(int64_t(p.kt) * rank / S), kt1 = int(int64_t(p.kt) * (rank + 1) / S);
    const int nk = kt1 - kt0;
    const int tr0 = 2 * mblk;
    const bool has1 = tr0 + 1 < p.row_tiles;
    const uint32_t cap_c = p.cap_c, cap_r = p.cap_r;

    if (tid == 0) {
        for (int s = 0; s < kMaxStages; ++s) {
            ptx::mbar_init(bar_addr(bar_full, s), 1);
            ptx::mbar_init(bar_addr(bar_empty, s), 4 + 1);  // one decoder group + MMA commit
        }
        for (int i = 0; i < kAStages; ++i) {
            ptx::mbar_init(bar_addr(bar_afull, i), 4);
            ptx::mbar_init(bar_addr(bar_aempty, i), 1);
        }
        ptx::mbar_init(bar_d, 1);
        ptx::fence_mbar_init();
    }
    if (warp == 1) {
        ptx::tmem_alloc(ptx::smem_addr(tmem_slot), p.tmem_cols);
        ptx::tmem_relinquish();
    }
    if (tid == 0) ptx::prefetch_tensormap(&xmap);
    uint8_t* it_tab = smem + kBarrierBytes;
    uint32_t* ct_tab = reinterpret_cast<uint32_t*>(smem + kBarrierBytes + kIndexTableBytes);
    build_decode_tables(it_tab, ct_tab, tid, blockDim.x);
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------ producer
        int2* goff = reinterpret_cast<int2*>(smem + p.off_goff);  // [2][kOffsetChunk + 1]
        const uint64_t pol_w = ptx::policy_evict_first();
        const uint64_t pol_x = ptx::policy_evict_last();
        bool ok = true;
        int issued = 0;
        for (int it = 0; it < nk && ok; ++it) {
            const int s = it % p.nstages;
            const int ci = it % kOffsetChunk;
            if (ci == 0) {
                // Cache the (common, rare) offsets of this chunk's tiles and
                // the following sentinel for both tile rows.
                const int cnt = min(kOffsetChunk, nk - it) + 1;
                for (int e = lane; e < 2 * cnt; e += 32) {
                    const int tr = e / cnt, i = e % cnt;
                    int2 v = make_int2(0, 0);
                    if (tr == 0 || has1)
                        v = reinterpret_cast<const int2*>(p.global)[(tr0 + tr) * p.kt + kt0 + it + i];
                    goff[tr * (kOffsetChunk + 1) + i] = v;
                }
                __syncwarp();
            }
            if (lane == 0) {
                if (it >= p.nstages)
                    ok = ptx::mbar_wait(bar_addr(bar_empty, s), ((it / p.nstages) - 1) & 1);
                if (ok) {
                    const int kt = kt0 + it;
                    const uint32_t slot = sbase + p.off_slots + uint32_t(s) * p.slot_bytes;
                    const uint32_t full = bar_addr(bar_full, s);
                    uint32_t clen[2] = {0, 0}, rlen[2] = {0, 0};
                    int2 g0[2];
                    uint32_t bytes = p.x_bytes;
                    const int ntiles = has1 ? 2 : 1;
                    for (int tau = 0; tau < ntiles; ++tau) {
                        g0[tau] = goff[tau * (kOffsetChunk + 1) + ci];
                        const int2 g1 = goff[tau * (kOffsetChunk + 1) + ci + 1];
                        const int dc = g1.x - g0[tau].x, dr = g1.y - g0[tau].y;
                        // Payload copies need 16-byte aligned sources; offsets
                        // of valid packed data always are.
                        if ((g0[tau].x & 15) == 0)
                            clen[tau] = min(uint32_t(max(dc, 0)), cap_c) & ~15u;
                        if ((g0[tau].y & 7) == 0)
                            rlen[tau] = (min(uint32_t(max(dr, 0)), cap_r) * 2u) & ~15u;
                        bytes += 3 * 512 + 32 + clen[tau] + rlen[tau];
                    }
                    ptx::mbar_arrive_expect_tx(full, bytes);
                    for (int tau = 0; tau < ntiles; ++tau) {
                        const size_t t = size_t(tr0 + tau) * p.kt + kt;
                        ptx::bulk_g2s(slot + tau * 1536, p.b1 + t * 64, 512, full, pol_w);
                        ptx::bulk_g2s(slot + tau * 1536 + 512, p.b2 + t * 64, 512, full, pol_w);
                        ptx::bulk_g2s(slot + tau * 1536 + 1024, p.b3 + t * 64, 512, full, pol_w);
                        ptx::bulk_g2s(slot + kSlotMedium + tau * 32, p.medium + t * 8, 32, full,
                                      pol_w);
                        if (clen[tau])
                            ptx::bulk_g2s(slot + kSlotCommon + tau * cap_c, p.sm + g0[tau].x,
                                          clen[tau], full, pol_w);
                        if (rlen[tau])
                            ptx::bulk_g2s(slot + kSlotCommon + 2 * cap_c + tau * 2 * cap_r,
                                          p.rare + g0[tau].y, rlen[tau], full, pol_w);
                    }
                    ptx::tma_load_2d(sbase + p.off_x + uint32_t(s) * p.x_bytes, &xmap, kt * 64,
                                     nblk * p.bn, full, pol_x);
                    ++issued;
                }
            }
            ok = __shfl_sync(kFullMask, ok, 0) != 0;
            __syncwarp();
        }
        // Never leave copies in flight: wait for every issued slot to land.
        if (lane == 0)
            for (int it = max(0, issued - p.nstages); it < issued; ++it)
                ptx::mbar_wait(bar_addr(bar_full, it % p.nstages), (it / p.nstages) & 1);
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc = ptx::idesc_bf16_m128(uint32_t(p.bn));
            for (int it = 0; it < nk; ++it) {
                const int s = it % p.nstages, i = it % kAStages;
                if (!ptx::mbar_wait(bar_addr(bar_afull, i), (it / kAStages) & 1)) break;
                if (!ptx::mbar_wait(bar_addr(bar_full, s), (it / p.nstages) & 1)) break;
                ptx::tc_fence_after();
                const uint64_t bdesc = ptx::smem_desc_sw128(sbase + p.off_x + uint32_t(s) * p.x_bytes);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    ptx::mma_bf16_ts(tmem, tmem + p.a_col0 + 32u * i + 8u * kk, bdesc + 2u * kk,
                                     idesc, (it | kk) != 0);
                ptx::mma_commit(bar_addr(bar_aempty, i));
                ptx::mma_commit(bar_addr(bar_empty, s));
            }
            ptx::mma_commit(bar_d);  // fires once every issued MMA has finished
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------ decoders
        const int dw = warp - 2, g = dw >> 2, q = warp & 3;
        const int tau = q >> 1;
        const bool valid = tau == 0 || has1;
        uint8_t* rb = smem + p.off_rb + uint32_t(dw * 32 + lane) * kRowBufferBytes;
        RowDecoder dec;
        dec.init(ct_tab, reinterpret_cast<const uint4*>(it_tab), rb, lane, 32 * (q & 1) + lane,
                 p.start_exp);
        const uint32_t trow = tmem + (uint32_t(32 * q) << 16) + p.a_col0;
        uint32_t out[32];
        for (int it = g; it < nk; it += NDG) {
            const int s = it % p.nstages, i = it % kAStages;
            bool ok = ptx::mbar_wait(bar_addr(bar_full, s), (it / p.nstages) & 1);
            if (ok && it >= kAStages)
                ok = ptx::mbar_wait(bar_addr(bar_aempty, i), ((it / kAStages) - 1) & 1);
            if (!__all_sync(kFullMask, ok)) break;
            const uint8_t* slot = smem + p.off_slots + uint32_t(s) * p.slot_bytes;
            if (valid) {
                dec.decode(reinterpret_cast<const uint32_t*>(slot + tau * 1536),
                           reinterpret_cast<const int*>(slot + kSlotMedium + tau * 32),
                           slot + kSlotCommon + tau * cap_c,
                           reinterpret_cast<const uint16_t*>(slot + kSlotCommon + 2 * cap_c +
                                                             tau * 2 * cap_r),
                           cap_c, cap_r, out);
            } else {
#pragma unroll
                for (int w = 0; w < 32; ++w) out[w] = 0;
            }
            __syncwarp();
            ptx::tmem_st_32x32b_x32(trow + 32u * i, out);
            ptx::tmem_wait_st();
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                ptx::mbar_arrive(bar_addr(bar_afull, i));
                ptx::mbar_arrive(bar_addr(bar_empty, s));
            }
        }
    }

    // ---------------------------------------------------------- epilogue
    float* red = reinterpret_cast<float*>(smem + p.off_x);  // [bn][128] FP32 when S > 1
    if (warp >= 2) {
        const int dw = warp - 2, g = dw >> 2, q = warp & 3;
        const bool dok = ptx::mbar_wait(bar_d, 0);
        ptx::tc_fence_after();
        const int row = 32 * q + lane;
        const int mrow = mblk * 128 + row;
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
            const int mrow = mblk * 128 + (gi & 31) * 4;
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
    uint32_t off_rb, off_goff, off_x, off_slots, slot_bytes, x_bytes, total;
    int nstages;
};

GemmLayout gemm_layout(int bn, uint32_t cap_c, uint32_t cap_r, int smem_limit) {
    GemmLayout l{};
    l.off_rb = kBarrierBytes + kIndexTableBytes + kCodeTableBytes;
    l.off_goff = l.off_rb + uint32_t(128 * kDecoderGroups) * kRowBufferBytes;
    l.off_x = round_up(l.off_goff + 2 * (kOffsetChunk + 1) * 8, 1024);
    l.x_bytes = uint32_t(bn) * 128;
    l.slot_bytes = round_up(kSlotCommon + 2 * cap_c + 4 * cap_r + 64, 128);
    const uint32_t per_stage = l.x_bytes + l.slot_bytes;
    const uint32_t avail = uint32_t(smem_limit) > l.off_x ? uint32_t(smem_limit) - l.off_x : 0;
    l.nstages = std::min<int>(kMaxStages, int(avail / per_stage));
    // Split-K reduction reuses the ring: it must hold a bn x 128 FP32 tile.
    l.off_slots = l.off_x + uint32_t(l.nstages) * l.x_bytes;
    l.total = l.off_slots + uint32_t(l.nstages) * l.slot_bytes;
    return l;
}

}  // namespace

int device_sm_count(int device) { return device_info(device).sms; }

bool encode_tensor_map_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                          uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
              box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int tile_n(int n) { return n > 256 ? 256 : std::max(16, (n + 15) / 16 * 16); }

static int active_clusters(int device, int size, uint32_t smem) {
    DeviceInfo& d = device_info(device);
    if (size <= 0 || size > 16) return 0;
    if (d.active_clusters[size]) return d.active_clusters[size];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(size * 64, 1, 1);
    cfg.blockDim = dim3(kGemmThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = size;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, zipgemm_kernel<kDecoderGroups>, &cfg) !=
            cudaSuccess ||
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
    cudaError_t e = cudaFuncSetAttribute(zipgemm_kernel<kDecoderGroups>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         d.smem_optin);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(zipgemm_kernel<kDecoderGroups>,
                                 cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
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
    p.cap_c = round_up(uint32_t(max_common), 16);
    p.cap_r = uint32_t(max_rare);
    p.start_exp = uint32_t(start_exp) & 255u;
    const GemmLayout l = gemm_layout(p.bn, p.cap_c, p.cap_r, d.smem_optin);
    if (l.nstages < 2) {
        zs_set_error("zipgemm: packed payload capacity leaves room for fewer than two stages");
        return cudaErrorInvalidConfiguration;
    }
    if (kparts > 1 && uint32_t(p.bn) * 128 * 4 > l.total - l.off_x) kparts = p.kparts = 1;
    p.nstages = l.nstages;
    p.off_rb = l.off_rb, p.off_goff = l.off_goff, p.off_x = l.off_x;
    p.off_slots = l.off_slots, p.slot_bytes = l.slot_bytes, p.x_bytes = l.x_bytes;
    p.a_col0 = uint32_t(std::max(p.bn, 32));
    uint32_t cols = 32;
    while (cols < p.a_col0 + 32u * kAStages) cols <<= 1;
    p.tmem_cols = cols;

    CUtensorMap xmap;
    if (!encode_tensor_map_2d(&xmap, x, uint64_t(k), uint64_t(n), uint64_t(k) * 2, 64,
                              uint32_t(p.bn))) {
        zs_set_error("zipgemm: activation tensor map rejected (x must be 16-byte aligned)");
        return cudaErrorInvalidValue;
    }

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(((m / 64 + 1) / 2) * kparts), unsigned((n + p.bn - 1) / p.bn), 1);
    cfg.blockDim = dim3(kGemmThreads, 1, 1);
    cfg.dynamicSmemBytes = l.total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = unsigned(kparts);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, zipgemm_kernel<kDecoderGroups>, xmap, p);
    if (e != cudaSuccess) {
        char msg[220];
        snprintf(msg, sizeof(msg),
                 "zipgemm launch (grid %u x %u, cluster %d, %u B shared, %d stages, bn %d): %s",
                 cfg.gridDim.x, cfg.gridDim.y, kparts, l.total, l.nstages, p.bn,
                 cudaGetErrorString(e));
        zs_set_error(msg);
    }
    return e;
}

}  // namespace zs
