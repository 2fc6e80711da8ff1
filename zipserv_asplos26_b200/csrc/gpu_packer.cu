// TCA-TBE encoder on the GPU, for weights that are already in device memory
// (no counterpart in the reference, which packs on the host only:
// csrc/HostPacker.h:95-183). Output is byte-identical to the host encoder
// (packer.cpp) and so to the reference's.
//
// Passes (all on the caller's stream):
//   1. exponent histogram of the whole matrix (256 bins);
//   2. the most populated 7-exponent window (one thread; ties to the lowest
//      base, as the host encoder);
//   3. per global tile: common count -> padded (common, rare) counts, and the
//      maxima of both;
//   4. exclusive prefix of the padded counts (one CTA) -> `global`;
//   --- the host reads the window, maxima and totals to size the streams ---
//   5. encode: one 64-thread CTA per global tile, one thread per 8x8 small
//      tile in stream order s = band*16 + group*4 + column*2 + row_tile: its
//      three code bit planes, then a CTA scan of the small tiles' counts
//      gives each thread where its sign|mantissa bytes and rare words go.
// The histogram and maxima live in a caller-provided scratch buffer
// (kPackScratchBytes), so the encoder allocates nothing.
//
// Included by zipserv_cuda.cu.
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cstdint>

#include "capi_internal.h"
#include "codec.h"

namespace zs {
namespace {

constexpr size_t kPackScratchBytes = 4096;
// Scratch layout: [0, 2048) u64 histogram; 2048: int base; 2052: int max
// common; 2056: int max rare.
struct PackScratch {
    unsigned long long hist[256];
    int base, max_common, max_rare, pad;
};

__device__ __forceinline__ uint32_t exponent_of(uint32_t w) { return (w >> 7) & 255u; }

__global__ void __launch_bounds__(256) pack_histogram(const uint4* w, size_t vectors,
                                                      PackScratch* s) {
    __shared__ uint32_t h[256];
    h[threadIdx.x] = 0;
    __syncthreads();
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < vectors;
         i += size_t(gridDim.x) * blockDim.x) {
        const uint4 v = w[i];
        const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            atomicAdd(&h[exponent_of(words[j] & 0xFFFFu)], 1u);
            atomicAdd(&h[exponent_of(words[j] >> 16)], 1u);
        }
    }
    __syncthreads();
    if (h[threadIdx.x]) atomicAdd(&s->hist[threadIdx.x], (unsigned long long)h[threadIdx.x]);
}

// codec.h best_window on the device: the window [b, b+7) with the most
// elements, ties to the lowest b; a caller-fixed base (>= 0) is kept.
__global__ void pack_window(PackScratch* s, int fixed_base) {
    if (threadIdx.x != 0) return;
    s->max_common = 0;
    s->max_rare = 0;
    if (fixed_base >= 0) {
        s->base = fixed_base;
        return;
    }
    unsigned long long sum = 0;
    for (int i = 0; i < 7; ++i) sum += s->hist[i];
    unsigned long long best = sum;
    int base = 0;
    for (int b = 1; b + 7 <= 256; ++b) {
        sum += s->hist[b + 6];
        sum -= s->hist[b - 1];
        if (sum > best) best = sum, base = b;
    }
    s->base = base;
}

// One warp per global tile: lane l counts rows 2l and 2l + 1.
__global__ void __launch_bounds__(256) pack_tile_counts(const uint16_t* w, int m, int k,
                                                         int32_t* g, PackScratch* s) {
    const int kt = k / 64, tiles = (m / 64) * kt;
    const int t = int(blockIdx.x) * 8 + int(threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (t >= tiles) return;
    const uint32_t ubase = uint32_t(s->base);
    const uint16_t* origin = w + (size_t(t / kt) * 64) * size_t(k) + size_t(t % kt) * 64;
    int common = 0;
    for (int i = 0; i < 2; ++i) {
        const uint4* row = reinterpret_cast<const uint4*>(origin + size_t(2 * lane + i) * k);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const uint4 v = row[c];
            const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                common += (exponent_of(words[j] & 0xFFFFu) - ubase) < 7u;
                common += (exponent_of(words[j] >> 16) - ubase) < 7u;
            }
        }
    }
#pragma unroll
    for (int d = 16; d; d >>= 1) common += __shfl_xor_sync(0xFFFFFFFFu, common, d);
    if (lane == 0) {
        const int pc = (common + 15) & ~15, pr = (4096 - common + 7) & ~7;
        g[2 * t + 2] = pc;  // prefixed by pack_scan
        g[2 * t + 3] = pr;
        atomicMax(&s->max_common, pc);
        atomicMax(&s->max_rare, pr);
    }
}

// Exclusive prefix of the padded counts over all tiles, in place: one CTA of
// 1024 threads, each owning a contiguous range of tiles.
__global__ void __launch_bounds__(1024) pack_scan(int32_t* g, int tiles) {
    __shared__ int2 warp_sums[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int begin = int(int64_t(tiles) * tid / 1024), end = int(int64_t(tiles) * (tid + 1) / 1024);
    int2 local = make_int2(0, 0);
    for (int t = begin; t < end; ++t) local.x += g[2 * t + 2], local.y += g[2 * t + 3];
    int2 incl = local;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int ax = __shfl_up_sync(0xFFFFFFFFu, incl.x, d);
        const int ay = __shfl_up_sync(0xFFFFFFFFu, incl.y, d);
        if (lane >= d) incl.x += ax, incl.y += ay;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int2 v = warp_sums[lane];
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int ax = __shfl_up_sync(0xFFFFFFFFu, v.x, d);
            const int ay = __shfl_up_sync(0xFFFFFFFFu, v.y, d);
            if (lane >= d) v.x += ax, v.y += ay;
        }
        warp_sums[lane] = v;  // inclusive over warps
    }
    __syncthreads();
    int2 run = make_int2(incl.x - local.x, incl.y - local.y);
    if (warp > 0) run.x += warp_sums[warp - 1].x, run.y += warp_sums[warp - 1].y;
    if (tid == 0) g[0] = g[1] = 0;
    for (int t = begin; t < end; ++t) {
        run.x += g[2 * t + 2], run.y += g[2 * t + 3];
        g[2 * t + 2] = run.x;
        g[2 * t + 3] = run.y;
    }
}

// One CTA per global tile, thread s = small tile s (the stream order).
__global__ void __launch_bounds__(64) pack_encode(const uint16_t* w, int m, int k,
                                                  const int32_t* g, const PackScratch* s,
                                                  uint8_t* sm, uint16_t* rare, uint64_t* b1,
                                                  uint64_t* b2, uint64_t* b3, int32_t* medium) {
    __shared__ int2 warp_tot[2];
    const int kt = k / 64, t = int(blockIdx.x), tid = threadIdx.x, lane = tid & 31;
    const int band = tid >> 4, group = (tid >> 2) & 3, column = (tid >> 1) & 1, rt = tid & 1;
    const uint32_t ubase = uint32_t(s->base);
    const uint16_t* origin = w + (size_t(t / kt) * 64 + size_t(band * 16 + rt * 8)) * size_t(k) +
                             size_t(t % kt) * 64 + size_t(group * 16 + column * 8);
    uint16_t v[64];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        const uint4 q = *reinterpret_cast<const uint4*>(origin + size_t(r) * k);
        const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            v[r * 8 + 2 * j] = uint16_t(words[j] & 0xFFFFu);
            v[r * 8 + 2 * j + 1] = uint16_t(words[j] >> 16);
        }
    }
    uint64_t m1 = 0, m2 = 0, m3 = 0;
    int nc = 0;
#pragma unroll
    for (int pos = 0; pos < 64; ++pos) {
        const uint32_t idx = exponent_of(v[pos]) - ubase;
        if (idx < 7u) {
            const uint64_t code = idx + 1;
            m1 |= (code & 1) << pos;
            m2 |= ((code >> 1) & 1) << pos;
            m3 |= (code >> 2) << pos;
            ++nc;
        }
    }
    const int nr = 64 - nc;
    // Exclusive scan of (commons, rares) over the 64 small tiles.
    int2 incl = make_int2(nc, nr);
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int ax = __shfl_up_sync(0xFFFFFFFFu, incl.x, d);
        const int ay = __shfl_up_sync(0xFFFFFFFFu, incl.y, d);
        if (lane >= d) incl.x += ax, incl.y += ay;
    }
    if (lane == 31) warp_tot[tid >> 5] = incl;
    __syncthreads();
    int2 ex = make_int2(incl.x - nc, incl.y - nr);
    if (tid >= 32) ex.x += warp_tot[0].x, ex.y += warp_tot[0].y;
    b1[size_t(t) * 64 + tid] = m1;
    b2[size_t(t) * 64 + tid] = m2;
    b3[size_t(t) * 64 + tid] = m3;
    if ((tid & 15) == 0) {
        medium[t * 8 + band * 2] = ex.x;
        medium[t * 8 + band * 2 + 1] = ex.y;
    }
    int ci = g[2 * t] + ex.x, ri = g[2 * t + 1] + ex.y;
#pragma unroll
    for (int pos = 0; pos < 64; ++pos) {
        const uint32_t word = v[pos];
        if (exponent_of(word) - ubase < 7u)
            sm[ci++] = uint8_t((word & 0x7Fu) | ((word >> 8) & 0x80u));
        else
            rare[ri++] = uint16_t(word);
    }
    // Zero padding up to the next tile's start.
    const int total_c = warp_tot[0].x + warp_tot[1].x, total_r = warp_tot[0].y + warp_tot[1].y;
    const int pad_c = g[2 * t + 2] - g[2 * t] - total_c, pad_r = g[2 * t + 3] - g[2 * t + 1] - total_r;
    if (tid < pad_c) sm[g[2 * t] + total_c + tid] = 0;
    if (tid < pad_r) rare[g[2 * t + 1] + total_r + tid] = 0;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace zs

extern "C" uint64_t zipserv_pack_device_scratch_bytes(void) { return zs::kPackScratchBytes; }

extern "C" int zipserv_pack_device_plan(void* stream, const void* weights, int m, int k,
                                        int base, void* global, void* scratch,
                                        int32_t* info) {
    if (!weights || !global || !scratch || !info || !zs::valid_matrix(m, k) ||
        uint64_t(m) * uint64_t(k) > uint64_t(INT_MAX) - 4096 || base < -1 || base > 249 ||
        !zs::aligned16(weights) || !zs::aligned16(global) || !zs::aligned16(scratch)) {
        zs_set_error("zipserv_pack_device_plan: invalid shape, base or pointer (16-byte "
                     "aligned device buffers required)");
        return int(cudaErrorInvalidValue);
    }
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    auto* sc = static_cast<zs::PackScratch*>(scratch);
    auto* g = static_cast<int32_t*>(global);
    const int tiles = (m / 64) * (k / 64);
    cudaError_t e = cudaMemsetAsync(sc, 0, sizeof(zs::PackScratch), s);
    if (e != cudaSuccess) return int(e);
    if (base < 0) {
        const size_t vectors = size_t(m) * size_t(k) / 8;
        const int blocks = int(std::min<size_t>(148 * 8, (vectors + 255) / 256));
        zs::pack_histogram<<<blocks, 256, 0, s>>>(static_cast<const uint4*>(weights), vectors, sc);
    }
    zs::pack_window<<<1, 32, 0, s>>>(sc, base);
    zs::pack_tile_counts<<<(tiles + 7) / 8, 256, 0, s>>>(static_cast<const uint16_t*>(weights),
                                                         m, k, g, sc);
    zs::pack_scan<<<1, 1024, 0, s>>>(g, tiles);
    int32_t host[5] = {};
    // base, max_common, max_rare from the scratch; totals from the prefix.
    if ((e = cudaMemcpyAsync(host, &sc->base, 3 * sizeof(int32_t), cudaMemcpyDeviceToHost, s)) !=
            cudaSuccess ||
        (e = cudaMemcpyAsync(host + 3, g + 2 * size_t(tiles), 2 * sizeof(int32_t),
                             cudaMemcpyDeviceToHost, s)) != cudaSuccess ||
        (e = cudaStreamSynchronize(s)) != cudaSuccess) {
        zs_set_error(cudaGetErrorString(e));
        return int(e);
    }
    info[0] = int32_t(uint8_t(host[0] - 1));  // start_exp = uint8(base - 1)
    info[1] = host[1];                        // max_common
    info[2] = host[2];                        // max_rare
    info[3] = host[3];                        // sm bytes
    info[4] = host[4] * 2;                    // rare bytes
    return 0;
}

extern "C" int zipserv_pack_device_encode(void* stream, const void* weights, int m, int k,
                                          const void* global, const void* scratch, void* sm,
                                          void* rare, void* b1, void* b2, void* b3,
                                          void* medium) {
    if (!weights || !global || !scratch || !b1 || !b2 || !b3 || !medium ||
        !zs::valid_matrix(m, k) || !zs::aligned16(weights) || (uintptr_t(b1) | uintptr_t(b2) |
        uintptr_t(b3)) & 7u || uintptr_t(medium) & 3u || uintptr_t(rare) & 1u) {
        zs_set_error("zipserv_pack_device_encode: invalid shape or pointer");
        return int(cudaErrorInvalidValue);
    }
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int tiles = (m / 64) * (k / 64);
    zs::pack_encode<<<tiles, 64, 0, s>>>(
        static_cast<const uint16_t*>(weights), m, k, static_cast<const int32_t*>(global),
        static_cast<const zs::PackScratch*>(scratch), static_cast<uint8_t*>(sm),
        static_cast<uint16_t*>(rare), static_cast<uint64_t*>(b1), static_cast<uint64_t*>(b2),
        static_cast<uint64_t*>(b3), static_cast<int32_t*>(medium));
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) zs_set_error(cudaGetErrorString(e));
    return int(e);
}
