// Host-visible parameters and launch helpers of the fused ZipGEMM kernel and
// the standalone decompress kernel.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace zs {

constexpr int kMaxStages = 8;    // ring slots (each holds `group` K slices)
constexpr int kMaxABuffers = 8;  // TMEM A buffers (32 columns each)
constexpr int kBarrierBytes = 1024;
constexpr int kOffsetChunk = 64;  // k-tiles of global offsets cached per refill
constexpr int kMaxGroup = 8;      // tiles per half of a compressed ring slot

// A compressed ring slot holds two runs ("halves") of up to kMaxGroup tiles
// that are consecutive in the packed streams (the fused GEMM: two tile rows
// of one row block over `group` K slices; decompression: two halves of a
// chunk of consecutive tiles). Byte offsets inside the slot: bitmap planes of
// half 0 at 0 ([3][group][512 B]), of half 1 at plane1 (64 B further mod 128,
// so the two half-warps that decode them read different banks), band offsets
// ([2][group][32 B]), payload starts of each tile relative to its half's run
// ([2][kMaxGroup] int2), then the common and rare payload runs of each half.
struct SlotLayout {
    uint32_t plane1, med, hdr, common0, common1, rare0, rare1, bytes;
};
SlotLayout slot_layout(int group, uint32_t cap_c, uint32_t cap_r);

struct GemmParams {
    const uint8_t* sm;
    const uint16_t* rare;
    const uint64_t* b1;
    const uint64_t* b2;
    const uint64_t* b3;
    const int* medium;
    const int* global;
    uint16_t* y;           // [n, m] BF16
    int m, n, k;
    int kt;                // k / 64
    int row_tiles;         // m / 64
    int kparts;            // CTAs per cluster along K
    int bn;                // N tile (multiple of 16, <= 256)
    int nstages;           // ring slots
    int group;             // K slices per ring slot (1, 2 or 4)
    uint32_t cap_c, cap_r;  // payload capacity per tile (bytes, words)
    uint32_t start_exp;
    uint32_t off_rb, off_goff, off_x, off_slots, x_bytes;
    SlotLayout slot;       // half tau = tile row 2*block + tau
    uint32_t a_col0, tmem_cols;
};

struct DecompressParams {
    const uint8_t* sm;
    const uint16_t* rare;
    const uint64_t* b1;
    const uint64_t* b2;
    const uint64_t* b3;
    const int* medium;
    const int* global;
    int m, k, kt, tiles;
    int nstages;
    int half;              // tiles per half; a slot holds a chunk of 2*half tiles
    int chunks;            // ceil(tiles / (2*half))
    uint32_t cap_c, cap_r;
    uint32_t start_exp;
    uint32_t off_rb, off_out, off_slots;
    SlotLayout slot;
};

// Launch the fused kernel; `kparts` = 0 selects the partition. Arguments are
// assumed validated.
cudaError_t launch_zipgemm(cudaStream_t stream, const void* sm, const void* rare, const void* b1,
                           const void* b2, const void* b3, const void* medium, const void* global,
                           int max_common, int max_rare, int start_exp, const void* x, void* y,
                           int m, int n, int k, int kparts);
int plan_kparts(int m, int n, int k, int device);

cudaError_t launch_decompress(cudaStream_t stream, const void* sm, const void* rare,
                              const void* b1, const void* b2, const void* b3,
                              const void* medium, const void* global, int max_common,
                              int max_rare, int start_exp, void* out, int m, int k);

// Shared by the host launchers.
bool encode_tensor_map_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                          uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer);
int device_sm_count(int device);

}  // namespace zs
