// Host-visible parameters and launch helpers of the fused ZipGEMM kernel and
// the standalone decompress kernel.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace zs {

constexpr int kMaxStages = 12;   // compressed/X ring slots
constexpr int kAStages = 4;      // TMEM A buffers (32 columns each)
constexpr int kBarrierBytes = 1024;
constexpr int kOffsetChunk = 64;  // k-tiles of global offsets cached per refill

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
    int nstages;
    uint32_t cap_c, cap_r;  // payload capacity per tile (bytes, words)
    uint32_t start_exp;
    uint32_t off_rb, off_goff, off_x, off_slots, slot_bytes, x_bytes;
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
    int m, k, kt, tiles, pairs;
    int nstages;
    uint32_t cap_c, cap_r;
    uint32_t start_exp;
    uint32_t off_rb, off_out, off_slots, slot_bytes;
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
