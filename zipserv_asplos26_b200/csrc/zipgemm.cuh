// Host-visible parameters and launch helpers of the fused ZipGEMM kernel and
// the standalone decompress kernel.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace zs {

constexpr int kMaxStages = 8;    // compressed ring slots
constexpr int kMaxX = 8;         // x ring slots (one K slice each)
constexpr int kMaxATiles = 8;    // decoded A tiles (decoder groups x tiles per group)
constexpr int kBarrierBytes = 1024;
constexpr int kChunk = 32;       // K slices per refill of the offset / band-offset caches
constexpr int kMaxGroup = 8;     // tiles per half of a compressed ring slot
// Decoded A tile: 128 rows x 64 BF16 in the tensor cores' K-major layout
// without swizzle, built from "core matrices" of 8 rows x 8 BF16 (8 rows of
// 16 bytes, 128 contiguous bytes, exactly one 8x8 small tile of the format).
// The 16 core matrices of one K chunk (8 columns) are contiguous along M
// (kAGroup = 128 bytes apart); the 8 K chunks are kACoreK = 2064 bytes
// apart (2048 + 16), which puts the 8 core matrices of one 8-row group on
// distinct banks.
constexpr uint32_t kAGroup = 128;
constexpr uint32_t kACoreK = 16 * kAGroup + 16;
constexpr uint32_t kATileBytes = 7 * kACoreK + 16 * kAGroup + 16;  // 16512, a multiple of 128
constexpr int kMaxTp = 8;        // ranks of a fused all-reduce

// A compressed ring slot holds two runs ("halves") of up to kMaxGroup tiles
// that are consecutive in the packed streams (the fused GEMM: two tile rows
// of one row block over `group` K slices; decompression: two halves of a
// chunk of consecutive tiles). Byte offsets inside the slot: bitmap planes
// (plane b of half tau at b*plane_stride + tau*plane1; the GEMM places half
// 1 64 bytes off modulo 128, decompression's tensor loads pack the halves),
// band offsets (decompression only:
// [2*group][32 B]), payload starts of each tile relative to its run
// ([2][kMaxGroup] int2), then the common payload runs of the two halves
// (the second 64 bytes further modulo 128, so the half-warps that decode the
// two halves read different banks) and the rare payload run(s).
struct SlotLayout {
    uint32_t plane_stride, plane1, med, hdr, common0, common1, rare0, rare1, bytes;
};
SlotLayout gemm_slot_layout(uint32_t plane_pitch, uint32_t cap_c, uint32_t cap_r, int S);
SlotLayout decompress_slot_layout(int half, uint32_t cap_c, uint32_t cap_r);

// Multipliers and the exponent palette of the small-tile decoder, kept in
// the kernel's parameter (constant) bank: the decoder's multiply-adds take
// them as constant-bank operands, so they run on the FMA pipe (a literal
// would be strength-reduced to shifts on the integer ALU) without holding
// registers.
struct DecodeConsts {
    uint32_t k2, k4, k8, kent, krank, khi;
    uint32_t xp_lo, xp_hi;  // exponent palette (see RowDecoder)
};

struct GemmParams {
    const uint8_t* sm;
    const uint16_t* rare;
    const int* global;
    uint16_t* y;           // [n, m] BF16
    float* ws_partials;    // [grid][2][pieces][32 lanes][16] FP32 partial tiles
    uint32_t* ws_counters;  // [grid][4 lane quarters] arrivals (zero between launches)
    int m, n, k;
    int kt;                // k / 64
    int row_tiles;         // m / 64
    int row_blocks;        // 128-row blocks: ceil(row_tiles / 2)
    int units;             // row_blocks * n blocks
    int steps;             // units * kt: the (unit, K slice) work items
    int S;                 // K slices per compressed slot (2 when kt is even, else 1)
    int groups;            // steps / S: the items are dealt out S at a time
    int nslots;            // compressed slots in the ring (2 * decoder groups / S)
    int grid;              // CTAs; CTA c owns items [S*(c*groups/grid), S*((c+1)*groups/grid))
    int pieces;            // 32-row x 16-column pieces of a unit's tile: 4 * bn / 16
    int resident;          // 1: every CTA runs at once (grid <= SMs), so the first
                           // part's CTA may wait for a unit's other parts
    int bn;                // N tile (multiple of 16, <= 256)
    int nx;                // x ring slots
    int na;                // decoded A tiles (>= decoder groups, <= kMaxATiles); step t
                           // writes tile t % na
    uint32_t cap_c, cap_r;  // payload capacity per tile (bytes, words)
    uint32_t start_exp;
    DecodeConsts dk;
    uint32_t plane_box_bytes;  // bytes one bitmap tensor load (or three) writes
    uint32_t off_a, off_x, off_slots;
    uint32_t x_bytes;      // one x slot: bn tokens x one K slice (bn * 128 bytes)
    SlotLayout slot;       // S K slices of the block's two tile rows
    uint32_t tmem_cols;    // columns of one accumulator (two are allocated)
    uint64_t reducer_wait_ns;  // how long a row block's first part waits for the others
    // Fused all-reduce of the output over tp_world ranks (row-parallel
    // layers; tp_world <= 1: off). tp_recv[r] is rank r's receive buffer as
    // this GPU addresses it (peer memory); tp_state is this rank's [epoch,
    // finished CTAs] pair.
    int tp_world, tp_rank;
    uint64_t* tp_recv[kMaxTp];
    uint32_t* tp_state;
};

struct DecompressParams {
    const uint8_t* sm;
    const uint16_t* rare;
    const int* medium;
    const int* global;
    int m, k, kt, tiles;
    int nstages;
    int half;              // tiles per half; a slot holds a chunk of 2*half tiles
    int chunks;            // ceil(tiles / (2*half))
    int plane_maps;
    uint32_t cap_c, cap_r;
    uint32_t start_exp;
    uint32_t off_out, off_slots;
    SlotLayout slot;
};

// Bitmap plane tensor maps: when b2 - b1 == b3 - b2 (one allocation, the
// layout the runtime uses) map 0 spans all three planes and one load brings
// a slot's bitmaps; otherwise one map per plane.
struct PlaneMaps {
    CUtensorMap map[3];
    int count;
};

// Caller-owned K-range fixup scratch: FP32 partial tiles (any contents) and
// arrival counters (zero-filled before their first use; every launch returns
// the counters it used to zero).
struct GemmScratch {
    void* partials;
    size_t partial_bytes;
    void* counters;
    size_t counter_bytes;
};

// Launch the fused kernel. `kparts` = 0: one CTA per SM (or fewer for small
// problems); kparts > 0: kparts CTAs per 128-row block. `scratch` null: the
// library's own per-stream scratch. Arguments are assumed validated.
struct TpExchange;
cudaError_t launch_zipgemm(cudaStream_t stream, const void* sm, const void* rare, const void* b1,
                           const void* b2, const void* b3, const void* medium, const void* global,
                           int max_common, int max_rare, int start_exp, const void* x, void* y,
                           int m, int n, int k, int kparts, const GemmScratch* scratch = nullptr,
                           const TpExchange* tp = nullptr);
int plan_kparts(int m, int n, int k, int device);
// Fused all-reduce exchange of one launch: the peers' receive buffers and
// flag areas (index = rank; the flag areas are reserved, values carry their
// own epoch) and this rank's state pair; sizes checked by the caller.
struct TpExchange {
    int world, rank;
    void* const* recv;
    void* const* flags;
    void* state;
};
// Receive buffer and flag bytes a fused all-reduce of an [n, m] output needs.
void allreduce_exchange_bytes(int m, int n, int world, size_t* recv_bytes, size_t* flag_bytes);
// How long (ns) the CTA holding a split row block's first K part waits for
// the other parts before falling back to the last-arrival reduction (both
// give identical results). Returns the previous value.
uint64_t set_reducer_wait_ns(uint64_t ns);
// Scratch the launch needs (both 0 when no CTA range splits a row block).
void gemm_workspace_bytes(int m, int n, int k, int kparts, int device, size_t* partial_bytes,
                          size_t* counter_bytes);

cudaError_t launch_decompress(cudaStream_t stream, const void* sm, const void* rare,
                              const void* b1, const void* b2, const void* b3,
                              const void* medium, const void* global, int max_common,
                              int max_rare, int start_exp, void* out, int m, int k);

// Shared by the host launchers.
bool encode_tensor_map_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                          uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer);
// Plane maps over tiles viewed as [outer][inner tiles] (the GEMM: [row
// tiles][k tiles], box `box_inner` x `box_outer` tiles; decompression: one
// row of all tiles).
bool encode_plane_maps(PlaneMaps* maps, const void* b1, const void* b2, const void* b3,
                       uint64_t inner, uint64_t outer, uint32_t box_words, uint32_t box_inner,
                       uint32_t box_outer);
int device_sm_count(int device);

}  // namespace zs
