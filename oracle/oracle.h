/*
 * TEST INFRASTRUCTURE ONLY. This is the CPU oracle for the ZipServ TCA-TBE
 * (triple-bitmap BF16) hot path: a plain-C restatement of the reference's
 * encoder, decoder and FP32-accumulated GEMM. Only tests/, the smoke check in
 * __graft_entry__.py and bench.py's cpu_baseline / reference arm may load it,
 * and then only as the checker. The product library never links or calls it.
 *
 * Parity is pinned: tests/test_oracle_golden.py checks every function here
 * against digests produced by the reference's own encoder compiled from its
 * sources (oracle/_ref, see oracle/Makefile) and against the reference's
 * known-answer cases (all 65 536 BF16 words, every exponent window, padding
 * boundaries, constant matrices, 448 000 exponent reconstructions).
 */
#ifndef ZIPSERV_ORACLE_H
#define ZIPSERV_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Encoder output. Buffer order and byte lengths follow the reference's
 * HostPacked::lengths (csrc/HostPacker.h:83-88): sm, rare, b1, b2, b3,
 * small, medium, global. `small` is NULL unless requested. */
typedef struct oracle_packed {
    uint8_t* sm;
    uint16_t* rare;
    uint64_t* b1;
    uint64_t* b2;
    uint64_t* b3;
    int32_t* small;
    int32_t* medium;
    int32_t* global;
    int32_t tiles, base, max_common, max_rare;
    uint64_t lengths[8];
} oracle_packed;

/* csrc/CodecUtils.h:11-14 */
int oracle_valid_matrix(int m, int k);
/* csrc/CodecUtils.h:16-24 */
int oracle_valid_gemm(int m, int n, int k, int split_k);
/* csrc/CodecUtils.h:26-29 */
int oracle_valid_counts(int common, int rare);
/* csrc/CodecUtils.h:40-53: argmax of the `width`-wide window sum, ties to the
 * lowest base. Returns -1 for an invalid width (the reference throws). */
int oracle_best_window(const uint64_t counts[256], int width);
/* csrc/CodecUtils.h:55-62 */
uint16_t oracle_exponent_bits(uint8_t start_exp, uint8_t code);

/* csrc/HostPacker.h:95-183 (single thread). base = -1 selects the window from
 * the exponent histogram. Returns 0, or -1 for invalid arguments. */
int oracle_pack(const uint16_t* words, int m, int k, int base, int include_small,
                oracle_packed* out);
void oracle_free(oracle_packed* packed);

/* tests/test_host_packer.cpp:14-44 and tests/test_host_runtime.py:138-177:
 * invert each small-tile index independently of the encoder's traversal and
 * check the medium and global offsets on the way. Inputs are the seven device
 * buffers in ABI order plus start_exp = uint8(base - 1). Returns 0, or a
 * positive code naming the first inconsistency (1 medium, 2 global padding,
 * 3 overrun). */
int oracle_decode(const uint8_t* sm, const uint16_t* rare, const uint64_t* b1,
                  const uint64_t* b2, const uint64_t* b3, const int32_t* medium,
                  const int32_t* global, int m, int k, int start_exp, uint16_t* out);

/* oracle_decode split over `threads` host threads by tile ranges (each tile
 * is independent given the global offsets); same result. */
int oracle_decode_mt(const uint8_t* sm, const uint16_t* rare, const uint64_t* b1,
                     const uint64_t* b2, const uint64_t* b3, const int32_t* medium,
                     const int32_t* global, int m, int k, int start_exp, uint16_t* out,
                     int threads);

/* Round-to-nearest-even FP32 -> BF16, as __float2bfloat16_rn. */
uint16_t oracle_f32_to_bf16(float value);
float oracle_bf16_to_f32(uint16_t bits);

/* tests/test_cuda.cu:125-131: y[n*m + row] = bf16(sum_j w[row,j] * x[n,j]),
 * summed in FP32 in ascending j. w is [m,k] row-major, x is [n,k] row-major.
 * y_f32 (optional) receives the unrounded sums. `threads` <= 1 runs serially;
 * the summation order per output is the same either way. */
void oracle_gemm(const uint16_t* w, const uint16_t* x, int m, int n, int k,
                 uint16_t* y, float* y_f32, int threads);

/* tests/test_cuda.cu:184-194: per-split FP32 partials [split][n][m] over the
 * K ranges [s*k/split, (s+1)*k/split), then y = bf16(sum over s ascending). */
void oracle_gemm_split(const uint16_t* w, const uint16_t* x, int m, int n, int k,
                       int split, float* partials, uint16_t* y);

/* std::mt19937 (Matsumoto & Nishimura 1998, the C++ standard's parameters) so
 * the reference tests' seeded inputs can be regenerated bit for bit. */
typedef struct oracle_mt19937 {
    uint32_t state[624];
    int index;
} oracle_mt19937;
void oracle_mt_seed(oracle_mt19937* mt, uint32_t seed);
uint32_t oracle_mt_next(oracle_mt19937* mt);
void oracle_mt_fill(oracle_mt19937* mt, uint32_t* out, size_t count);

#ifdef __cplusplus
}
#endif
#endif
