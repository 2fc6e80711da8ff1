// C++ entry points of the B200 ZipServ library, one for one with the
// reference's native API header (build/L_API.cuh:32-102): same names, C++
// linkage, argument order and meaning, so code written against the reference
// header links against libzipserv_b200.so unchanged.
//
// Shared contract (build/L_API.cuh:23-31): packed inputs come from
// InitBF16MatrixTripleBitmap / zipserv_compress; M and K are positive
// multiples of 64, N may be zero; Split_K >= 1 divides K/64; products fit
// int32 and (M/64)*Split_K <= 65535. Device buffers belong to the caller and
// must outlive the enqueued work. Shapes and pointers are validated (null or
// not 16-byte aligned -> cudaErrorInvalidValue), packed contents are not.
// Weight reconstruction is bit-exact; GEMM sums are FP32 and may round
// differently from another backend.
//
// Difference from the reference, by design: the K reduction runs inside the
// fused kernel in FP32 (partial pieces exchanged between CTAs through L2 and
// added in a fixed order), not in a second kernel over a Split_K workspace.
// The workspace argument is still validated (required when Split_K > 1) but
// never written.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

// build/L_API.cuh:32-50
cudaError_t BF16TripleBitmap_MM_API(cudaStream_t stream, const uint8_t* SignMantissa,
                                    const __nv_bfloat16* CompressedFull,
                                    const uint64_t* Bitmap1, const uint64_t* Bitmap2,
                                    const uint64_t* Bitmap3, const int* TileOffsets_Median,
                                    const int* TileOffsets_Global, const int max_high_freq_count,
                                    const int max_full_count, const uint8_t start_exp,
                                    const __nv_bfloat16* B, __nv_bfloat16* C,
                                    const int M_Global, const int N_Global, const int K_Global,
                                    __nv_bfloat16* Reduction_Workspace, int Split_K);

// build/L_API.cuh:54-59
cudaError_t BF16TripleBitmap_MM_API_FP32(cudaStream_t stream, const uint8_t* sm,
                                         const __nv_bfloat16* rare, const uint64_t* b1,
                                         const uint64_t* b2, const uint64_t* b3,
                                         const int* medium, const int* global, int max_common,
                                         int max_rare, uint8_t start_exp, const __nv_bfloat16* x,
                                         __nv_bfloat16* y, int m, int n, int k, float* workspace,
                                         int split_k);

// build/L_API.cuh:60-74. Dense row-major M x K output, bit-exact.
cudaError_t BF16TripleBitmap_Decompress_API(cudaStream_t stream, const uint8_t* SignMantissa,
                                            const __nv_bfloat16* CompressedFull,
                                            const uint64_t* Bitmap1, const uint64_t* Bitmap2,
                                            const uint64_t* Bitmap3,
                                            const int* TileOffsets_Median,
                                            const int* TileOffsets_Global,
                                            const int max_high_freq_count,
                                            const int max_full_count, const uint8_t start_exp,
                                            __nv_bfloat16* Output, const int M_Global,
                                            const int K_Global);

// build/L_API.cuh:75-102. CPU packing with a caller-chosen window
// top_exponents[0..6] (seven consecutive values, first in [0, 249]; decoding
// then uses start_exp = uint8(top_exponents[0] - 1)). Tile sizes must be the
// fixed (8, 16, 64, 8, 64, 64). Returns the number of global tiles or -1; on
// success the caller owns eight malloc'd buffers (free()), including the
// per-small-tile offsets; on failure nothing is transferred.
__host__ int InitBF16MatrixTripleBitmap(__nv_bfloat16* A_bf16, int M, int K, int tile_M,
                                        int tile_M_median, int tile_M_global, int tile_K,
                                        int tile_K_median, int tile_K_global,
                                        const int* top_exponents, uint8_t** sign_mantissa,
                                        __nv_bfloat16** compressed_full, uint64_t** bitmap1,
                                        uint64_t** bitmap2, uint64_t** bitmap3,
                                        int** TileOffsets, int** TileOffsets_median,
                                        int** TileOffsets_global, int& max_high_freq_count,
                                        int& max_full_count);
