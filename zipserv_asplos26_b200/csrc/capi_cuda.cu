// GPU half of the C ABI: the L_API C++ entry points (build/L_API.cuh:32-74)
// and the extern "C" bridge (integrations/vllm/native/bridge.cu:8-51), plus
// the extensions declared in include/zipserv_bridge.h. Validation mirrors
// csrc/L_API.cu:245-252 and :344-351; on top of it every device pointer must
// be 16-byte aligned (the bulk and tensor copies require it).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>

#include "../../include/zipserv_bridge.h"
#include "capi_internal.h"
#include "codec.h"
#include "zipgemm.cuh"

#include "ptx.cuh"

namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

cudaError_t fail(cudaError_t e, const char* what) {
    zs_set_error(what);
    return e;
}

cudaError_t mm_impl(cudaStream_t stream, const void* sm, const void* rare, const void* b1,
                    const void* b2, const void* b3, const void* medium, const void* global,
                    int max_common, int max_rare, int start_exp, const void* x, void* y, int m,
                    int n, int k, const void* workspace, int split_k, int kparts,
                    const zs::GemmScratch* scratch = nullptr,
                    const zs::TpExchange* tp = nullptr) {
    if (!zs::valid_gemm(m, n, k, split_k) || !zs::valid_counts(max_common, max_rare))
        return fail(cudaErrorInvalidValue,
                    "invalid GEMM shape, Split-K or packed maxima (M, K multiples of 64; "
                    "Split-K divides K/64; int32 products)");
    if (n == 0) return cudaSuccess;
    if (!b1 || !b2 || !b3 || !medium || !global || !x || !y || (max_common && !sm) ||
        (max_rare && !rare) || (split_k > 1 && !workspace))
        return fail(cudaErrorInvalidValue, "null device pointer");
    if (!aligned16(b1) || !aligned16(b2) || !aligned16(b3) || !aligned16(medium) ||
        !aligned16(global) || !aligned16(x) || !aligned16(y) || (sm && !aligned16(sm)) ||
        (rare && !aligned16(rare)))
        return fail(cudaErrorInvalidValue, "device buffers must be 16-byte aligned");
    return zs::launch_zipgemm(stream, sm, rare, b1, b2, b3, medium, global, max_common,
                              max_rare, start_exp, x, y, m, n, k, kparts, scratch, tp);
}

cudaError_t decode_impl(cudaStream_t stream, const void* sm, const void* rare, const void* b1,
                        const void* b2, const void* b3, const void* medium, const void* global,
                        int max_common, int max_rare, int start_exp, void* out, int m, int k) {
    if (!zs::valid_matrix(m, k) || m / 64 > 65535 || !zs::valid_counts(max_common, max_rare))
        return fail(cudaErrorInvalidValue,
                    "invalid decode shape or packed maxima (M, K multiples of 64)");
    if (!b1 || !b2 || !b3 || !medium || !global || !out || (max_common && !sm) ||
        (max_rare && !rare))
        return fail(cudaErrorInvalidValue, "null device pointer");
    if (!aligned16(b1) || !aligned16(b2) || !aligned16(b3) || !aligned16(medium) ||
        !aligned16(global) || !aligned16(out) || (sm && !aligned16(sm)) ||
        (rare && !aligned16(rare)))
        return fail(cudaErrorInvalidValue, "device buffers must be 16-byte aligned");
    return zs::launch_decompress(stream, sm, rare, b1, b2, b3, medium, global, max_common,
                                 max_rare, start_exp, out, m, k);
}

}  // namespace

// ------------------------------------------------------- L_API (C++ linkage)

cudaError_t BF16TripleBitmap_MM_API(cudaStream_t stream, const uint8_t* SignMantissa,
                                    const __nv_bfloat16* CompressedFull,
                                    const uint64_t* Bitmap1, const uint64_t* Bitmap2,
                                    const uint64_t* Bitmap3, const int* TileOffsets_Median,
                                    const int* TileOffsets_Global, const int max_high_freq_count,
                                    const int max_full_count, const uint8_t start_exp,
                                    const __nv_bfloat16* B, __nv_bfloat16* C, const int M_Global,
                                    const int N_Global, const int K_Global,
                                    __nv_bfloat16* Reduction_Workspace, int Split_K) {
    return mm_impl(stream, SignMantissa, CompressedFull, Bitmap1, Bitmap2, Bitmap3,
                   TileOffsets_Median, TileOffsets_Global, max_high_freq_count, max_full_count,
                   start_exp, B, C, M_Global, N_Global, K_Global, Reduction_Workspace, Split_K, 0);
}

cudaError_t BF16TripleBitmap_MM_API_FP32(cudaStream_t stream, const uint8_t* sm,
                                         const __nv_bfloat16* rare, const uint64_t* b1,
                                         const uint64_t* b2, const uint64_t* b3,
                                         const int* medium, const int* global, int max_common,
                                         int max_rare, uint8_t start_exp, const __nv_bfloat16* x,
                                         __nv_bfloat16* y, int m, int n, int k, float* workspace,
                                         int split_k) {
    return mm_impl(stream, sm, rare, b1, b2, b3, medium, global, max_common, max_rare,
                   start_exp, x, y, m, n, k, workspace, split_k, 0);
}

cudaError_t BF16TripleBitmap_Decompress_API(cudaStream_t stream, const uint8_t* SignMantissa,
                                            const __nv_bfloat16* CompressedFull,
                                            const uint64_t* Bitmap1, const uint64_t* Bitmap2,
                                            const uint64_t* Bitmap3,
                                            const int* TileOffsets_Median,
                                            const int* TileOffsets_Global,
                                            const int max_high_freq_count,
                                            const int max_full_count, const uint8_t start_exp,
                                            __nv_bfloat16* Output, const int M_Global,
                                            const int K_Global) {
    return decode_impl(stream, SignMantissa, CompressedFull, Bitmap1, Bitmap2, Bitmap3,
                       TileOffsets_Median, TileOffsets_Global, max_high_freq_count,
                       max_full_count, start_exp, Output, M_Global, K_Global);
}

// ------------------------------------------------------------- C bridge

extern "C" int zipserv_mm(void* stream, const void* sm, const void* rare, const void* b1,
                          const void* b2, const void* b3, const void* medium, const void* global,
                          int max_common, int max_rare, int start_exp, const void* x, void* y,
                          int m, int n, int k, void* workspace, int split_k) {
    return int(mm_impl(static_cast<cudaStream_t>(stream), sm, rare, b1, b2, b3, medium, global,
                       max_common, max_rare, start_exp & 255, x, y, m, n, k, workspace, split_k,
                       0));
}

extern "C" int zipserv_mm_fp32(void* stream, const void* sm, const void* rare, const void* b1,
                               const void* b2, const void* b3, const void* medium,
                               const void* global, int max_common, int max_rare, int start_exp,
                               const void* x, void* y, int m, int n, int k, void* workspace,
                               int split_k) {
    return int(mm_impl(static_cast<cudaStream_t>(stream), sm, rare, b1, b2, b3, medium, global,
                       max_common, max_rare, start_exp & 255, x, y, m, n, k, workspace, split_k,
                       0));
}

extern "C" int zipserv_decode(void* stream, const void* sm, const void* rare, const void* b1,
                              const void* b2, const void* b3, const void* medium,
                              const void* global, int max_common, int max_rare, int start_exp,
                              void* output, int m, int k) {
    return int(decode_impl(static_cast<cudaStream_t>(stream), sm, rare, b1, b2, b3, medium,
                           global, max_common, max_rare, start_exp & 255, output, m, k));
}

extern "C" int zipserv_mm_kparts(void* stream, const void* sm, const void* rare, const void* b1,
                                 const void* b2, const void* b3, const void* medium,
                                 const void* global, int max_common, int max_rare, int start_exp,
                                 const void* x, void* y, int m, int n, int k, int k_parts) {
    if (k_parts < 0 || k_parts > 16 || (zs::valid_matrix(m, k) && k_parts > k / 64)) {
        zs_set_error("k_parts must be in [0, min(16, K/64)]");
        return int(cudaErrorInvalidValue);
    }
    return int(mm_impl(static_cast<cudaStream_t>(stream), sm, rare, b1, b2, b3, medium, global,
                       max_common, max_rare, start_exp & 255, x, y, m, n, k, nullptr, 1,
                       k_parts));
}

extern "C" int zipserv_mm_workspace_size(int m, int n, int k, int k_parts,
                                         uint64_t* partial_bytes, uint64_t* counter_bytes) {
    if (!partial_bytes || !counter_bytes) return int(cudaErrorInvalidValue);
    *partial_bytes = *counter_bytes = 0;
    if (!zs::valid_gemm(m, n, k, 1) || k_parts < 0 || k_parts > 16 || k_parts > k / 64) {
        zs_set_error("invalid GEMM shape or k_parts");
        return int(cudaErrorInvalidValue);
    }
    if (n == 0) return 0;
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return int(e);
    size_t p = 0, c = 0;
    zs::gemm_workspace_bytes(m, n, k, k_parts, device, &p, &c);
    *partial_bytes = p, *counter_bytes = c;
    return 0;
}

extern "C" int zipserv_mm_ws(void* stream, const void* sm, const void* rare, const void* b1,
                             const void* b2, const void* b3, const void* medium,
                             const void* global, int max_common, int max_rare, int start_exp,
                             const void* x, void* y, int m, int n, int k, int k_parts,
                             void* partials, uint64_t partial_bytes, void* counters,
                             uint64_t counter_bytes) {
    if (k_parts < 0 || k_parts > 16 || (zs::valid_matrix(m, k) && k_parts > k / 64)) {
        zs_set_error("k_parts must be in [0, min(16, K/64)]");
        return int(cudaErrorInvalidValue);
    }
    const zs::GemmScratch scratch{partials, size_t(partial_bytes), counters,
                                  size_t(counter_bytes)};
    return int(mm_impl(static_cast<cudaStream_t>(stream), sm, rare, b1, b2, b3, medium, global,
                       max_common, max_rare, start_exp & 255, x, y, m, n, k, nullptr, 1,
                       k_parts, &scratch));
}

extern "C" int zipserv_mm_plan(int m, int n, int k) {
    if (!zs::valid_gemm(m, n, k, 1)) return -1;
    if (n == 0) return 1;
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return -1;
    return zs::plan_kparts(m, n, k, device);
}

extern "C" uint64_t zipserv_mm_reducer_wait(uint64_t ns) { return zs::set_reducer_wait_ns(ns); }

// ------------------------------------------------ fused row-parallel all-reduce

extern "C" int zipserv_mm_allreduce_sizes(int m, int n, int world, uint64_t* recv_bytes,
                                          uint64_t* flag_bytes) {
    if (!recv_bytes || !flag_bytes) return int(cudaErrorInvalidValue);
    size_t r = 0, f = 0;
    zs::allreduce_exchange_bytes(m, n, world, &r, &f);
    *recv_bytes = r, *flag_bytes = f;
    if (!r) {
        zs_set_error("zipserv_mm_allreduce_sizes: invalid M, N or world (2..8)");
        return int(cudaErrorInvalidValue);
    }
    return 0;
}

extern "C" int zipserv_mm_allreduce(void* stream, const void* sm, const void* rare,
                                    const void* b1, const void* b2, const void* b3,
                                    const void* medium, const void* global, int max_common,
                                    int max_rare, int start_exp, const void* x, void* y, int m,
                                    int n, int k, int world, int rank, void* const* recv,
                                    void* const* flags, void* state, uint64_t recv_bytes,
                                    uint64_t flag_bytes) {
    if (world < 2 || world > zs::kMaxTp || rank < 0 || rank >= world || !recv || !flags ||
        !state || !aligned16(state)) {
        zs_set_error("zipserv_mm_allreduce: world must be 2..8, rank in [0, world), exchange "
                     "pointers non-null (state 16-byte aligned)");
        return int(cudaErrorInvalidValue);
    }
    if (n > 0 && zs::valid_gemm(m, n, k, 1)) {
        size_t need_r = 0, need_f = 0;
        zs::allreduce_exchange_bytes(m, n, world, &need_r, &need_f);
        if (recv_bytes < need_r || flag_bytes < need_f) {
            zs_set_error("zipserv_mm_allreduce: receive buffer or flags smaller than "
                         "zipserv_mm_allreduce_sizes reports");
            return int(cudaErrorInvalidValue);
        }
        for (int r = 0; r < world; ++r)
            if (!recv[r] || !flags[r] || !aligned16(recv[r]) || !aligned16(flags[r])) {
                zs_set_error("zipserv_mm_allreduce: every rank's buffers must be non-null and "
                             "16-byte aligned");
                return int(cudaErrorInvalidValue);
            }
    }
    const zs::TpExchange tp{world, rank, recv, flags, state};
    return int(mm_impl(static_cast<cudaStream_t>(stream), sm, rare, b1, b2, b3, medium, global,
                       max_common, max_rare, start_exp & 255, x, y, m, n, k, nullptr, 1, 0,
                       nullptr, &tp));
}

// Device memory a process shares with the other ranks through CUDA IPC.
extern "C" int zipserv_ipc_alloc(uint64_t bytes, void** ptr) {
    if (!ptr || !bytes) return int(cudaErrorInvalidValue);
    cudaError_t e = cudaMalloc(ptr, bytes);
    if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
    if (e != cudaSuccess) zs_set_error(cudaGetErrorString(e));
    return int(e);
}
extern "C" int zipserv_ipc_free(void* ptr) { return int(cudaFree(ptr)); }
extern "C" int zipserv_ipc_handle(void* ptr, void* handle) {
    if (!ptr || !handle) return int(cudaErrorInvalidValue);
    return int(cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), ptr));
}
extern "C" int zipserv_ipc_open(const void* handle, void** ptr) {
    if (!ptr || !handle) return int(cudaErrorInvalidValue);
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) zs_set_error(cudaGetErrorString(e));
    return int(e);
}
extern "C" int zipserv_ipc_close(void* ptr) { return int(cudaIpcCloseMemHandle(ptr)); }

extern "C" int zipserv_device_flags(unsigned* flags, int clear) {
    if (!flags) return int(cudaErrorInvalidValue);
    cudaError_t e = cudaMemcpyFromSymbol(flags, zs::g_device_flags, sizeof(unsigned));
    if (e == cudaSuccess && clear) {
        const unsigned zero = 0;
        e = cudaMemcpyToSymbol(zs::g_device_flags, &zero, sizeof(unsigned));
    }
    if (e != cudaSuccess) zs_set_error(cudaGetErrorString(e));
    return int(e);
}
