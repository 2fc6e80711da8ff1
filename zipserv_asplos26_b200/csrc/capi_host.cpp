// Host half of the C ABI: error channel, version, packing and the legacy
// packing entry point (see include/zipserv_bridge.h, include/L_API.h).
#include <cstdint>
#include <cstring>
#include <exception>
#include <limits>
#include <new>
#include <string>

#include "../../include/zipserv_bridge.h"
#include "codec.h"
#include "packer.h"
#include "capi_internal.h"

namespace {
thread_local std::string g_last_error;
}

void zs_set_error(const char* message) { g_last_error = message ? message : ""; }

extern "C" const char* zipserv_error(void) { return g_last_error.c_str(); }

extern "C" int zipserv_abi_version(void) { return ZIPSERV_ABI_VERSION; }

extern "C" void zipserv_free(Packed* out) {
    if (!out) return;
    for (auto& p : out->buffers) {
        std::free(p);
        p = nullptr;
    }
}

extern "C" int zipserv_compress(const void* weights, int m, int k, Packed* out) {
    // integrations/vllm/native/host_bridge.cpp:18-43
    if (!out) {
        zs_set_error("Missing output descriptor");
        return -1;
    }
    std::memset(out, 0, sizeof(*out));
    if (!weights || m <= 0 || k <= 0 || m % 64 || k % 64 ||
        uint64_t(m) * uint64_t(k) > uint64_t(std::numeric_limits<int>::max()) - 4096) {
        zs_set_error("BF16 matrix must have positive 64-aligned dimensions and int32 offsets");
        return -1;
    }
    try {
        zs::HostPacked p = zs::pack_bf16(weights, m, k, -1, false, 0);
        const zs::PackedLengths len = zs::packed_lengths(p.global.get(), p.tiles);
        const uint64_t lengths[7] = {len.sm, len.rare, len.bitmap, len.bitmap,
                                     len.bitmap, len.medium, len.global};
        std::memcpy(out->lengths, lengths, sizeof(lengths));
        out->m = m;
        out->k = k;
        out->max_common = p.max_common;
        out->max_rare = p.max_rare;
        out->start_exp = uint8_t(p.base - 1);
        void* buffers[7] = {p.sm.release(), p.rare.release(), p.b1.release(), p.b2.release(),
                            p.b3.release(), p.medium.release(), p.global.release()};
        std::memcpy(out->buffers, buffers, sizeof(buffers));
        return 0;
    } catch (const std::exception& e) {
        std::memset(out, 0, sizeof(*out));
        zs_set_error(e.what());
        return -1;
    }
}

__host__ int InitBF16MatrixTripleBitmap(__nv_bfloat16* A_bf16, int M, int K, int tile_M,
                                        int tile_M_median, int tile_M_global, int tile_K,
                                        int tile_K_median, int tile_K_global,
                                        const int* top_exponents, uint8_t** sign_mantissa,
                                        __nv_bfloat16** compressed_full, uint64_t** bitmap1,
                                        uint64_t** bitmap2, uint64_t** bitmap3,
                                        int** TileOffsets, int** TileOffsets_median,
                                        int** TileOffsets_global, int& max_high_freq_count,
                                        int& max_full_count) {
    // csrc/L_API.cu:411-455: fixed tile geometry, explicit window.
    if (!A_bf16 || !zs::valid_matrix(M, K) || tile_M != 8 || tile_K != 8 || tile_M_median != 16 ||
        tile_K_median != 64 || tile_M_global != 64 || tile_K_global != 64 ||
        !zs::valid_exponents(top_exponents) || !sign_mantissa || !compressed_full || !bitmap1 ||
        !bitmap2 || !bitmap3 || !TileOffsets || !TileOffsets_median || !TileOffsets_global)
        return -1;
    try {
        zs::HostPacked p = zs::pack_bf16(A_bf16, M, K, top_exponents[0], true, 0);
        *sign_mantissa = p.sm.release();
        *compressed_full = reinterpret_cast<__nv_bfloat16*>(p.rare.release());
        *bitmap1 = p.b1.release();
        *bitmap2 = p.b2.release();
        *bitmap3 = p.b3.release();
        *TileOffsets = p.small.release();
        *TileOffsets_median = p.medium.release();
        *TileOffsets_global = p.global.release();
        max_high_freq_count = p.max_common;
        max_full_count = p.max_rare;
        return p.tiles;
    } catch (const std::exception&) {
        return -1;
    }
}
