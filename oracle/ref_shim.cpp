// TEST INFRASTRUCTURE ONLY. Glue that exposes the reference's own encoders,
// compiled from the reference sources where they lie (see oracle/Makefile),
// through a C ABI so tests/golden/make_golden.py can record their output.
//
//   ref_pack        -> zipserv::pack_bf16            (csrc/HostPacker.h:95-183)
//   ref_pack_legacy -> zipserv_test::reference_pack_bf16 (tests/reference_packer.h:16-268)
//
// Nothing here is part of the product library.
#include "HostPacker.h"
#include "reference_packer.h"

#include <cstring>
#include <random>
#include <exception>

extern "C" {

struct ref_packed {
    void* buffers[8];    // sm, rare, b1, b2, b3, small, medium, global (malloc'd)
    uint64_t lengths[8]; // bytes, HostPacked::lengths order
    int32_t tiles, base, max_common, max_rare;
};

int ref_pack(const uint16_t* words, int m, int k, int base, int include_small,
             unsigned workers, ref_packed* out) {
    std::memset(out, 0, sizeof(*out));
    try {
        auto p = zipserv::pack_bf16(words, m, k, base, include_small != 0, workers);
        const auto lengths = p.lengths();
        for (int i = 0; i < 8; ++i) out->lengths[i] = lengths[i];
        out->tiles = p.tiles;
        out->base = p.base;
        out->max_common = p.max_common;
        out->max_rare = p.max_rare;
        out->buffers[0] = p.common.release();
        out->buffers[1] = p.rare.release();
        out->buffers[2] = p.b1.release();
        out->buffers[3] = p.b2.release();
        out->buffers[4] = p.b3.release();
        out->buffers[5] = p.small.release();
        out->buffers[6] = p.medium.release();
        out->buffers[7] = p.global.release();
        return 0;
    } catch (const std::exception&) {
        return -1;
    }
}

int ref_pack_legacy(const uint16_t* words, int m, int k, int base, ref_packed* out) {
    std::memset(out, 0, sizeof(*out));
    int exponents[7];
    for (int i = 0; i < 7; ++i) exponents[i] = base + i;
    uint8_t* sm = nullptr;
    uint16_t* rare = nullptr;
    uint64_t *b1 = nullptr, *b2 = nullptr, *b3 = nullptr;
    int *small = nullptr, *medium = nullptr, *global = nullptr;
    int max_common = 0, max_rare = 0;
    const int tiles = zipserv_test::reference_pack_bf16(
        const_cast<uint16_t*>(words), m, k, 8, 16, 64, 8, 64, 64, exponents, &sm, &rare,
        &b1, &b2, &b3, &small, &medium, &global, max_common, max_rare);
    if (tiles <= 0) return -1;
    out->buffers[0] = sm;
    out->buffers[1] = rare;
    out->buffers[2] = b1;
    out->buffers[3] = b2;
    out->buffers[4] = b3;
    out->buffers[5] = small;
    out->buffers[6] = medium;
    out->buffers[7] = global;
    out->lengths[0] = uint64_t(global[2 * tiles]);
    out->lengths[1] = uint64_t(global[2 * tiles + 1]) * 2;
    out->lengths[2] = out->lengths[3] = out->lengths[4] = uint64_t(tiles) * 512;
    out->lengths[5] = uint64_t(tiles) * 512;
    out->lengths[6] = uint64_t(tiles) * 32;
    out->lengths[7] = (uint64_t(tiles) + 1) * 8;
    out->tiles = tiles;
    out->base = base;
    out->max_common = max_common;
    out->max_rare = max_rare;
    return 0;
}

void ref_free(ref_packed* out) {
    for (auto& b : out->buffers) {
        std::free(b);
        b = nullptr;
    }
}

// std::mt19937 itself, to pin the oracle's restatement of the generator.
void ref_mt_fill(uint32_t seed, uint32_t* out, size_t count) {
    std::mt19937 rng(seed);
    for (size_t i = 0; i < count; ++i) out[i] = rng();
}

int ref_best_window(const uint64_t* counts, int width) {
    try {
        return zipserv::best_exponent_window(counts, width);
    } catch (const std::exception&) {
        return -1;
    }
}
}
