// Host TCA-TBE encoder (see packer.h, codec.h).
//
// Three data-parallel passes over 64x64 tiles, each split into contiguous tile
// ranges across std::threads:
//   1. exponent histogram -> window base (skipped when the caller fixes base);
//   2. per-tile common count -> padded counts, serial exclusive prefix, maxima;
//   3. encode every tile straight into its exactly-sized output slice.
// Pass 3 writes disjoint slices, so the output is identical for any worker
// count. All allocation and validation happens before any thread starts.
#include "packer.h"

#include <algorithm>
#include <array>
#include <cstring>
#include <exception>
#include <stdexcept>
#include <thread>
#include <vector>

#include "codec.h"

namespace zs {
namespace {

template <class T>
HostBuffer<T> alloc(size_t count) {
    void* p = std::malloc(std::max<size_t>(1, count) * sizeof(T));
    if (!p) throw std::bad_alloc();
    return HostBuffer<T>(static_cast<T*>(p));
}

inline void load8(const unsigned char* src, uint16_t (&w)[8]) { std::memcpy(w, src, 16); }

// Run fn(begin, end) over [0, count) split into `workers` contiguous ranges.
// fn must not throw. Threads already started are joined if a later start fails.
template <class Fn>
void for_ranges(int count, unsigned workers, const Fn& fn) {
    if (workers <= 1 || count <= 1) {
        fn(0, count);
        return;
    }
    workers = std::min<unsigned>(workers, unsigned(count));
    std::vector<std::thread> pool;
    pool.reserve(workers - 1);
    auto range = [&](unsigned i) {
        return std::pair<int, int>(int(int64_t(count) * i / workers),
                                   int(int64_t(count) * (i + 1) / workers));
    };
    std::exception_ptr failure;
    try {
        for (unsigned i = 1; i < workers; ++i) {
            auto r = range(i);
            pool.emplace_back([&fn, r] { fn(r.first, r.second); });
        }
    } catch (...) {
        failure = std::current_exception();
    }
    auto r0 = range(0);
    fn(r0.first, r0.second);
    // Ranges whose thread could not start run here, after the others.
    for (unsigned i = unsigned(pool.size()) + 1; i < workers && failure; ++i) {
        auto r = range(i);
        fn(r.first, r.second);
    }
    for (auto& t : pool) t.join();
}

}  // namespace

unsigned default_workers(int tiles) {
    // ZIPSERV_PACK_WORKERS (1..64) pins the count; the output never depends on it.
    if (const char* env = std::getenv("ZIPSERV_PACK_WORKERS")) {
        const long v = std::strtol(env, nullptr, 10);
        if (v >= 1 && v <= 64) return unsigned(v);
    }
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    // About 256 tiles (1M words) per worker keeps thread start-up negligible.
    return std::max(1u, std::min({hw, 64u, unsigned(tiles / 256)}));
}

HostPacked pack_bf16(const void* words, int m, int k, int base, bool include_small,
                     unsigned workers) {
    if (!words || !valid_matrix(m, k) || base < -1 || base > 249)
        throw std::invalid_argument("BF16 packing requires a 64-aligned matrix with int32 "
                                    "offsets and an exponent window base in [0, 249]");
    if (workers > 64) throw std::invalid_argument("packing workers must be in [0, 64]");
    const auto* bytes = static_cast<const unsigned char*>(words);
    const int kt = k / 64;
    HostPacked out;
    out.tiles = (m / 64) * kt;
    const int tiles = out.tiles;
    if (!workers) workers = default_workers(tiles);
    workers = std::min<unsigned>(workers, unsigned(tiles));

    if (base < 0) {
        std::vector<std::array<uint64_t, 256>> hist(workers);
        for (auto& h : hist) h.fill(0);
        // One histogram per worker over a contiguous row range, merged after.
        const int rows = m;
        std::vector<int> bounds(workers + 1);
        for (unsigned i = 0; i <= workers; ++i) bounds[i] = int(int64_t(rows) * i / workers);
        for_ranges(int(workers), workers, [&](int b, int e) {
            for (int wi = b; wi < e; ++wi) {
                auto& h = hist[wi];
                for (int r = bounds[wi]; r < bounds[wi + 1]; ++r) {
                    const unsigned char* row = bytes + size_t(r) * k * 2;
                    for (int c = 0; c < k; c += 8) {
                        uint16_t w[8];
                        load8(row + size_t(c) * 2, w);
                        for (int i = 0; i < 8; ++i) ++h[(w[i] >> 7) & 255];
                    }
                }
            }
        });
        for (unsigned i = 1; i < workers; ++i)
            for (int e = 0; e < 256; ++e) hist[0][e] += hist[i][e];
        base = best_window(hist[0].data(), 7);
    }
    out.base = base;
    const unsigned ubase = unsigned(base);

    out.global = alloc<int32_t>(size_t(tiles + 1) * 2);
    int32_t* g = out.global.get();
    g[0] = g[1] = 0;
    for_ranges(tiles, workers, [&](int t0, int t1) {
        for (int t = t0; t < t1; ++t) {
            const unsigned char* origin =
                bytes + (size_t(t / kt) * 64 * k + size_t(t % kt) * 64) * 2;
            int common = 0;
            for (int r = 0; r < 64; ++r) {
                const unsigned char* row = origin + size_t(r) * k * 2;
                for (int c = 0; c < 64; c += 8) {
                    uint16_t w[8];
                    load8(row + c * 2, w);
                    for (int i = 0; i < 8; ++i) common += (((w[i] >> 7) & 255u) - ubase) < 7u;
                }
            }
            g[2 * t + 2] = (common + 15) & ~15;
            g[2 * t + 3] = (4096 - common + 7) & ~7;
        }
    });
    for (int t = 0; t < tiles; ++t) {
        out.max_common = std::max(out.max_common, int(g[2 * t + 2]));
        out.max_rare = std::max(out.max_rare, int(g[2 * t + 3]));
        g[2 * t + 2] += g[2 * t];
        g[2 * t + 3] += g[2 * t + 1];
    }

    out.sm = alloc<uint8_t>(size_t(g[2 * tiles]));
    out.rare = alloc<uint16_t>(size_t(g[2 * tiles + 1]));
    out.b1 = alloc<uint64_t>(size_t(tiles) * 64);
    out.b2 = alloc<uint64_t>(size_t(tiles) * 64);
    out.b3 = alloc<uint64_t>(size_t(tiles) * 64);
    out.medium = alloc<int32_t>(size_t(tiles) * 8);
    if (include_small) out.small = alloc<int32_t>(size_t(tiles) * 128);

    uint8_t* sm = out.sm.get();
    uint16_t* rare = out.rare.get();
    uint64_t *b1 = out.b1.get(), *b2 = out.b2.get(), *b3 = out.b3.get();
    int32_t* medium = out.medium.get();
    int32_t* small = out.small.get();
    for_ranges(tiles, workers, [&](int t0, int t1) {
        for (int t = t0; t < t1; ++t) {
            const unsigned char* origin =
                bytes + (size_t(t / kt) * 64 * k + size_t(t % kt) * 64) * 2;
            const int cstart = g[2 * t], rstart = g[2 * t + 1];
            int ci = cstart, ri = rstart;
            for (int s = 0; s < 64; ++s) {
                const int band = s >> 4, group = (s >> 2) & 3, column = (s >> 1) & 1,
                          rt = s & 1;
                if ((s & 15) == 0) {
                    medium[t * 8 + band * 2] = ci - cstart;
                    medium[t * 8 + band * 2 + 1] = ri - rstart;
                }
                const int c_before = ci, r_before = ri;
                uint64_t m1 = 0, m2 = 0, m3 = 0;
                const unsigned char* tile_origin =
                    origin + (size_t(band * 16 + rt * 8) * k + group * 16 + column * 8) * 2;
                for (int r = 0; r < 8; ++r) {
                    uint16_t w[8];
                    load8(tile_origin + size_t(r) * k * 2, w);
                    for (int c = 0; c < 8; ++c) {
                        const unsigned idx = ((w[c] >> 7) & 255u) - ubase;
                        if (idx < 7u) {
                            const uint64_t code = idx + 1;
                            const int pos = r * 8 + c;
                            m1 |= (code & 1) << pos;
                            m2 |= ((code >> 1) & 1) << pos;
                            m3 |= (code >> 2) << pos;
                            sm[ci++] = uint8_t((w[c] & 0x7F) | ((w[c] >> 8) & 0x80));
                        } else {
                            rare[ri++] = w[c];
                        }
                    }
                }
                b1[size_t(t) * 64 + s] = m1;
                b2[size_t(t) * 64 + s] = m2;
                b3[size_t(t) * 64 + s] = m3;
                if (small) {
                    small[(size_t(t) * 64 + s) * 2] = ci - c_before;
                    small[(size_t(t) * 64 + s) * 2 + 1] = ri - r_before;
                }
            }
            // Padding up to the next tile's start is zero.
            std::memset(sm + ci, 0, size_t(g[2 * t + 2] - ci));
            std::memset(rare + ri, 0, size_t(g[2 * t + 3] - ri) * 2);
        }
    });
    return out;
}

}  // namespace zs
