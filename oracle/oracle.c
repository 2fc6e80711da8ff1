/*
 * TEST INFRASTRUCTURE ONLY: CPU oracle for the TCA-TBE codec and the
 * FP32-accumulated reference GEMM. See oracle.h for who may use it.
 *
 * Every function restates a reference function in plain C; the citation in
 * each comment is the reference file:line whose behaviour it follows.
 */
#include "oracle.h"

#include <limits.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

int oracle_valid_matrix(int m, int k) {
    /* csrc/CodecUtils.h:11-14 */
    return m > 0 && k > 0 && m % 64 == 0 && k % 64 == 0 &&
           (int64_t)m * k <= INT_MAX;
}

int oracle_valid_gemm(int m, int n, int k, int split_k) {
    /* csrc/CodecUtils.h:16-24 */
    if (!oracle_valid_matrix(m, k) || n < 0 || split_k < 1 || (k / 64) % split_k != 0)
        return 0;
    if ((int64_t)m * n > INT_MAX || (int64_t)k * n > INT_MAX) return 0;
    return (int64_t)m * n * split_k <= INT_MAX && (int64_t)(m / 64) * split_k <= 65535;
}

int oracle_valid_counts(int common, int rare) {
    /* csrc/CodecUtils.h:26-29 */
    return common >= 0 && common <= 4096 && common % 16 == 0 && rare >= 0 &&
           rare <= 4096 && rare % 8 == 0 && common + rare >= 4096;
}

int oracle_best_window(const uint64_t counts[256], int width) {
    /* csrc/CodecUtils.h:40-53: running window sum, strict improvement only,
     * so ties keep the lowest base. */
    if (!counts || width < 1 || width > 7) return -1;
    uint64_t current = 0;
    for (int i = 0; i < width; ++i) current += counts[i];
    uint64_t best = current;
    int base = 0;
    for (int start = 1; start <= 256 - width; ++start) {
        current -= counts[start - 1];
        current += counts[start + width - 1];
        if (current > best) {
            best = current;
            base = start;
        }
    }
    return base;
}

uint16_t oracle_exponent_bits(uint8_t start_exp, uint8_t code) {
    /* csrc/CodecUtils.h:55-62: the exponent wraps in 8 bits before the shift. */
    return (uint16_t)((uint8_t)(start_exp + code) << 7);
}

static void* xmalloc(size_t bytes) { return malloc(bytes ? bytes : 1); }

void oracle_free(oracle_packed* p) {
    if (!p) return;
    free(p->sm);
    free(p->rare);
    free(p->b1);
    free(p->b2);
    free(p->b3);
    free(p->small);
    free(p->medium);
    free(p->global);
    memset(p, 0, sizeof(*p));
}

int oracle_pack(const uint16_t* words, int m, int k, int base, int include_small,
                oracle_packed* out) {
    /* csrc/HostPacker.h:95-183 restated serially. */
    if (!out) return -1;
    memset(out, 0, sizeof(*out));
    if (!words || !oracle_valid_matrix(m, k) || base < -1 || base > 249) return -1;
    const int kt = k / 64;
    const int tiles = (m / 64) * kt;
    out->tiles = tiles;
    if (base < 0) {
        /* choose_base, csrc/HostPacker.h:61-70 */
        uint64_t hist[256];
        memset(hist, 0, sizeof(hist));
        for (int64_t i = 0; i < (int64_t)m * k; ++i) ++hist[(words[i] >> 7) & 255];
        base = oracle_best_window(hist, 7);
    }
    out->base = base;
    int32_t* g = (int32_t*)xmalloc(sizeof(int32_t) * 2 * ((size_t)tiles + 1));
    out->global = g;
    g[0] = g[1] = 0;
    /* Count pass: padded common / rare counts per 64x64 tile (:108-121). */
    for (int t = 0; t < tiles; ++t) {
        const int row = (t / kt) * 64, col = (t % kt) * 64;
        int common = 0;
        for (int r = 0; r < 64; ++r)
            for (int c = 0; c < 64; ++c) {
                const unsigned e = (words[(size_t)(row + r) * k + col + c] >> 7) & 255u;
                common += (e - (unsigned)base) < 7u;
            }
        g[2 * (t + 1)] = (common + 15) & ~15;
        g[2 * (t + 1) + 1] = (4096 - common + 7) & ~7;
    }
    /* Serial exclusive prefix and maxima of the padded counts (:122-127). */
    for (int t = 0; t < tiles; ++t) {
        if (g[2 * (t + 1)] > out->max_common) out->max_common = g[2 * (t + 1)];
        if (g[2 * (t + 1) + 1] > out->max_rare) out->max_rare = g[2 * (t + 1) + 1];
        g[2 * (t + 1)] += g[2 * t];
        g[2 * (t + 1) + 1] += g[2 * t + 1];
    }
    out->sm = (uint8_t*)xmalloc((size_t)g[2 * tiles]);
    out->rare = (uint16_t*)xmalloc(sizeof(uint16_t) * (size_t)g[2 * tiles + 1]);
    out->b1 = (uint64_t*)xmalloc(sizeof(uint64_t) * 64 * (size_t)tiles);
    out->b2 = (uint64_t*)xmalloc(sizeof(uint64_t) * 64 * (size_t)tiles);
    out->b3 = (uint64_t*)xmalloc(sizeof(uint64_t) * 64 * (size_t)tiles);
    out->medium = (int32_t*)xmalloc(sizeof(int32_t) * 8 * (size_t)tiles);
    if (include_small) out->small = (int32_t*)xmalloc(sizeof(int32_t) * 128 * (size_t)tiles);
    /* Encode pass (:135-181): small tiles ordered medium, group, column,
     * row_tile; elements inside a small tile row-major. */
    for (int t = 0; t < tiles; ++t) {
        const int row = (t / kt) * 64, col = (t % kt) * 64;
        const int c0 = g[2 * t], r0 = g[2 * t + 1];
        int ci = c0, ri = r0, s = t * 64;
        for (int med = 0; med < 4; ++med) {
            out->medium[t * 8 + med * 2] = ci - c0;
            out->medium[t * 8 + med * 2 + 1] = ri - r0;
            for (int grp = 0; grp < 4; ++grp)
                for (int column = 0; column < 2; ++column)
                    for (int rt = 0; rt < 2; ++rt, ++s) {
                        uint64_t m1 = 0, m2 = 0, m3 = 0;
                        const int pc = ci, pr = ri;
                        for (int r = 0; r < 8; ++r)
                            for (int c = 0; c < 8; ++c) {
                                const size_t idx = (size_t)(row + med * 16 + rt * 8 + r) * k +
                                                   col + grp * 16 + column * 8 + c;
                                const uint16_t w = words[idx];
                                const unsigned ei = ((w >> 7) & 255u) - (unsigned)base;
                                if (ei < 7u) {
                                    const unsigned code = ei + 1u;
                                    const int pos = r * 8 + c;
                                    m1 |= (uint64_t)(code & 1u) << pos;
                                    m2 |= (uint64_t)((code >> 1) & 1u) << pos;
                                    m3 |= (uint64_t)((code >> 2) & 1u) << pos;
                                    out->sm[ci++] = (uint8_t)((w & 127u) | ((w >> 8) & 128u));
                                } else {
                                    out->rare[ri++] = w;
                                }
                            }
                        out->b1[s] = m1;
                        out->b2[s] = m2;
                        out->b3[s] = m3;
                        if (out->small) {
                            out->small[2 * s] = ci - pc;
                            out->small[2 * s + 1] = ri - pr;
                        }
                    }
        }
        /* Only the padding is cleared (:178-179). */
        while (ci < g[2 * (t + 1)]) out->sm[ci++] = 0;
        while (ri < g[2 * (t + 1) + 1]) out->rare[ri++] = 0;
    }
    out->lengths[0] = (uint64_t)g[2 * tiles];
    out->lengths[1] = (uint64_t)g[2 * tiles + 1] * 2u;
    out->lengths[2] = out->lengths[3] = out->lengths[4] = (uint64_t)tiles * 512u;
    out->lengths[5] = out->small ? (uint64_t)tiles * 512u : 0u;
    out->lengths[6] = (uint64_t)tiles * 32u;
    out->lengths[7] = ((uint64_t)tiles + 1u) * 8u;
    return 0;
}

typedef struct decode_job {
    const uint8_t* sm;
    const uint16_t* rare;
    const uint64_t *b1, *b2, *b3;
    const int32_t *medium, *global;
    int m, k, start_exp, t0, t1;
    uint16_t* out;
    int status;
} decode_job;

static int decode_tiles(const decode_job* j) {
    /* tests/test_host_packer.cpp:14-44: invert the small-tile index
     * row = 64*(t/kt) + 16*(s/16) + 8*(s%2), col = 64*(t%kt) + 16*((s/4)%4) + 8*((s/2)%2). */
    const int kt = j->k / 64;
    const int tiles = (j->m / 64) * kt;
    const uint64_t total_common = (uint64_t)j->global[2 * tiles];
    const uint64_t total_rare = (uint64_t)j->global[2 * tiles + 1];
    for (int t = j->t0; t < j->t1; ++t) {
        int64_t ci = j->global[2 * t], ri = j->global[2 * t + 1];
        for (int s = 0; s < 64; ++s) {
            if (s % 16 == 0) {
                if (j->medium[t * 8 + (s / 16) * 2] != ci - j->global[2 * t]) return 1;
                if (j->medium[t * 8 + (s / 16) * 2 + 1] != ri - j->global[2 * t + 1]) return 1;
            }
            const int row = (t / kt) * 64 + (s / 16) * 16 + (s % 2) * 8;
            const int col = (t % kt) * 64 + ((s / 4) % 4) * 16 + ((s / 2) % 2) * 8;
            const size_t small = (size_t)t * 64 + s;
            for (int bit = 0; bit < 64; ++bit) {
                const unsigned code = (unsigned)((j->b1[small] >> bit) & 1u) |
                                      (unsigned)(((j->b2[small] >> bit) & 1u) << 1) |
                                      (unsigned)(((j->b3[small] >> bit) & 1u) << 2);
                uint16_t w;
                if (code) {
                    if ((uint64_t)ci >= total_common) return 3;
                    const uint8_t p = j->sm[ci++];
                    w = (uint16_t)(((p & 128u) << 8) |
                                   oracle_exponent_bits((uint8_t)j->start_exp, (uint8_t)code) |
                                   (p & 127u));
                } else {
                    if ((uint64_t)ri >= total_rare) return 3;
                    w = j->rare[ri++];
                }
                j->out[(size_t)(row + bit / 8) * j->k + col + bit % 8] = w;
            }
        }
        if ((ci + 15) / 16 * 16 != j->global[2 * (t + 1)]) return 2;
        if ((ri + 7) / 8 * 8 != j->global[2 * (t + 1) + 1]) return 2;
    }
    return 0;
}

static void* decode_thread(void* arg) {
    decode_job* j = (decode_job*)arg;
    j->status = decode_tiles(j);
    return NULL;
}

int oracle_decode_mt(const uint8_t* sm, const uint16_t* rare, const uint64_t* b1,
                     const uint64_t* b2, const uint64_t* b3, const int32_t* medium,
                     const int32_t* global, int m, int k, int start_exp, uint16_t* out,
                     int threads) {
    const int tiles = (m / 64) * (k / 64);
    if (threads < 1) threads = 1;
    if (threads > tiles) threads = tiles;
    decode_job* jobs = (decode_job*)xmalloc(sizeof(decode_job) * (size_t)threads);
    pthread_t* ids = (pthread_t*)xmalloc(sizeof(pthread_t) * (size_t)threads);
    int* started = (int*)xmalloc(sizeof(int) * (size_t)threads);
    for (int i = 0; i < threads; ++i) {
        decode_job j = {sm, rare, b1, b2, b3, medium, global, m, k, start_exp,
                        (int)((int64_t)tiles * i / threads), (int)((int64_t)tiles * (i + 1) / threads),
                        out, 0};
        jobs[i] = j;
        started[i] = 0;
    }
    for (int i = 1; i < threads; ++i) started[i] = pthread_create(&ids[i], NULL, decode_thread, &jobs[i]) == 0;
    jobs[0].status = decode_tiles(&jobs[0]);
    int status = jobs[0].status;
    for (int i = 1; i < threads; ++i) {
        if (started[i]) pthread_join(ids[i], NULL);
        else jobs[i].status = decode_tiles(&jobs[i]);
        if (!status) status = jobs[i].status;
    }
    free(jobs);
    free(ids);
    free(started);
    return status;
}

int oracle_decode(const uint8_t* sm, const uint16_t* rare, const uint64_t* b1,
                  const uint64_t* b2, const uint64_t* b3, const int32_t* medium,
                  const int32_t* global, int m, int k, int start_exp, uint16_t* out) {
    return oracle_decode_mt(sm, rare, b1, b2, b3, medium, global, m, k, start_exp, out, 1);
}

uint16_t oracle_f32_to_bf16(float value) {
    uint32_t u;
    memcpy(&u, &value, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

float oracle_bf16_to_f32(uint16_t bits) {
    const uint32_t u = (uint32_t)bits << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

typedef struct gemm_job {
    const uint16_t *w, *x;
    int m, n, k, row0, row1;
    uint16_t* y;
    float* y_f32;
} gemm_job;

static void gemm_rows(const gemm_job* j) {
    /* tests/test_cuda.cu:125-131: float sum over ascending column index. */
    float* wrow = (float*)xmalloc(sizeof(float) * (size_t)j->k);
    float* xrow = (float*)xmalloc(sizeof(float) * (size_t)j->k);
    for (int row = j->row0; row < j->row1; ++row) {
        for (int c = 0; c < j->k; ++c) wrow[c] = oracle_bf16_to_f32(j->w[(size_t)row * j->k + c]);
        for (int col = 0; col < j->n; ++col) {
            const uint16_t* xr = j->x + (size_t)col * j->k;
            float sum = 0.0f;
            for (int c = 0; c < j->k; ++c) xrow[c] = oracle_bf16_to_f32(xr[c]);
            for (int c = 0; c < j->k; ++c) sum += wrow[c] * xrow[c];
            const size_t o = (size_t)col * j->m + row;
            if (j->y) j->y[o] = oracle_f32_to_bf16(sum);
            if (j->y_f32) j->y_f32[o] = sum;
        }
    }
    free(wrow);
    free(xrow);
}

static void* gemm_thread(void* arg) {
    gemm_rows((const gemm_job*)arg);
    return NULL;
}

void oracle_gemm(const uint16_t* w, const uint16_t* x, int m, int n, int k, uint16_t* y,
                 float* y_f32, int threads) {
    if (threads < 1) threads = 1;
    if (threads > m) threads = m;
    gemm_job* jobs = (gemm_job*)xmalloc(sizeof(gemm_job) * (size_t)threads);
    pthread_t* ids = (pthread_t*)xmalloc(sizeof(pthread_t) * (size_t)threads);
    for (int i = 0; i < threads; ++i) {
        gemm_job j = {w, x, m, n, k, (int)((int64_t)m * i / threads),
                      (int)((int64_t)m * (i + 1) / threads), y, y_f32};
        jobs[i] = j;
    }
    int started = 0;
    for (int i = 1; i < threads; ++i)
        if (pthread_create(&ids[i], NULL, gemm_thread, &jobs[i]) == 0) ++started;
        else gemm_rows(&jobs[i]);
    gemm_rows(&jobs[0]);
    for (int i = 1; i <= started; ++i) pthread_join(ids[i], NULL);
    free(jobs);
    free(ids);
}

void oracle_gemm_split(const uint16_t* w, const uint16_t* x, int m, int n, int k, int split,
                       float* partials, uint16_t* y) {
    /* tests/test_cuda.cu:184-194 */
    const size_t count = (size_t)m * n;
    memset(partials, 0, sizeof(float) * count * (size_t)split);
    const int span = k / split;
    for (int token = 0; token < n; ++token)
        for (int row = 0; row < m; ++row) {
            const size_t offset = (size_t)token * m + row;
            for (int c = 0; c < k; ++c)
                partials[(size_t)(c / span) * count + offset] +=
                    oracle_bf16_to_f32(w[(size_t)row * k + c]) *
                    oracle_bf16_to_f32(x[(size_t)token * k + c]);
            float sum = 0.0f;
            for (int s = 0; s < split; ++s) sum += partials[(size_t)s * count + offset];
            y[offset] = oracle_f32_to_bf16(sum);
        }
}

void oracle_mt_seed(oracle_mt19937* mt, uint32_t seed) {
    mt->state[0] = seed;
    for (int i = 1; i < 624; ++i)
        mt->state[i] = 1812433253u * (mt->state[i - 1] ^ (mt->state[i - 1] >> 30)) + (uint32_t)i;
    mt->index = 624;
}

uint32_t oracle_mt_next(oracle_mt19937* mt) {
    if (mt->index >= 624) {
        for (int i = 0; i < 624; ++i) {
            const uint32_t y = (mt->state[i] & 0x80000000u) | (mt->state[(i + 1) % 624] & 0x7fffffffu);
            mt->state[i] = mt->state[(i + 397) % 624] ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
        }
        mt->index = 0;
    }
    uint32_t y = mt->state[mt->index++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}

void oracle_mt_fill(oracle_mt19937* mt, uint32_t* out, size_t count) {
    for (size_t i = 0; i < count; ++i) out[i] = oracle_mt_next(mt);
}
