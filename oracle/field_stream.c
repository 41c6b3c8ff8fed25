/*
 * Oracle (test infrastructure only): Goldilocks field, quadratic extension
 * and the ChaCha8 FpStream.
 *
 * Field: rust/volta-field/src/lib.rs:10-103 (Fp add/sub/mul/reduce128),
 *        lib.rs:140-210 (Fp2 with phi^2 = 7).  Products are reduced with a
 *        plain unsigned __int128 remainder here, a deliberately different
 *        route from the reference's 2^64 = 2^32-1 folding so that the oracle
 *        is an independent check of the device reduction.
 * Stream: lib.rs:222-268 (FpStream::domain_separated, next_fp rejection,
 *         next_fp2, next_bits) over rand_chacha 0.3.1's ChaCha8Rng:
 *         state = "expand 32-byte k" | key | block counter (64-bit LE, words
 *         12..13) | stream id (64-bit LE, words 14..15); 4 double rounds;
 *         output words consumed as little-endian u64 pairs (low word first).
 *         Pinned by the reference's byte-identity record
 *         benchmarks/results/p7b-chacha8-fp-diff-2026-07-13-32653fd7e076.json.
 */
#include "oracle.h"

#include <omp.h>
#include <string.h>

/* Thread count of every OpenMP loop in the oracle.  Set explicitly by the
 * CPU baseline so that a launcher's OMP_NUM_THREADS (torchrun sets 1 when it
 * starts several processes) does not silently serialise it. */
void or_set_threads(int n) {
    if (n > 0) omp_set_num_threads(n);
}

int or_max_threads(void) { return omp_get_max_threads(); }

#define P_GOLD 0xFFFFFFFF00000001ULL

uint64_t or_fp_add(uint64_t a, uint64_t b) {
    unsigned __int128 s = (unsigned __int128)a + b;
    return (uint64_t)(s % P_GOLD);
}

uint64_t or_fp_sub(uint64_t a, uint64_t b) {
    unsigned __int128 s = (unsigned __int128)a + P_GOLD - (b % P_GOLD);
    return (uint64_t)(s % P_GOLD);
}

uint64_t or_fp_mul(uint64_t a, uint64_t b) {
    unsigned __int128 m = (unsigned __int128)a * b;
    return (uint64_t)(m % P_GOLD);
}

uint64_t or_fp_pow(uint64_t a, uint64_t e) {
    uint64_t acc = 1, base = a % P_GOLD;
    while (e) {
        if (e & 1) acc = or_fp_mul(acc, base);
        base = or_fp_mul(base, base);
        e >>= 1;
    }
    return acc;
}

uint64_t or_fp_inv(uint64_t a) { return or_fp_pow(a, P_GOLD - 2); }

static uint64_t fneg(uint64_t a) { return a ? P_GOLD - a : 0; }

ofp2 or_fp2_add(ofp2 a, ofp2 b) {
    ofp2 r = {or_fp_add(a.c0, b.c0), or_fp_add(a.c1, b.c1)};
    return r;
}

ofp2 or_fp2_sub(ofp2 a, ofp2 b) {
    ofp2 r = {or_fp_sub(a.c0, b.c0), or_fp_sub(a.c1, b.c1)};
    return r;
}

ofp2 or_fp2_mul(ofp2 a, ofp2 b) {
    /* (a0 + a1 phi)(b0 + b1 phi) = a0 b0 + 7 a1 b1 + (a0 b1 + a1 b0) phi */
    ofp2 r;
    r.c0 = or_fp_add(or_fp_mul(a.c0, b.c0), or_fp_mul(7, or_fp_mul(a.c1, b.c1)));
    r.c1 = or_fp_add(or_fp_mul(a.c0, b.c1), or_fp_mul(a.c1, b.c0));
    return r;
}

ofp2 or_fp2_inv(ofp2 a) {
    uint64_t norm = or_fp_sub(or_fp_mul(a.c0, a.c0), or_fp_mul(7, or_fp_mul(a.c1, a.c1)));
    uint64_t ni = or_fp_inv(norm);
    ofp2 r = {or_fp_mul(a.c0, ni), or_fp_mul(fneg(a.c1), ni)};
    return r;
}

void or_fp_mul_batch(const uint64_t* a, const uint64_t* b, uint64_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = or_fp_mul(a[i], b[i]);
}

/* ------------------------------------------------------------------ */
/* ChaCha8                                                              */
/* ------------------------------------------------------------------ */

static uint32_t rotl(uint32_t x, int n) { return (x << n) | (x >> (32 - n)); }

#define QR(a, b, c, d)            \
    do {                          \
        a += b; d = rotl(d ^ a, 16); \
        c += d; b = rotl(b ^ c, 12); \
        a += b; d = rotl(d ^ a, 8);  \
        c += d; b = rotl(b ^ c, 7);  \
    } while (0)

static void chacha8_block(const uint32_t key[8], uint64_t counter, uint64_t stream,
                          uint32_t out[16]) {
    uint32_t s[16];
    s[0] = 0x61707865u;
    s[1] = 0x3320646eu;
    s[2] = 0x79622d32u;
    s[3] = 0x6b206574u;
    for (int i = 0; i < 8; ++i) s[4 + i] = key[i];
    s[12] = (uint32_t)counter;
    s[13] = (uint32_t)(counter >> 32);
    s[14] = (uint32_t)stream;
    s[15] = (uint32_t)(stream >> 32);
    uint32_t x[16];
    memcpy(x, s, sizeof x);
    for (int dr = 0; dr < 4; ++dr) {
        QR(x[0], x[4], x[8], x[12]);
        QR(x[1], x[5], x[9], x[13]);
        QR(x[2], x[6], x[10], x[14]);
        QR(x[3], x[7], x[11], x[15]);
        QR(x[0], x[5], x[10], x[15]);
        QR(x[1], x[6], x[11], x[12]);
        QR(x[2], x[7], x[8], x[13]);
        QR(x[3], x[4], x[9], x[14]);
    }
    for (int i = 0; i < 16; ++i) out[i] = x[i] + s[i];
}

void or_stream_init(or_stream* s, const uint8_t seed[32], uint64_t domain) {
    for (int i = 0; i < 8; ++i) {
        s->key[i] = (uint32_t)seed[4 * i] | ((uint32_t)seed[4 * i + 1] << 8) |
                    ((uint32_t)seed[4 * i + 2] << 16) | ((uint32_t)seed[4 * i + 3] << 24);
    }
    s->stream = domain;
    s->block = 0;
    s->idx = 8;
}

uint64_t or_stream_next_u64(or_stream* s) {
    if (s->idx == 8) {
        chacha8_block(s->key, s->block, s->stream, s->words);
        s->block++;
        s->idx = 0;
    }
    uint64_t lo = s->words[2 * s->idx], hi = s->words[2 * s->idx + 1];
    s->idx++;
    return lo | (hi << 32);
}

uint64_t or_stream_next_fp(or_stream* s) {
    for (;;) {
        uint64_t v = or_stream_next_u64(s);
        if (v < P_GOLD) return v;
    }
}

ofp2 or_stream_next_fp2(or_stream* s) {
    ofp2 r;
    r.c0 = or_stream_next_fp(s);
    r.c1 = or_stream_next_fp(s);
    return r;
}

uint64_t or_stream_next_bits(or_stream* s, unsigned width) {
    uint64_t raw = or_stream_next_u64(s);
    return width >= 64 ? raw : (raw & ((1ULL << width) - 1));
}

void or_chacha_fp_rows(const uint8_t seed[32], uint64_t base, size_t rows, size_t count,
                       uint64_t* out) {
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < rows; ++r) {
        or_stream st;
        or_stream_init(&st, seed, base + (uint64_t)r);
        for (size_t j = 0; j < count; ++j) out[r * count + j] = or_stream_next_fp(&st);
    }
}

void or_chacha_fp2_rows_padded(const uint8_t seed[32], uint64_t base, size_t rows,
                               size_t count, size_t padded, ofp2* out) {
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < rows; ++r) {
        or_stream st;
        or_stream_init(&st, seed, base + (uint64_t)r);
        for (size_t j = 0; j < count; ++j) out[r * padded + j] = or_stream_next_fp2(&st);
        for (size_t j = count; j < padded; ++j) {
            out[r * padded + j].c0 = 0;
            out[r * padded + j].c1 = 0;
        }
    }
}

void or_stream_fill_u64(const uint8_t seed[32], uint64_t domain, size_t n, uint64_t* out) {
    or_stream st;
    or_stream_init(&st, seed, domain);
    for (size_t i = 0; i < n; ++i) out[i] = or_stream_next_u64(&st);
}

uint64_t or_fnv_u64(uint64_t h, const uint64_t* v, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        h ^= v[i];
        h *= 0x00000100000001B3ULL;
    }
    return h;
}
