/*
 * Oracle (test infrastructure only): Ligero PCS pieces and the GEMM epilogue.
 *
 *   NTT           rust/volta-pcs/src/ntt.rs:9-70 (DIT, bit-reversed reorder,
 *                 omega = 7^((p-1) >> log2 n), natural-order output)
 *   BLAKE3        third-party crate blake3 1.8.5 (rust/Cargo.lock), restated
 *                 from the published BLAKE3 specification: 7-round
 *                 compression, 1 KiB chunks of 64-byte blocks, flags
 *                 CHUNK_START=1 CHUNK_END=2 PARENT=4 ROOT=8, left subtree =
 *                 largest power of two of chunks leaving one for the right.
 *   column leaves rust/volta-pcs/src/ligero.rs:351-359 (LE u64 down a column),
 *                 ligero.rs:595-616
 *   merkle        rust/volta-pcs/src/merkle.rs:9-51 (levels leaf->root,
 *                 parent = blake3(left || right), path = siblings bottom-up)
 *   messages      ligero.rs:553-585 (w mod p || pads || 0)
 *   combine rows  rust/volta-accel/src/lib.rs:6478-6560 (CPU semantics)
 *   GEMM epilogue rust/volta-gpt2/src/gemm.rs:19-154
 */
#include "oracle.h"

#include <stdlib.h>
#include <string.h>

#define P_GOLD 0xFFFFFFFF00000001ULL

static uint64_t embed_i64(int64_t v) { return v >= 0 ? (uint64_t)v : P_GOLD - (uint64_t)(-v); }

/* ------------------------------------------------------------------ */
/* NTT                                                                  */
/* ------------------------------------------------------------------ */

static size_t bitrev(size_t i, unsigned bits) {
    size_t r = 0;
    for (unsigned b = 0; b < bits; ++b) r |= ((i >> b) & 1) << (bits - 1 - b);
    return r;
}

static void ntt_row(uint64_t* a, size_t n, const uint64_t* tw) {
    unsigned bits = 0;
    while (((size_t)1 << bits) < n) ++bits;
    for (size_t i = 0; i < n; ++i) {
        size_t j = bitrev(i, bits);
        if (i < j) {
            uint64_t t = a[i];
            a[i] = a[j];
            a[j] = t;
        }
    }
    for (size_t len = 2; len <= n; len *= 2) {
        size_t step = n / len;
        for (size_t s = 0; s < n; s += len)
            for (size_t k = 0; k < len / 2; ++k) {
                uint64_t u = a[s + k], v = or_fp_mul(a[s + k + len / 2], tw[k * step]);
                a[s + k] = or_fp_add(u, v);
                a[s + k + len / 2] = or_fp_sub(u, v);
            }
    }
}

static uint64_t* twiddles(size_t n) {
    unsigned bits = 0;
    while (((size_t)1 << bits) < n) ++bits;
    uint64_t w = or_fp_pow(7, (P_GOLD - 1) >> bits);
    uint64_t* tw = (uint64_t*)malloc(sizeof(uint64_t) * (n / 2 + 1));
    uint64_t acc = 1;
    for (size_t i = 0; i < n / 2; ++i) {
        tw[i] = acc;
        acc = or_fp_mul(acc, w);
    }
    return tw;
}

void or_ntt_batch(const uint64_t* in, size_t rows, size_t msg_len, size_t n, uint64_t* out) {
    uint64_t* tw = twiddles(n);
#pragma omp parallel for schedule(dynamic)
    for (size_t r = 0; r < rows; ++r) {
        uint64_t* o = out + r * n;
        for (size_t j = 0; j < n; ++j) o[j] = j < msg_len ? in[r * msg_len + j] : 0;
        ntt_row(o, n, tw);
    }
    free(tw);
}

void or_ntt_fp2_batch(const ofp2* in, size_t rows, size_t msg_len, size_t n, ofp2* out) {
    uint64_t* tw = twiddles(n);
#pragma omp parallel for schedule(dynamic)
    for (size_t r = 0; r < rows; ++r) {
        uint64_t* c0 = (uint64_t*)malloc(sizeof(uint64_t) * n);
        uint64_t* c1 = (uint64_t*)malloc(sizeof(uint64_t) * n);
        for (size_t j = 0; j < n; ++j) {
            ofp2 v = j < msg_len ? in[r * msg_len + j] : (ofp2){0, 0};
            c0[j] = v.c0;
            c1[j] = v.c1;
        }
        ntt_row(c0, n, tw);
        ntt_row(c1, n, tw);
        for (size_t j = 0; j < n; ++j) {
            out[r * n + j].c0 = c0[j];
            out[r * n + j].c1 = c1[j];
        }
        free(c0);
        free(c1);
    }
    free(tw);
}

/* ------------------------------------------------------------------ */
/* BLAKE3                                                               */
/* ------------------------------------------------------------------ */

static const uint32_t B3_IV[8] = {0x6A09E667u, 0xBB67AE85u, 0x3C6EF372u, 0xA54FF53Au,
                                  0x510E527Fu, 0x9B05688Cu, 0x1F83D9ABu, 0x5BE0CD19u};
static const uint8_t B3_PERM[16] = {2, 6, 3, 10, 7, 0, 4, 13, 1, 11, 12, 5, 9, 14, 15, 8};

static uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

static void b3_g(uint32_t* s, int a, int b, int c, int d, uint32_t mx, uint32_t my) {
    s[a] = s[a] + s[b] + mx;
    s[d] = rotr(s[d] ^ s[a], 16);
    s[c] = s[c] + s[d];
    s[b] = rotr(s[b] ^ s[c], 12);
    s[a] = s[a] + s[b] + my;
    s[d] = rotr(s[d] ^ s[a], 8);
    s[c] = s[c] + s[d];
    s[b] = rotr(s[b] ^ s[c], 7);
}

/* Compression returning the 8-word chaining value (first half of output). */
static void b3_compress(const uint32_t cv[8], const uint8_t block[64], uint64_t counter,
                        uint32_t block_len, uint32_t flags, uint32_t out[8]) {
    uint32_t m[16], s[16], t[16];
    for (int i = 0; i < 16; ++i)
        m[i] = (uint32_t)block[4 * i] | ((uint32_t)block[4 * i + 1] << 8) |
               ((uint32_t)block[4 * i + 2] << 16) | ((uint32_t)block[4 * i + 3] << 24);
    for (int i = 0; i < 8; ++i) s[i] = cv[i];
    for (int i = 0; i < 4; ++i) s[8 + i] = B3_IV[i];
    s[12] = (uint32_t)counter;
    s[13] = (uint32_t)(counter >> 32);
    s[14] = block_len;
    s[15] = flags;
    for (int r = 0; r < 7; ++r) {
        b3_g(s, 0, 4, 8, 12, m[0], m[1]);
        b3_g(s, 1, 5, 9, 13, m[2], m[3]);
        b3_g(s, 2, 6, 10, 14, m[4], m[5]);
        b3_g(s, 3, 7, 11, 15, m[6], m[7]);
        b3_g(s, 0, 5, 10, 15, m[8], m[9]);
        b3_g(s, 1, 6, 11, 12, m[10], m[11]);
        b3_g(s, 2, 7, 8, 13, m[12], m[13]);
        b3_g(s, 3, 4, 9, 14, m[14], m[15]);
        if (r < 6) {
            for (int i = 0; i < 16; ++i) t[i] = m[B3_PERM[i]];
            memcpy(m, t, sizeof m);
        }
    }
    for (int i = 0; i < 8; ++i) out[i] = s[i] ^ s[i + 8];
}

/* Chaining value of one chunk (<= 1024 bytes); root flag when it is the only chunk.
 * key: the 8 key words (the IV for plain hashing); mode: the mode flag added to
 * every compression (0 hash, 16 keyed hash, 32 key-derivation context, 64
 * key-derivation material). */
static void b3_chunk_cv(const uint8_t* data, size_t len, uint64_t chunk_index, int is_root,
                        const uint32_t key[8], uint32_t mode, uint32_t out[8]) {
    uint32_t cv[8];
    memcpy(cv, key, sizeof cv);
    size_t nblocks = len == 0 ? 1 : (len + 63) / 64;
    for (size_t b = 0; b < nblocks; ++b) {
        uint8_t block[64] = {0};
        size_t take = len - b * 64 < 64 ? len - b * 64 : 64;
        if (len) memcpy(block, data + b * 64, take);
        uint32_t flags = mode;
        if (b == 0) flags |= 1;
        if (b + 1 == nblocks) {
            flags |= 2;
            if (is_root) flags |= 8;
        }
        b3_compress(cv, block, chunk_index, (uint32_t)(len ? take : 0), flags, cv);
    }
    memcpy(out, cv, sizeof cv);
}

static void b3_parent(const uint32_t l[8], const uint32_t r[8], int is_root, const uint32_t key[8],
                      uint32_t mode, uint32_t out[8]) {
    uint8_t block[64];
    for (int i = 0; i < 8; ++i) {
        for (int k = 0; k < 4; ++k) {
            block[4 * i + k] = (uint8_t)(l[i] >> (8 * k));
            block[32 + 4 * i + k] = (uint8_t)(r[i] >> (8 * k));
        }
    }
    b3_compress(key, block, 0, 64, mode | 4 | (is_root ? 8 : 0), out);
}

/* Subtree over chunks [first, first+count) of the input. */
static void b3_subtree(const uint8_t* data, size_t len, size_t first, size_t count, int is_root,
                       const uint32_t key[8], uint32_t mode, uint32_t out[8]) {
    if (count == 1) {
        size_t off = first * 1024;
        size_t take = len - off < 1024 ? len - off : 1024;
        b3_chunk_cv(data + off, take, first, is_root, key, mode, out);
        return;
    }
    size_t left = 1;
    while (left * 2 < count) left *= 2;
    uint32_t lcv[8], rcv[8];
    b3_subtree(data, len, first, left, 0, key, mode, lcv);
    b3_subtree(data, len, first + left, count - left, 0, key, mode, rcv);
    b3_parent(lcv, rcv, is_root, key, mode, out);
}

static void b3_root(const uint8_t* data, size_t len, const uint32_t key[8], uint32_t mode, uint8_t out[32]) {
    size_t chunks = len == 0 ? 1 : (len + 1023) / 1024;
    uint32_t cv[8];
    b3_subtree(data, len, 0, chunks, 1, key, mode, cv);
    for (int i = 0; i < 8; ++i)
        for (int k = 0; k < 4; ++k) out[4 * i + k] = (uint8_t)(cv[i] >> (8 * k));
}

void or_blake3(const uint8_t* data, size_t len, uint8_t out[32]) { b3_root(data, len, B3_IV, 0, out); }

/* derive_key mode: the context string hashed with the context flag gives
 * the key with which the material is hashed (material flag). */
void or_blake3_derive_key(const uint8_t* context, size_t context_len, const uint8_t* data, size_t len,
                          uint8_t out[32]) {
    uint8_t k[32];
    uint32_t key[8];
    b3_root(context, context_len, B3_IV, 32, k);
    for (int i = 0; i < 8; ++i)
        key[i] = (uint32_t)k[4 * i] | ((uint32_t)k[4 * i + 1] << 8) | ((uint32_t)k[4 * i + 2] << 16) |
                 ((uint32_t)k[4 * i + 3] << 24);
    b3_root(data, len, key, 64, out);
}

void or_hash_fp_columns(const uint64_t* m, size_t rows, size_t cols, uint8_t* leaves) {
#pragma omp parallel
    {
        uint8_t* buf = (uint8_t*)malloc(rows * 8);
#pragma omp for schedule(static)
        for (size_t j = 0; j < cols; ++j) {
            for (size_t i = 0; i < rows; ++i) {
                uint64_t v = m[i * cols + j];
                for (int k = 0; k < 8; ++k) buf[8 * i + k] = (uint8_t)(v >> (8 * k));
            }
            or_blake3(buf, rows * 8, leaves + 32 * j);
        }
        free(buf);
    }
}

void or_hash_fp2_columns(const ofp2* m, size_t rows, size_t cols, uint8_t* leaves) {
#pragma omp parallel
    {
        uint8_t* buf = (uint8_t*)malloc(rows * 16);
#pragma omp for schedule(static)
        for (size_t j = 0; j < cols; ++j) {
            for (size_t i = 0; i < rows; ++i) {
                ofp2 v = m[i * cols + j];
                for (int k = 0; k < 8; ++k) {
                    buf[16 * i + k] = (uint8_t)(v.c0 >> (8 * k));
                    buf[16 * i + 8 + k] = (uint8_t)(v.c1 >> (8 * k));
                }
            }
            or_blake3(buf, rows * 16, leaves + 32 * j);
        }
        free(buf);
    }
}

void or_merkle_tree(const uint8_t* leaves, size_t n, uint8_t* tree) {
    memcpy(tree, leaves, n * 32);
    size_t off = 0, len = n;
    while (len > 1) {
        size_t parent = len / 2;
#pragma omp parallel for schedule(static)
        for (size_t i = 0; i < parent; ++i) {
            uint8_t buf[64];
            memcpy(buf, tree + 32 * (off + 2 * i), 64);
            or_blake3(buf, 64, tree + 32 * (off + len + i));
        }
        off += len;
        len = parent;
    }
}

void or_merkle_paths(const uint8_t* tree, size_t leaves, const uint32_t* idx, size_t q,
                     uint8_t* paths) {
    size_t bits = 0;
    while (((size_t)1 << bits) < leaves) ++bits;
    for (size_t k = 0; k < q; ++k) {
        size_t i = idx[k], off = 0, len = leaves;
        for (size_t level = 0; level < bits; ++level) {
            memcpy(paths + 32 * (k * bits + level), tree + 32 * (off + (i ^ 1)), 32);
            off += len;
            len /= 2;
            i >>= 1;
        }
    }
}

/* ------------------------------------------------------------------ */
/* PCS rows                                                             */
/* ------------------------------------------------------------------ */

void or_pcs_messages(const int16_t* w, const uint64_t* pads, size_t rows, size_t cols,
                     size_t pad, size_t code_len, uint64_t* out) {
    for (size_t r = 0; r < rows; ++r)
        for (size_t j = 0; j < code_len; ++j) {
            uint64_t v = 0;
            if (j < cols)
                v = embed_i64(w[r * cols + j]);
            else if (j < cols + pad)
                v = pads[r * pad + (j - cols)];
            out[r * code_len + j] = v;
        }
}

void or_pcs_combine_rows(const int16_t* w, const uint64_t* pads, const ofp2* coeffs,
                         size_t rows, size_t cols, size_t pad, size_t combos, ofp2* out) {
    size_t msg = cols + pad;
#pragma omp parallel for schedule(static)
    for (size_t z = 0; z < combos * msg; ++z) {
        size_t k = z / msg, j = z % msg;
        ofp2 acc = {0, 0};
        for (size_t r = 0; r < rows; ++r) {
            uint64_t v = j < cols ? embed_i64(w[r * cols + j]) : pads[r * pad + (j - cols)];
            ofp2 c = coeffs[k * rows + r];
            ofp2 t = {or_fp_mul(c.c0, v), or_fp_mul(c.c1, v)};
            acc = or_fp2_add(acc, t);
        }
        out[z] = acc;
    }
}

/* ------------------------------------------------------------------ */
/* GEMM + requant + MAC correction                                      */
/* ------------------------------------------------------------------ */

void or_gemm_i64(const int16_t* a, const int16_t* b, int64_t* out, size_t m, size_t k,
                 size_t n) {
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < m; ++i)
        for (size_t j = 0; j < n; ++j) {
            int64_t acc = 0;
            for (size_t q = 0; q < k; ++q) acc += (int64_t)a[i * k + q] * (int64_t)b[q * n + j];
            out[i * n + j] = acc;
        }
}

void or_gemm_requant_auth(const int16_t* a, const int16_t* b, const uint64_t* masks,
                          int16_t* out, uint64_t* corr, size_t m, size_t k, size_t n,
                          uint32_t shift) {
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < m; ++i)
        for (size_t j = 0; j < n; ++j) {
            int64_t acc = 0;
            for (size_t q = 0; q < k; ++q) acc += (int64_t)a[i * k + q] * (int64_t)b[q * n + j];
            /* round half up then clamp to i16 (gemm.rs:19-22) */
            int64_t y = (acc + ((int64_t)1 << (shift - 1))) >> shift;
            if (y > 32767) y = 32767;
            if (y < -32768) y = -32768;
            size_t z = i * n + j;
            out[z] = (int16_t)y;
            corr[z] = or_fp_sub(embed_i64(y), masks[z]);
        }
}
