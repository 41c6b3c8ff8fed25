/*
 * Oracle (test infrastructure only): sumcheck round evaluations, folds,
 * LogUp fraction tree, eq tables and the clear protocol drivers.
 *
 * References (okrame/volta-zk):
 *   product round    rust/volta-proto/src/sumcheck_clear.rs:33-45,
 *                    rust/volta-accel/src/lib.rs:3647-3679 (CPU branch)
 *   triple round     rust/volta-proto/src/hadamard.rs:222-240 (g(0),g(2),g(3))
 *   LogUp round      rust/volta-proto/src/logup.rs:409-472 (run_general_rounds)
 *   folds            logup.rs:474-500, rust/volta-proto/src/mle.rs:23-30
 *   tree             logup.rs:169-240 (build_tree_cpu), flattened root-to-leaf
 *                    as rust/volta-accel/src/lib.rs:5511-5513 describes
 *   suffix eq        logup.rs:284-305
 *   eq rows          mle.rs:7-20 (eq_vec), one table per row
 *   aux round        logup.rs:740-900 (layer_leaf_ones_aux), per-pair form
 *   logup_prove      logup.rs:1472-1545, 1624-1640, 1760-1771
 *   matrix fold      rust/volta-accel/src/lib.rs:2968-3035 (CPU semantics)
 */
#include "oracle.h"

#include <stdlib.h>
#include <string.h>

#define P_GOLD 0xFFFFFFFF00000001ULL

static ofp2 Z2(void) {
    ofp2 z = {0, 0};
    return z;
}
static ofp2 ONE2(void) {
    ofp2 o = {1, 0};
    return o;
}
static ofp2 mk(uint64_t a, uint64_t b) {
    ofp2 r = {a, b};
    return r;
}
#define ADD or_fp2_add
#define SUB or_fp2_sub
#define MUL or_fp2_mul

/* v0 + t (v1 - v0) at t = 2, 3 */
static ofp2 at2(ofp2 v0, ofp2 v1) {
    ofp2 d = SUB(v1, v0);
    return ADD(ADD(v0, d), d);
}
static ofp2 at3(ofp2 v0, ofp2 v1) {
    ofp2 d = SUB(v1, v0);
    return ADD(ADD(ADD(v0, d), d), d);
}

void or_product_round(const ofp2* a, const ofp2* b, size_t pairs, ofp2 out[2]) {
    ofp2 g0 = Z2(), g2 = Z2();
    for (size_t i = 0; i < pairs; ++i) {
        g0 = ADD(g0, MUL(a[2 * i], b[2 * i]));
        g2 = ADD(g2, MUL(at2(a[2 * i], a[2 * i + 1]), at2(b[2 * i], b[2 * i + 1])));
    }
    out[0] = g0;
    out[1] = g2;
}

void or_triple_product_round(const ofp2* a, const ofp2* b, const ofp2* c, size_t pairs,
                             ofp2 out[3]) {
    ofp2 g0 = Z2(), g2 = Z2(), g3 = Z2();
#pragma omp parallel
    {
        ofp2 l0 = Z2(), l2 = Z2(), l3 = Z2();
#pragma omp for schedule(static)
        for (size_t i = 0; i < pairs; ++i) {
            ofp2 a0 = a[2 * i], a1 = a[2 * i + 1];
            ofp2 b0 = b[2 * i], b1 = b[2 * i + 1];
            ofp2 c0 = c[2 * i], c1 = c[2 * i + 1];
            l0 = ADD(l0, MUL(MUL(a0, b0), c0));
            l2 = ADD(l2, MUL(MUL(at2(a0, a1), at2(b0, b1)), at2(c0, c1)));
            l3 = ADD(l3, MUL(MUL(at3(a0, a1), at3(b0, b1)), at3(c0, c1)));
        }
#pragma omp critical
        {
            g0 = ADD(g0, l0);
            g2 = ADD(g2, l2);
            g3 = ADD(g3, l3);
        }
    }
    out[0] = g0;
    out[1] = g2;
    out[2] = g3;
}

void or_logup_general_round(const ofp2* p0, const ofp2* p1, const ofp2* q0, const ofp2* q1,
                            const ofp2* s, size_t pairs, ofp2 out[4]) {
    ofp2 t0 = Z2(), t1 = Z2(), t2 = Z2(), t3 = Z2();
#pragma omp parallel
    {
        ofp2 l0 = Z2(), l1 = Z2(), l2 = Z2(), l3 = Z2();
#pragma omp for schedule(static)
        for (size_t i = 0; i < pairs; ++i) {
            ofp2 a0 = p0[2 * i], a2 = at2(a0, p0[2 * i + 1]);
            ofp2 b0 = p1[2 * i], b2 = at2(b0, p1[2 * i + 1]);
            ofp2 c0 = q0[2 * i], c2 = at2(c0, q0[2 * i + 1]);
            ofp2 d0 = q1[2 * i], d2 = at2(d0, q1[2 * i + 1]);
            l0 = ADD(l0, MUL(s[i], ADD(MUL(a0, d0), MUL(b0, c0))));
            l1 = ADD(l1, MUL(s[i], ADD(MUL(a2, d2), MUL(b2, c2))));
            l2 = ADD(l2, MUL(s[i], MUL(c0, d0)));
            l3 = ADD(l3, MUL(s[i], MUL(c2, d2)));
        }
#pragma omp critical
        {
            t0 = ADD(t0, l0);
            t1 = ADD(t1, l1);
            t2 = ADD(t2, l2);
            t3 = ADD(t3, l3);
        }
    }
    out[0] = t0;
    out[1] = t1;
    out[2] = t2;
    out[3] = t3;
}

void or_fold_rows(const ofp2* in, size_t rows, size_t len, ofp2 r, ofp2* out) {
    size_t half = len / 2;
#pragma omp parallel for schedule(static)
    for (size_t z = 0; z < rows * half; ++z) {
        size_t row = z / half, i = z % half;
        const ofp2* src = in + row * len;
        out[z] = ADD(src[2 * i], MUL(SUB(src[2 * i + 1], src[2 * i]), r));
    }
}

/* Flattened tree: level k (2^k nodes) at offset 2^k - 1; level depth-1 is
 * the first combine of the leaves. */
void or_logup_tree(const uint64_t* leaf, const uint32_t* mult, size_t n, uint64_t alpha1,
                   int neg_mult, ofp2* p, ofp2* q) {
    size_t half = n / 2;
    uint64_t w7a1sq = or_fp_mul(7, or_fp_mul(alpha1, alpha1));
    size_t off = half - 1;
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < half; ++i) {
        uint64_t a = leaf[2 * i], b = leaf[2 * i + 1];
        uint64_t sum = or_fp_add(a, b);
        if (neg_mult) {
            uint64_t ma = mult[2 * i], mb = mult[2 * i + 1];
            uint64_t x = or_fp_add(or_fp_mul(ma, b), or_fp_mul(mb, a));
            uint64_t y = or_fp_mul(or_fp_add(ma, mb), alpha1);
            p[off + i] = mk(or_fp_sub(0, x), or_fp_sub(0, y));
        } else {
            p[off + i] = mk(sum, or_fp_add(alpha1, alpha1));
        }
        q[off + i] = mk(or_fp_add(or_fp_mul(a, b), w7a1sq), or_fp_mul(sum, alpha1));
    }
    size_t len = half;
    while (len > 1) {
        size_t parent = len / 2;
        size_t coff = len - 1, poff = parent - 1;
#pragma omp parallel for schedule(static)
        for (size_t i = 0; i < parent; ++i) {
            ofp2 pa = p[coff + 2 * i], pb = p[coff + 2 * i + 1];
            ofp2 qa = q[coff + 2 * i], qb = q[coff + 2 * i + 1];
            p[poff + i] = ADD(MUL(pa, qb), MUL(pb, qa));
            q[poff + i] = MUL(qa, qb);
        }
        len = parent;
    }
}

void or_materialize_leaves(const uint64_t* leaf, const uint32_t* mult, size_t n,
                           uint64_t alpha1, int neg_mult, ofp2* p, ofp2* q) {
    for (size_t i = 0; i < n; ++i) {
        p[i] = neg_mult ? mk(or_fp_sub(0, (uint64_t)mult[i]), 0) : ONE2();
        q[i] = mk(leaf[i], alpha1);
    }
}

/* Flat suffix tables: table j (eq over point[j+1..], 2^(L-1-j) entries)
 * starts at offset 2^(L-1-j) - 1. */
void or_suffix_eq(const ofp2* point, size_t L, ofp2* out) {
    out[0] = ONE2();
    size_t size = 1;
    for (size_t j = L - 1; j > 0; --j) {
        const ofp2* in = out + size - 1;
        ofp2* o = out + 2 * size - 1;
        for (size_t i = 0; i < size; ++i) {
            ofp2 v1 = MUL(in[i], point[j]);
            o[2 * i] = SUB(in[i], v1);
            o[2 * i + 1] = v1;
        }
        size *= 2;
    }
}

void or_eq_vec(const ofp2* point, size_t len, ofp2* out) {
    out[0] = ONE2();
    size_t size = 1;
    ofp2* tmp = (ofp2*)malloc(sizeof(ofp2) << len);
    for (size_t k = len; k-- > 0;) {
        for (size_t i = 0; i < size; ++i) {
            ofp2 v1 = MUL(out[i], point[k]);
            tmp[2 * i] = SUB(out[i], v1);
            tmp[2 * i + 1] = v1;
        }
        size *= 2;
        memcpy(out, tmp, size * sizeof(ofp2));
    }
    free(tmp);
}

void or_eq_rows(const ofp2* points, size_t rows, size_t dims, ofp2* out) {
    size_t width = (size_t)1 << dims;
    for (size_t r = 0; r < rows; ++r) or_eq_vec(points + r * dims, dims, out + r * width);
}

void or_aux_round(const ofp2* q0, const ofp2* q1, const ofp2* suffix, const ofp2* columns,
                  const ofp2* eq_rows, const uint32_t* claim_cols, const ofp2* weights,
                  size_t column_count, size_t claim_count, size_t vector_len, ofp2 lambda,
                  ofp2 cpref, ofp2 point, ofp2 out[3]) {
    size_t pairs = vector_len / 2;
    ofp2 pq[3] = {Z2(), Z2(), Z2()}, qq[3] = {Z2(), Z2(), Z2()}, aux[3] = {Z2(), Z2(), Z2()};
    for (size_t i = 0; i < pairs; ++i) {
        ofp2 c[3] = {q0[2 * i], at2(q0[2 * i], q0[2 * i + 1]), at3(q0[2 * i], q0[2 * i + 1])};
        ofp2 d[3] = {q1[2 * i], at2(q1[2 * i], q1[2 * i + 1]), at3(q1[2 * i], q1[2 * i + 1])};
        ofp2 s = suffix[i];
        for (int t = 0; t < 3; ++t) {
            pq[t] = ADD(pq[t], MUL(s, ADD(c[t], d[t])));
            qq[t] = ADD(qq[t], MUL(s, MUL(c[t], d[t])));
        }
        for (size_t k = 0; k < claim_count; ++k) {
            size_t col = claim_cols[k];
            if (col >= column_count) continue;
            const ofp2* v0 = columns + (2 * col) * vector_len;
            const ofp2* v1 = columns + (2 * col + 1) * vector_len;
            const ofp2* e = eq_rows + k * vector_len;
            ofp2 w0 = weights[2 * k], w1 = weights[2 * k + 1];
            ofp2 a[3] = {v0[2 * i], at2(v0[2 * i], v0[2 * i + 1]), at3(v0[2 * i], v0[2 * i + 1])};
            ofp2 b[3] = {v1[2 * i], at2(v1[2 * i], v1[2 * i + 1]), at3(v1[2 * i], v1[2 * i + 1])};
            ofp2 ee[3] = {e[2 * i], at2(e[2 * i], e[2 * i + 1]), at3(e[2 * i], e[2 * i + 1])};
            for (int t = 0; t < 3; ++t)
                aux[t] = ADD(aux[t], MUL(ee[t], ADD(MUL(w0, a[t]), MUL(w1, b[t]))));
        }
    }
    /* ell(t) = eq(point, t) at t = 0, 2, 3: 1 - p, 3p - 1, 5p - 2 */
    ofp2 p = point;
    ofp2 l0 = SUB(ONE2(), p);
    ofp2 l2 = SUB(ADD(ADD(p, p), p), ONE2());
    ofp2 l3 = SUB(ADD(ADD(ADD(p, p), ADD(p, p)), p), mk(2, 0));
    ofp2 ell[3] = {l0, l2, l3};
    for (int t = 0; t < 3; ++t)
        out[t] = ADD(MUL(ell[t], MUL(cpref, ADD(MUL(lambda, pq[t]), qq[t]))), aux[t]);
}

static uint64_t load_base(const void* in, size_t idx, int kind) {
    switch (kind) {
        case 0: { /* i16 */
            int64_t v = ((const int16_t*)in)[idx];
            return v >= 0 ? (uint64_t)v : P_GOLD - (uint64_t)(-v);
        }
        case 1: { /* i64 */
            int64_t v = ((const int64_t*)in)[idx];
            return v >= 0 ? (uint64_t)v : P_GOLD - (uint64_t)(-v);
        }
        case 4: /* u32 */
            return ((const uint32_t*)in)[idx];
        default: /* canonical Fp */
            return ((const uint64_t*)in)[idx];
    }
}

void or_matrix_fold(const void* input, const ofp2* weights, size_t rows, size_t stride,
                    size_t column_offset, size_t cols, size_t out_pad, int kind, int axis,
                    ofp2* out) {
    size_t real = axis == 0 ? cols : rows;
    size_t terms = axis == 0 ? rows : cols;
#pragma omp parallel for schedule(static)
    for (size_t o = 0; o < out_pad; ++o) {
        ofp2 acc = Z2();
        if (o < real) {
            for (size_t t = 0; t < terms; ++t) {
                size_t idx = axis == 0 ? t * stride + column_offset + o
                                       : o * stride + column_offset + t;
                ofp2 v;
                if (kind == 3) {
                    v = ((const ofp2*)input)[idx];
                } else {
                    v = mk(load_base(input, idx, kind), 0);
                }
                acc = ADD(acc, MUL(weights[t], v));
            }
        }
        out[o] = acc;
    }
}

/* ------------------------------------------------------------------ */
/* Protocol drivers                                                     */
/* ------------------------------------------------------------------ */

void or_triple_sumcheck(ofp2* a, ofp2* b, ofp2* c, size_t n, const uint8_t chal_seed[32],
                        ofp2* messages, ofp2* finals) {
    or_stream tx;
    or_stream_init(&tx, chal_seed, UINT64_MAX);
    size_t len = n, round = 0;
    ofp2* tmp = (ofp2*)malloc(sizeof(ofp2) * (n / 2 + 1));
    while (len > 1) {
        size_t pairs = len / 2;
        or_triple_product_round(a, b, c, pairs, messages + 3 * round);
        ofp2 r = or_stream_next_fp2(&tx);
        ofp2* v[3] = {a, b, c};
        for (int k = 0; k < 3; ++k) {
            or_fold_rows(v[k], 1, len, r, tmp);
            memcpy(v[k], tmp, pairs * sizeof(ofp2));
        }
        len = pairs;
        ++round;
    }
    free(tmp);
    finals[0] = a[0];
    finals[1] = b[0];
    finals[2] = c[0];
}

/* One fraction tree, clear sink (logup.rs:1472-1545 + 1624-1640).  Leaf
 * layers use the materialised general form; the leaf-layer specialisations
 * of the reference are algebraic rewrites of the same sums. */
static size_t prove_frac_tree(const uint64_t* leaf_a, const uint32_t* mult, size_t n,
                              uint64_t alpha1, or_stream* chal, ofp2* out) {
    size_t w = 0;
    int neg = mult != NULL;
    size_t depth = 0;
    while (((size_t)1 << depth) < n) ++depth;
    ofp2* tp = (ofp2*)malloc(sizeof(ofp2) * (n - 1));
    ofp2* tq = (ofp2*)malloc(sizeof(ofp2) * (n - 1));
    or_logup_tree(leaf_a, mult, n, alpha1, neg, tp, tq);
    out[w++] = tp[0];
    out[w++] = tq[0];
    ofp2* lp = (ofp2*)malloc(sizeof(ofp2) * n);
    ofp2* lq = (ofp2*)malloc(sizeof(ofp2) * n);
    or_materialize_leaves(leaf_a, mult, n, alpha1, neg, lp, lq);
    ofp2* point = (ofp2*)malloc(sizeof(ofp2) * (depth + 1));
    ofp2* npoint = (ofp2*)malloc(sizeof(ofp2) * (depth + 1));
    size_t L = 0;
    size_t vcap = n / 2;
    ofp2* v[4];
    for (int k = 0; k < 4; ++k) v[k] = (ofp2*)malloc(sizeof(ofp2) * vcap);
    ofp2* tmp = (ofp2*)malloc(sizeof(ofp2) * vcap);
    ofp2* suffix = (ofp2*)malloc(sizeof(ofp2) * (vcap > 0 ? vcap : 1));
    for (size_t l = 0; l < depth; ++l) {
        size_t child_len = (size_t)1 << (l + 1);
        const ofp2 *cp, *cq;
        if (l + 1 == depth) {
            cp = lp;
            cq = lq;
        } else {
            cp = tp + (child_len - 1);
            cq = tq + (child_len - 1);
        }
        size_t vl = child_len / 2;
        for (size_t i = 0; i < vl; ++i) {
            v[0][i] = cp[2 * i];
            v[1][i] = cp[2 * i + 1];
            v[2][i] = cq[2 * i];
            v[3][i] = cq[2 * i + 1];
        }
        ofp2 lambda = or_stream_next_fp2(chal);
        ofp2 cpref = ONE2();
        if (L > 0) or_suffix_eq(point, L, suffix);
        size_t len = vl;
        for (size_t j = 0; j < L; ++j) {
            size_t half = len / 2;
            size_t soff = ((size_t)1 << (L - 1 - j)) - 1;
            ofp2 acc[4];
            or_logup_general_round(v[0], v[1], v[2], v[3], suffix + soff, half, acc);
            ofp2 h0 = MUL(cpref, ADD(MUL(lambda, acc[0]), acc[2]));
            ofp2 h2 = MUL(cpref, ADD(MUL(lambda, acc[1]), acc[3]));
            out[w++] = h0;
            out[w++] = h2;
            ofp2 r = or_stream_next_fp2(chal);
            for (int k = 0; k < 4; ++k) {
                or_fold_rows(v[k], 1, len, r, tmp);
                memcpy(v[k], tmp, half * sizeof(ofp2));
            }
            ofp2 pj = point[j];
            ofp2 pr = MUL(pj, r);
            cpref = MUL(cpref, ADD(SUB(SUB(ADD(pr, pr), pj), r), ONE2()));
            npoint[1 + j] = r;
            len = half;
        }
        for (int k = 0; k < 4; ++k) out[w++] = v[k][0];
        ofp2 t = or_stream_next_fp2(chal);
        npoint[0] = t;
        L = L + 1;
        memcpy(point, npoint, L * sizeof(ofp2));
    }
    for (int k = 0; k < 4; ++k) free(v[k]);
    free(tmp);
    free(suffix);
    free(point);
    free(npoint);
    free(lp);
    free(lq);
    free(tp);
    free(tq);
    return w;
}

size_t or_logup_prove(const int16_t* f, size_t n_f, const int16_t* table, size_t n_t,
                      const uint32_t* mult, const uint8_t chal_seed[32], uint64_t chal_domain,
                      ofp2* out, size_t out_cap) {
    (void)out_cap;
    or_stream chal;
    or_stream_init(&chal, chal_seed, chal_domain);
    ofp2 alpha = or_stream_next_fp2(&chal);
    size_t w = 0;
    out[w++] = alpha;
    uint64_t* a = (uint64_t*)malloc(sizeof(uint64_t) * (n_f > n_t ? n_f : n_t));
    for (size_t i = 0; i < n_f; ++i) {
        int64_t v = f[i];
        uint64_t x = v >= 0 ? (uint64_t)v : P_GOLD - (uint64_t)(-v);
        a[i] = or_fp_sub(alpha.c0, x);
    }
    w += prove_frac_tree(a, NULL, n_f, alpha.c1, &chal, out + w);
    for (size_t i = 0; i < n_t; ++i) {
        int64_t v = table[i];
        uint64_t x = v >= 0 ? (uint64_t)v : P_GOLD - (uint64_t)(-v);
        a[i] = or_fp_sub(alpha.c0, x);
    }
    w += prove_frac_tree(a, mult, n_t, alpha.c1, &chal, out + w);
    free(a);
    return w;
}

/* The same proof over canonical Fp query and table columns (packed pair
 * values in + 2^k out, range remainders): logup.rs:1760-1771 with the
 * columns already embedded in Fp (rust/volta-proto/src/block_proof.rs
 * range_table / pair_table, range_cols_padded / pair_cols_padded). */
size_t or_logup_prove_fp(const uint64_t* f, size_t n_f, const uint64_t* table, size_t n_t,
                         const uint32_t* mult, const uint8_t chal_seed[32], uint64_t chal_domain,
                         ofp2* out, size_t out_cap) {
    (void)out_cap;
    or_stream chal;
    or_stream_init(&chal, chal_seed, chal_domain);
    ofp2 alpha = or_stream_next_fp2(&chal);
    size_t w = 0;
    out[w++] = alpha;
    uint64_t* a = (uint64_t*)malloc(sizeof(uint64_t) * (n_f > n_t ? n_f : n_t));
    for (size_t i = 0; i < n_f; ++i) a[i] = or_fp_sub(alpha.c0, f[i]);
    w += prove_frac_tree(a, NULL, n_f, alpha.c1, &chal, out + w);
    for (size_t i = 0; i < n_t; ++i) a[i] = or_fp_sub(alpha.c0, table[i]);
    w += prove_frac_tree(a, mult, n_t, alpha.c1, &chal, out + w);
    free(a);
    return w;
}
