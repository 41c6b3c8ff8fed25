// Sumcheck round engine: product / triple-product / LogUp round messages,
// multilinear folds, eq tables and the small Fp2 vector primitives of the
// seam.
//
// Reference entry points (okrame/volta-zk cuda/volta_cuda_backend.cu):
//   fp2_product_round{,_into,_scaled_into}_device   4827-4893
//   fp2_triple_product_round{,_into}_device         5106-5153
//   logup_general_round{,_device,_into_device}      6655-6769
//   logup_fold4{,_device}                           6771-6808
//   fp2_deinterleave_device                         6810-6831
//   logup_suffix_eq_device                          6833-6860
//   fp2_fold_rows_device                            6862-6882
//   logup_eq_rows_device                            6884-6918
//   logup_aux_round{,_into}_device                  7008-7062
//   fp2_dot_device, fp2_dot_scaled_pair_into_device, fp2_pair_sum_device
//                                                   4715-4746, 5001-5069
//   claim_reduce_f_two_into_device, x4d_link_eq_accumulate_device 4895-4999
//   fp2_add_inplace / mobius_inverse / affine_eq_weights 7101-7149
//   fp2_row_dots_device, fp2_powers_device          4049-4126
//   reserve_*_workspace                             4748-4785
// CPU semantics: rust/volta-proto/src/logup.rs:284-500, hadamard.rs:222-240,
// sumcheck_clear.rs:33-45, mle.rs:7-30.
#include "reduce.cuh"
#include "runtime.cuh"

#include <algorithm>

namespace vzb {

// ---------------------------------------------------------------------------
// evaluation functors (one per message shape)
// ---------------------------------------------------------------------------

// The round evaluations accumulate the last product of each term lazily
// (Fp2W: unreduced 128-bit products), so each pair pays one canonical
// reduction per inner product only.  at2 = v1 + (v1 - v0) and
// at3 = at2 + (v1 - v0) are formed as "weak" values (< 2^64), which the
// products accept.

struct ProductEval {  // [g(0), g(2)] of a*b
    const Fp2 *a, *b;
    __device__ __forceinline__ void operator()(size_t i, Fp2W* w) const {
        const Fp2 a0 = ldcs2(a + 2 * i), a1 = ldcs2(a + 2 * i + 1);
        const Fp2 b0 = ldcs2(b + 2 * i), b1 = ldcs2(b + 2 * i + 1);
        f2w_mac(w[0], a0, b0);
        f2w_mac(w[1], d2add_weak(a1, d2sub(a1, a0)), d2add_weak(b1, d2sub(b1, b0)));
    }
};

struct TripleEval {  // [g(0), g(2), g(3)] of a*b*c
    const Fp2 *a, *b, *c;
    __device__ __forceinline__ void operator()(size_t i, Fp2W* w) const {
        const Fp2 a0 = ldcs2(a + 2 * i), a1 = ldcs2(a + 2 * i + 1);
        const Fp2 b0 = ldcs2(b + 2 * i), b1 = ldcs2(b + 2 * i + 1);
        const Fp2 c0 = ldcs2(c + 2 * i), c1 = ldcs2(c + 2 * i + 1);
        const Fp2 da = d2sub(a1, a0), db = d2sub(b1, b0), dc = d2sub(c1, c0);
        const Fp2 a2 = d2add_weak(a1, da), b2 = d2add_weak(b1, db), c2 = d2add_weak(c1, dc);
        const Fp2 a3 = d2add_weak(a2, da), b3 = d2add_weak(b2, db), c3 = d2add_weak(c2, dc);
        f2w_mac(w[0], d2mul(a0, b0), c0);
        f2w_mac(w[1], d2mul(a2, b2), c2);
        f2w_mac(w[2], d2mul(a3, b3), c3);
    }
};

// RoundAcc = sum_i S[i] * (a0 d0 + b0 c0, a2 d2 + b2 c2, c0 d0, c2 d2)
struct LogupEval {
    const Fp2 *p0, *p1, *q0, *q1, *s;
    __device__ __forceinline__ void operator()(size_t i, Fp2W* w) const {
        const Fp2 a0 = ldcs2(p0 + 2 * i), a1 = ldcs2(p0 + 2 * i + 1);
        const Fp2 b0 = ldcs2(p1 + 2 * i), b1 = ldcs2(p1 + 2 * i + 1);
        const Fp2 c0 = ldcs2(q0 + 2 * i), c1 = ldcs2(q0 + 2 * i + 1);
        const Fp2 d0 = ldcs2(q1 + 2 * i), d1 = ldcs2(q1 + 2 * i + 1);
        const Fp2 si = ldg2(s + i);
        const Fp2 a2 = d2add_weak(a1, d2sub(a1, a0)), b2 = d2add_weak(b1, d2sub(b1, b0));
        const Fp2 c2 = d2add_weak(c1, d2sub(c1, c0)), d2 = d2add_weak(d1, d2sub(d1, d0));
        Fp2W t;
        f2w_zero(t);
        f2w_mac(t, a0, d0);
        f2w_mac(t, b0, c0);
        f2w_mac(w[0], si, f2w_reduce(t));
        f2w_zero(t);
        f2w_mac(t, a2, d2);
        f2w_mac(t, b2, c2);
        f2w_mac(w[1], si, f2w_reduce(t));
        f2w_mac(w[2], si, d2mul(c0, d0));
        f2w_mac(w[3], si, d2mul(c2, d2));
    }
};

// Fused fold + next round.  Round j's challenge r folds the current vectors
// (len entries) into fresh half-length vectors and, in the same pass,
// evaluates round j + 1 on the folded values: item i reads entries 4i..4i+3,
// writes folded entries 2i, 2i+1 and accumulates the pair (2i, 2i+1).
// This halves the launches per round and skips re-reading the folded
// vectors.
__device__ __forceinline__ void fold4_pair(const Fp2* in, Fp2* out, size_t i, Fp2 r, Fp2& x0, Fp2& x1) {
    const Fp2 v0 = ldcs2(in + 4 * i), v1 = ldcs2(in + 4 * i + 1);
    const Fp2 v2 = ldcs2(in + 4 * i + 2), v3 = ldcs2(in + 4 * i + 3);
    x0 = d2fold(v0, v1, r);
    x1 = d2fold(v2, v3, r);
    st2(out + 2 * i, x0);
    st2(out + 2 * i + 1, x1);
}

struct TripleFoldEval {
    const Fp2 *a, *b, *c;
    Fp2 *ao, *bo, *co;
    Fp2 r;
    __device__ __forceinline__ void operator()(size_t i, Fp2W* w) const {
        Fp2 a0, a1, b0, b1, c0, c1;
        fold4_pair(a, ao, i, r, a0, a1);
        fold4_pair(b, bo, i, r, b0, b1);
        fold4_pair(c, co, i, r, c0, c1);
        const Fp2 da = d2sub(a1, a0), db = d2sub(b1, b0), dc = d2sub(c1, c0);
        const Fp2 a2 = d2add_weak(a1, da), b2 = d2add_weak(b1, db), c2 = d2add_weak(c1, dc);
        const Fp2 a3 = d2add_weak(a2, da), b3 = d2add_weak(b2, db), c3 = d2add_weak(c2, dc);
        f2w_mac(w[0], d2mul(a0, b0), c0);
        f2w_mac(w[1], d2mul(a2, b2), c2);
        f2w_mac(w[2], d2mul(a3, b3), c3);
    }
};

// Fused fold + next product round: fold a, b (len entries) with r into
// half-length vectors and accumulate the next round's [g(0), g(2)].
struct ProductFoldEval {
    const Fp2 *a, *b;
    Fp2 *ao, *bo;
    Fp2 r;
    __device__ __forceinline__ void operator()(size_t i, Fp2W* w) const {
        Fp2 a0, a1, b0, b1;
        fold4_pair(a, ao, i, r, a0, a1);
        fold4_pair(b, bo, i, r, b0, b1);
        f2w_mac(w[0], a0, b0);
        f2w_mac(w[1], d2add_weak(a1, d2sub(a1, a0)), d2add_weak(b1, d2sub(b1, b0)));
    }
};

// Round 0 of a triple product over base-field tables (Fp values, i.e. Fp2
// values with c1 = 0): the products stay in Fp (two base products per point
// instead of two Fp2 products) and the message has c1 = 0.
struct TripleEvalFp {
    const uint64_t *a, *b, *c;
    __device__ __forceinline__ void operator()(size_t i, Fp2W* w) const {
        const uint64_t a0 = __ldcs(a + 2 * i), a1 = __ldcs(a + 2 * i + 1);
        const uint64_t b0 = __ldcs(b + 2 * i), b1 = __ldcs(b + 2 * i + 1);
        const uint64_t c0 = __ldcs(c + 2 * i), c1 = __ldcs(c + 2 * i + 1);
        const uint64_t da = dsub(a1, a0), db = dsub(b1, b0), dc = dsub(c1, c0);
        const uint64_t a2 = dadd_weak(a1, da), b2 = dadd_weak(b1, db), c2 = dadd_weak(c1, dc);
        const uint64_t a3 = dadd_weak(a2, da), b3 = dadd_weak(b2, db), c3 = dadd_weak(c2, dc);
        wadd(w[0].c0, dmul_wide(dmul(a0, b0), c0));
        wadd(w[1].c0, dmul_wide(dmul(a2, b2), c2));
        wadd(w[2].c0, dmul_wide(dmul(a3, b3), c3));
    }
};

// Fold of a base-field pair with an Fp2 challenge: x0 + r (x1 - x0) =
// (x0 + r.c0 d, r.c1 d), d = x1 - x0 in Fp.
__device__ __forceinline__ Fp2 fold_fp(uint64_t x0, uint64_t x1, Fp2 r) {
    const uint64_t d = dsub(x1, x0);
    return Fp2{dadd(x0, dmul(r.c0, d)), dmul(r.c1, d)};
}

// Fold of base-field tables into Fp2 tables fused with the next round (as
// TripleFoldEval; inputs 4i .. 4i + 3, outputs 2i, 2i + 1).
struct TripleFoldEvalFp {
    const uint64_t *a, *b, *c;
    Fp2 *ao, *bo, *co;
    Fp2 r;
    __device__ __forceinline__ void fold(const uint64_t* in, Fp2* out, size_t i, Fp2& x0, Fp2& x1) const {
        const uint64_t v0 = __ldcs(in + 4 * i), v1 = __ldcs(in + 4 * i + 1);
        const uint64_t v2 = __ldcs(in + 4 * i + 2), v3 = __ldcs(in + 4 * i + 3);
        x0 = fold_fp(v0, v1, r);
        x1 = fold_fp(v2, v3, r);
        st2(out + 2 * i, x0);
        st2(out + 2 * i + 1, x1);
    }
    __device__ __forceinline__ void operator()(size_t i, Fp2W* w) const {
        Fp2 a0, a1, b0, b1, c0, c1;
        fold(a, ao, i, a0, a1);
        fold(b, bo, i, b0, b1);
        fold(c, co, i, c0, c1);
        const Fp2 da = d2sub(a1, a0), db = d2sub(b1, b0), dc = d2sub(c1, c0);
        const Fp2 a2 = d2add_weak(a1, da), b2 = d2add_weak(b1, db), c2 = d2add_weak(c1, dc);
        const Fp2 a3 = d2add_weak(a2, da), b3 = d2add_weak(b2, db), c3 = d2add_weak(c2, dc);
        f2w_mac(w[0], d2mul(a0, b0), c0);
        f2w_mac(w[1], d2mul(a2, b2), c2);
        f2w_mac(w[2], d2mul(a3, b3), c3);
    }
};

struct LogupFoldEval {
    const Fp2 *p0, *p1, *q0, *q1, *s;
    Fp2 *o0, *o1, *o2, *o3;
    Fp2 r;
    __device__ __forceinline__ void operator()(size_t i, Fp2W* w) const {
        Fp2 a0, a1, b0, b1, c0, c1, d0, d1;
        fold4_pair(p0, o0, i, r, a0, a1);
        fold4_pair(p1, o1, i, r, b0, b1);
        fold4_pair(q0, o2, i, r, c0, c1);
        fold4_pair(q1, o3, i, r, d0, d1);
        const Fp2 si = ldg2(s + i);
        const Fp2 a2 = d2add_weak(a1, d2sub(a1, a0)), b2 = d2add_weak(b1, d2sub(b1, b0));
        const Fp2 c2 = d2add_weak(c1, d2sub(c1, c0)), d2 = d2add_weak(d1, d2sub(d1, d0));
        Fp2W t;
        f2w_zero(t);
        f2w_mac(t, a0, d0);
        f2w_mac(t, b0, c0);
        f2w_mac(w[0], si, f2w_reduce(t));
        f2w_zero(t);
        f2w_mac(t, a2, d2);
        f2w_mac(t, b2, c2);
        f2w_mac(w[1], si, f2w_reduce(t));
        f2w_mac(w[2], si, d2mul(c0, d0));
        f2w_mac(w[3], si, d2mul(c2, d2));
    }
};

// The same two evaluations read straight from interleaved fraction-tree
// children (p0 = P[2k], p1 = P[2k+1], q0 = Q[2k], q1 = Q[2k+1]): the
// deinterleave pass of the reference's layer setup (logup.rs:1335-1360)
// becomes part of the first round's loads.
struct LogupEvalIL {
    const Fp2 *P, *Q, *s;
    __device__ __forceinline__ void operator()(size_t i, Fp2W* w) const {
        const Fp2 a0 = ldcs2(P + 4 * i), b0 = ldcs2(P + 4 * i + 1), a1 = ldcs2(P + 4 * i + 2), b1 = ldcs2(P + 4 * i + 3);
        const Fp2 c0 = ldcs2(Q + 4 * i), d0 = ldcs2(Q + 4 * i + 1), c1 = ldcs2(Q + 4 * i + 2), d1 = ldcs2(Q + 4 * i + 3);
        const Fp2 si = ldg2(s + i);
        const Fp2 a2 = d2add_weak(a1, d2sub(a1, a0)), b2 = d2add_weak(b1, d2sub(b1, b0));
        const Fp2 c2 = d2add_weak(c1, d2sub(c1, c0)), d2 = d2add_weak(d1, d2sub(d1, d0));
        Fp2W t;
        f2w_zero(t);
        f2w_mac(t, a0, d0);
        f2w_mac(t, b0, c0);
        f2w_mac(w[0], si, f2w_reduce(t));
        f2w_zero(t);
        f2w_mac(t, a2, d2);
        f2w_mac(t, b2, c2);
        f2w_mac(w[1], si, f2w_reduce(t));
        f2w_mac(w[2], si, d2mul(c0, d0));
        f2w_mac(w[3], si, d2mul(c2, d2));
    }
};

struct LogupFoldEvalIL {
    const Fp2 *P, *Q, *s;
    Fp2 *o0, *o1, *o2, *o3;
    Fp2 r;
    __device__ __forceinline__ void operator()(size_t i, Fp2W* w) const {
        Fp2 x[8], y[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            x[k] = ldcs2(P + 8 * i + k);
            y[k] = ldcs2(Q + 8 * i + k);
        }
        const Fp2 a0 = d2fold(x[0], x[2], r), a1 = d2fold(x[4], x[6], r);
        const Fp2 b0 = d2fold(x[1], x[3], r), b1 = d2fold(x[5], x[7], r);
        const Fp2 c0 = d2fold(y[0], y[2], r), c1 = d2fold(y[4], y[6], r);
        const Fp2 d0 = d2fold(y[1], y[3], r), d1 = d2fold(y[5], y[7], r);
        st2(o0 + 2 * i, a0);
        st2(o0 + 2 * i + 1, a1);
        st2(o1 + 2 * i, b0);
        st2(o1 + 2 * i + 1, b1);
        st2(o2 + 2 * i, c0);
        st2(o2 + 2 * i + 1, c1);
        st2(o3 + 2 * i, d0);
        st2(o3 + 2 * i + 1, d1);
        const Fp2 si = ldg2(s + i);
        const Fp2 a2 = d2add_weak(a1, d2sub(a1, a0)), b2 = d2add_weak(b1, d2sub(b1, b0));
        const Fp2 c2 = d2add_weak(c1, d2sub(c1, c0)), d2 = d2add_weak(d1, d2sub(d1, d0));
        Fp2W t;
        f2w_zero(t);
        f2w_mac(t, a0, d0);
        f2w_mac(t, b0, c0);
        f2w_mac(w[0], si, f2w_reduce(t));
        f2w_zero(t);
        f2w_mac(t, a2, d2);
        f2w_mac(t, b2, c2);
        f2w_mac(w[1], si, f2w_reduce(t));
        f2w_mac(w[2], si, d2mul(c0, d0));
        f2w_mac(w[3], si, d2mul(c2, d2));
    }
};

struct DotEval {
    const Fp2 *a, *b;
    __device__ __forceinline__ void operator()(size_t i, Fp2W* w) const { f2w_mac(w[0], ldcs2(a + i), ldcs2(b + i)); }
};

struct PairSumEval {  // sums of an array of (g0, g2) pairs
    const Fp2* in;
    __device__ __forceinline__ void operator()(size_t i, Acc<2>& acc) const {
        acc.v[0] = f2add(acc.v[0], ldcs2(in + 2 * i));
        acc.v[1] = f2add(acc.v[1], ldcs2(in + 2 * i + 1));
    }
};

// Degree-3 aux-leaf round (logup.rs:740-900 per pair):
// pq(t) = S (c_t + d_t), qq(t) = S c_t d_t, aux(t) = sum_k e_t (w0 v0_t + w1 v1_t)
struct AuxEval {
    const Fp2 *q0, *q1, *s, *columns, *eq, *weights;
    const uint32_t* claim_cols;
    size_t column_count, claim_count, vector_len;
    __device__ __forceinline__ void operator()(size_t i, Acc<9>& acc) const {
        const Fp2 c0 = ldg2(q0 + 2 * i), c1 = ldg2(q0 + 2 * i + 1);
        const Fp2 d0 = ldg2(q1 + 2 * i), d1 = ldg2(q1 + 2 * i + 1);
        const Fp2 ct[3] = {c0, f2at2(c0, c1), f2at3(c0, c1)};
        const Fp2 dt[3] = {d0, f2at2(d0, d1), f2at3(d0, d1)};
        const Fp2 si = ldg2(s + i);
#pragma unroll
        for (int t = 0; t < 3; ++t) {
            acc.v[t] = f2add(acc.v[t], f2mul(si, f2add(ct[t], dt[t])));
            acc.v[3 + t] = f2add(acc.v[3 + t], f2mul(si, f2mul(ct[t], dt[t])));
        }
        for (size_t k = 0; k < claim_count; ++k) {
            const size_t col = claim_cols[k];
            if (col >= column_count) continue;
            const Fp2* v0 = columns + (2 * col) * vector_len;
            const Fp2* v1 = columns + (2 * col + 1) * vector_len;
            const Fp2* e = eq + k * vector_len;
            const Fp2 w0 = ldg2(weights + 2 * k), w1 = ldg2(weights + 2 * k + 1);
            const Fp2 x0 = ldg2(v0 + 2 * i), x1 = ldg2(v0 + 2 * i + 1);
            const Fp2 y0 = ldg2(v1 + 2 * i), y1 = ldg2(v1 + 2 * i + 1);
            const Fp2 e0 = ldg2(e + 2 * i), e1 = ldg2(e + 2 * i + 1);
            const Fp2 xt[3] = {x0, f2at2(x0, x1), f2at3(x0, x1)};
            const Fp2 yt[3] = {y0, f2at2(y0, y1), f2at3(y0, y1)};
            const Fp2 et[3] = {e0, f2at2(e0, e1), f2at3(e0, e1)};
#pragma unroll
            for (int t = 0; t < 3; ++t)
                acc.v[6 + t] = f2add(acc.v[6 + t],
                                     f2mul(et[t], f2add(f2mul(w0, xt[t]), f2mul(w1, yt[t]))));
        }
    }
};

// Assemble the aux message: l(t) * cpref * (lambda pq + qq) + aux, with
// l(0) = 1 - p, l(2) = 3p - 1, l(3) = 5p - 2.
struct AuxEpi {
    Fp2* out;
    Fp2 lambda, cpref, point;
    __device__ void operator()(const Acc<9>& a) const {
        const Fp2 p = point;
        const Fp2 l0 = f2sub(f2one(), p);
        const Fp2 l2 = f2sub(f2add(f2add(p, p), p), f2one());
        const Fp2 l3 = f2sub(f2add(f2add(f2add(p, p), f2add(p, p)), p), Fp2{2, 0});
        const Fp2 ell[3] = {l0, l2, l3};
        for (int t = 0; t < 3; ++t)
            out[t] = f2add(f2mul(ell[t], f2mul(cpref, f2add(f2mul(lambda, a.v[t]), a.v[3 + t]))),
                           a.v[6 + t]);
    }
};

struct ScaledPairEpi {  // (scale * dot, -scale * dot)
    Fp2* out;
    Fp2 scale;
    __device__ void operator()(const Acc<1>& a) const {
        const Fp2 v = f2mul(scale, a.v[0]);
        out[0] = v;
        out[1] = f2neg(v);
    }
};

template <int K, class Eval, class Epi>
__global__ void __launch_bounds__(kReduceThreads) reduce_rounds_kernel(
    Eval eval, size_t items, Fp2* partials, unsigned* counter, Epi epi) {
    Acc<K> acc;
    acc.zero();
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < items; i += stride)
        eval(i, acc);
    grid_finish<K>(acc, partials, counter, epi);
}

template <int K, class Eval, class Epi>
static int launch_reduce_wide(Context* c, const Eval& eval, size_t items, const Epi& epi,
                              unsigned per_sm = 4) {
    static_assert(K <= 9, "partials workspace holds 9 accumulators per block");
    const unsigned blocks = grid_for(c, items, kReduceThreads, per_sm < 8 ? per_sm : 8);
    if (!c->ws[kWsPartials].ptr) return fail_message(c, "reduction workspace missing");
    reduce_wide_kernel<K, Eval, Epi><<<blocks, kReduceThreads, 0, c->stream>>>(
        eval, items, ws<Fp2>(c, kWsPartials), ws<unsigned>(c, kWsCounter), epi);
    VZB_LAUNCHED(c);
    return 0;
}

template <int K, class Eval, class Epi>
static int launch_reduce(Context* c, const Eval& eval, size_t items, const Epi& epi,
                         unsigned per_sm = 4) {
    static_assert(K <= 9, "partials workspace holds 9 accumulators per block");
    // grid_for caps the grid at sm_count * per_sm <= sm_count * 8 blocks, the
    // size of the partials workspace allocated at context creation
    const unsigned blocks = grid_for(c, items, kReduceThreads, per_sm < 8 ? per_sm : 8);
    if (!c->ws[kWsPartials].ptr) return fail_message(c, "reduction workspace missing");
    reduce_rounds_kernel<K, Eval, Epi><<<blocks, kReduceThreads, 0, c->stream>>>(
        eval, items, ws<Fp2>(c, kWsPartials), ws<unsigned>(c, kWsCounter), epi);
    VZB_LAUNCHED(c);
    return 0;
}

// Output of a round message: a device pointer (arena mailbox) or a host
// pointer served through the context's mapped pinned mailbox.
struct MsgOut {
    Fp2* dev;
    Fp2* host;
    size_t count;
    unsigned* flag;  // device address of the mailbox flag (host-bound messages)
    unsigned seq;
};

static MsgOut msg_out(Context* c, Fp2* dev, Fp2* host, size_t count) {
    if (dev) return MsgOut{dev, nullptr, count, nullptr, 0};
    unsigned* flag = reinterpret_cast<unsigned*>(static_cast<char*>(c->host_mailbox_dev) + kMailboxFlagOffset);
    return MsgOut{static_cast<Fp2*>(c->host_mailbox_dev), host, count, flag, ++c->mail_seq};
}

template <int K>
static StoreEpi<K> store_epi(const MsgOut& o, Fp2 scale = Fp2{1, 0}, bool scaled = false) {
    return StoreEpi<K>{o.dev, scale, scaled, o.host ? o.flag : nullptr, o.seq};
}

// `flagged`: the kernel publishes the message with the mailbox flag
static int finish_msg(Context* c, int op, const MsgOut& o, bool flagged = true) {
    if (op_mark(c, 2)) return -1;
    if (!o.host) return op_finish(c, op, 0, 0);
    const size_t bytes = o.count * sizeof(Fp2);
    if (flagged ? op_finish_message(c, op, bytes, o.seq) : op_finish(c, op, 0, bytes)) return -1;
    std::memcpy(o.host, c->host_mailbox, bytes);  // message published (flag) or stream synchronised
    return 0;
}

// ---------------------------------------------------------------------------
// folds and element-wise kernels
// ---------------------------------------------------------------------------

// out[row, i] = in[row, 2i] + (in[row, 2i+1] - in[row, 2i]) r
__global__ void fold_rows_kernel(const Fp2* __restrict__ in, Fp2* __restrict__ out, size_t rows,
                                 size_t pairs, Fp2 r) {
    const size_t total = rows * pairs;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t z = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; z < total; z += stride) {
        const size_t row = z / pairs, i = z - row * pairs;
        const Fp2* src = in + row * 2 * pairs;
        st2(out + z, f2fold(ldcs2(src + 2 * i), ldcs2(src + 2 * i + 1), r));
    }
}

struct Quad {
    const Fp2* in[4];
    Fp2* out[4];
};

__global__ void fold4_kernel(Quad q, size_t pairs, Fp2 r) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < pairs; i += stride) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
            st2(q.out[k] + i, f2fold(ldcs2(q.in[k] + 2 * i), ldcs2(q.in[k] + 2 * i + 1), r));
    }
}

__global__ void deinterleave_kernel(const Fp2* in, Fp2* even, Fp2* odd, size_t pairs) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < pairs; i += stride) {
        st2(even + i, ldcs2(in + 2 * i));
        st2(odd + i, ldcs2(in + 2 * i + 1));
    }
}

__global__ void add_inplace_kernel(Fp2* t, const Fp2* a, size_t n) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
        st2(t + i, f2add(ldg2(t + i), ldg2(a + i)));
}

// ---------------------------------------------------------------------------
// eq tables
//
// eq(point, i) = prod_b (bit_b(i) ? point[b] : 1 - point[b]) (LSB-first,
// mle.rs:7-20).  A table of 2^n entries is the outer product of a table over
// the low 12 coordinates and a table over the rest, so every entry beyond
// 2^12 costs one product.  Tables up to 2^12 are built by in-block expansion
// in shared memory.
// ---------------------------------------------------------------------------

constexpr int kEqTileBits = 11;
constexpr int kEqTile = 1 << kEqTileBits;

// Block-wide: write eq(point[0..n), .) * scale (* *scale_dev) (n <= 11) to `out`.
__device__ void eq_block_build(const Fp2* point, int n, Fp2 scale, const Fp2* scale_dev, Fp2* out) {
    __shared__ Fp2 buf[kEqTile];
    if (threadIdx.x == 0) buf[0] = scale_dev ? d2mul(scale, *scale_dev) : scale;
    __syncthreads();
    int size = 1;
    for (int k = n - 1; k >= 0; --k) {
        const Fp2 pk = point[k];
        // expand in place from the top so sources are read before overwrite
        Fp2 lo[kEqTile / 256], hi[kEqTile / 256];
        int cnt = 0;
        for (int i = threadIdx.x; i < size; i += blockDim.x, ++cnt) {
            const Fp2 v = buf[i];
            hi[cnt] = d2mul(v, pk);
            lo[cnt] = d2sub(v, hi[cnt]);
        }
        __syncthreads();
        cnt = 0;
        for (int i = threadIdx.x; i < size; i += blockDim.x, ++cnt) {
            buf[2 * i] = lo[cnt];
            buf[2 * i + 1] = hi[cnt];
        }
        __syncthreads();
        size *= 2;
    }
    for (int i = threadIdx.x; i < size; i += blockDim.x) out[i] = buf[i];
    __syncthreads();
}

// One block per table: tables[t] = eq(points + t * stride_pts, n_t) with n_t <= 12.
struct EqJob {
    const Fp2* point;
    int n;
    Fp2 scale;
    Fp2* out;
    const Fp2* scale_dev;  // optional device-resident factor
};
constexpr int kMaxEqJobs = 320;
struct EqJobs {
    EqJob job[kMaxEqJobs];
    int count;
};

__global__ void __launch_bounds__(256) eq_small_kernel(EqJobs jobs) {
    const EqJob j = jobs.job[blockIdx.x];
    eq_block_build(j.point, j.n, j.scale, j.scale_dev, j.out);
}

// out[i] = lo[i & (2^lo_bits - 1)] * hi[i >> lo_bits] (+ add[i] if add)
__global__ void eq_outer_kernel(const Fp2* lo, int lo_bits, const Fp2* hi, size_t total, Fp2* out,
                                const Fp2* add) {
    const size_t mask = (size_t{1} << lo_bits) - 1;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
        Fp2 v = d2mul(ldg2(lo + (i & mask)), ldg2(hi + (i >> lo_bits)));
        if (add) v = d2add(v, ldg2(add + i));
        st2(out + i, v);
    }
}

// Several outer-product tables in one launch: table t has 2^bits[t] entries,
// out_t[i] = lo_t[i & (2^11 - 1)] * hi_t[i >> 11].  The tables are laid out
// back to back in the launch's index space (first[t] = sum of earlier sizes).
constexpr int kMaxOuterTables = 12;
struct OuterTables {
    const Fp2* lo[kMaxOuterTables];
    const Fp2* hi[kMaxOuterTables];
    Fp2* out[kMaxOuterTables];
    size_t first[kMaxOuterTables + 1];
    int count;
};

__global__ void eq_outer_multi_kernel(OuterTables t) {
    const size_t total = t.first[t.count];
    const size_t mask = kEqTile - 1;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t z = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; z < total; z += stride) {
        int k = 0;
        while (z >= t.first[k + 1]) ++k;
        const size_t i = z - t.first[k];
        st2(t.out[k] + i, d2mul(ldg2(t.lo[k] + (i & mask)), ldg2(t.hi[k] + (i >> kEqTileBits))));
    }
}

// Full eq table of n coordinates (any n < 48) scaled by `scale`, written to
// `out`; `tmp` must hold 2^12 + 2^(n-12) entries when n > 12.
static int eq_table(Context* c, const Fp2* point, int n, Fp2 scale, Fp2* out, Fp2* tmp,
                    const Fp2* add = nullptr, const Fp2* scale_dev = nullptr) {
    if (n <= kEqTileBits && !add) {
        EqJobs jobs{};
        jobs.job[0] = EqJob{point, n, scale, out, scale_dev};
        jobs.count = 1;
        eq_small_kernel<<<1, 256, 0, c->stream>>>(jobs);
        VZB_LAUNCHED(c);
        return 0;
    }
    const int lo_bits = n < kEqTileBits ? n : kEqTileBits;
    Fp2* lo = tmp;
    Fp2* hi = tmp + kEqTile;
    // low table unscaled; high table (recursively) carries the scale
    EqJobs jobs{};
    jobs.job[0] = EqJob{point, lo_bits, Fp2{1, 0}, lo, nullptr};
    jobs.count = 1;
    eq_small_kernel<<<1, 256, 0, c->stream>>>(jobs);
    VZB_LAUNCHED(c);
    const int hi_bits = n - lo_bits;
    if (hi_bits <= kEqTileBits) {
        jobs.job[0] = EqJob{point + lo_bits, hi_bits, scale, hi, scale_dev};
        eq_small_kernel<<<1, 256, 0, c->stream>>>(jobs);
        VZB_LAUNCHED(c);
    } else {
        if (eq_table(c, point + lo_bits, hi_bits, scale, hi, hi + (size_t{1} << hi_bits), nullptr,
                     scale_dev))
            return -1;
    }
    const size_t total = size_t{1} << n;
    eq_outer_kernel<<<grid_for(c, total, 256), 256, 0, c->stream>>>(lo, lo_bits, hi, total, out, add);
    VZB_LAUNCHED(c);
    return 0;
}

// scratch entries eq_table needs for n coordinates
static size_t eq_tmp_entries(int n) {
    if (n <= kEqTileBits) return 0;
    size_t t = kEqTile;
    int rest = n - kEqTileBits;
    t += size_t{1} << rest;
    if (rest > kEqTileBits) t += eq_tmp_entries(rest);
    return t;
}

// In-tile subset-sum stages (strides < 2^12) of the Mobius transform.
__global__ void mobius_tile_kernel(Fp2* v, size_t n) {
    __shared__ Fp2 tile[kEqTile];
    const size_t tile_n = n < kEqTile ? n : kEqTile;
    const size_t base = static_cast<size_t>(blockIdx.x) * tile_n;
    for (size_t i = threadIdx.x; i < tile_n; i += blockDim.x) tile[i] = v[base + i];
    __syncthreads();
    for (size_t stride = 1; stride < tile_n; stride <<= 1) {
        for (size_t i = threadIdx.x; i < tile_n / 2; i += blockDim.x) {
            const size_t blk = i / stride, off = i - blk * stride;
            const size_t low = blk * 2 * stride + off;
            tile[low + stride] = f2add(tile[low + stride], tile[low]);
        }
        __syncthreads();
    }
    for (size_t i = threadIdx.x; i < tile_n; i += blockDim.x) v[base + i] = tile[i];
}

__global__ void mobius_stage_kernel(Fp2* v, size_t pairs, size_t stride) {
    const size_t gs = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < pairs; i += gs) {
        const size_t blk = i / stride, off = i - blk * stride;
        const size_t low = blk * 2 * stride + off;
        st2(v + low + stride, f2add(ldg2(v + low + stride), ldg2(v + low)));
    }
}

// values[i] = rho * eq(point, i) + gamma * (i < source_count ? values[i] : 0)
__global__ void affine_eq_kernel(Fp2* values, const Fp2* eqv, size_t n, size_t source_count,
                                 Fp2 rho, Fp2 gamma) {
    const size_t gs = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += gs) {
        const Fp2 coef = i < source_count ? ldg2(values + i) : Fp2{0, 0};
        st2(values + i, f2add(f2mul(rho, ldg2(eqv + i)), f2mul(gamma, coef)));
    }
}

__global__ void powers_kernel(Fp2 base, Fp2* out, size_t count) {
    const size_t gs = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += gs) {
        // base^(i+1) by square-and-multiply
        size_t e = i + 1;
        Fp2 acc{1, 0}, b = base;
        while (e) {
            if (e & 1) acc = f2mul(acc, b);
            b = f2mul(b, b);
            e >>= 1;
        }
        st2(out + i, acc);
    }
}

__global__ void __launch_bounds__(256) row_dots_kernel(const Fp2* a, size_t as, const Fp2* b,
                                                       size_t bs, Fp2* out, size_t rows,
                                                       size_t len) {
    for (size_t row = blockIdx.x; row < rows; row += gridDim.x) {
        Acc<1> acc;
        acc.zero();
        for (size_t j = threadIdx.x; j < len; j += blockDim.x)
            acc.v[0] = f2add(acc.v[0], f2mul(ldg2(a + row * as + j), ldg2(b + row * bs + j)));
        acc = block_sum<1>(acc);
        if (threadIdx.x == 0) out[row] = acc.v[0];
    }
}

}  // namespace vzb

using namespace vzb;

// ===========================================================================
// C ABI
// ===========================================================================

namespace {

int resolve_pairs_input(Context* c, uint64_t id, size_t offset, size_t pairs, const Fp2** out) {
    size_t n = 0;
    if (!mul_ok(pairs, 2, &n)) return fail_message(c, "resident geometry overflows size_t");
    void* p = nullptr;
    if (region_elems(c, id, offset, n, sizeof(Fp2), &p)) return -1;
    *out = static_cast<const Fp2*>(p);
    return 0;
}

int product_round(Context* c, uint64_t a_id, size_t a_off, uint64_t b_id, size_t b_off,
                  size_t pairs, Fp2* host, uint64_t out_id, size_t out_off, bool scaled, Fp2 scale) {
    const Fp2 *a = nullptr, *b = nullptr;
    if (resolve_pairs_input(c, a_id, a_off, pairs, &a) || resolve_pairs_input(c, b_id, b_off, pairs, &b))
        return -1;
    Fp2* dev = nullptr;
    if (!host) {
        void* p = nullptr;
        if (region_elems(c, out_id, out_off, 2, sizeof(Fp2), &p)) return -1;
        dev = static_cast<Fp2*>(p);
    }
    const MsgOut o = msg_out(c, dev, host, 2);
    if (op_begin(c) || op_mark(c, 1)) return -1;
    if (launch_reduce_wide<2>(c, ProductEval{a, b}, pairs, store_epi<2>(o, scale, scaled))) return -1;
    return finish_msg(c, kOpGemm, o);
}

int triple_round(Context* c, uint64_t a_id, size_t a_off, uint64_t b_id, size_t b_off,
                 uint64_t c_id, size_t c_off, size_t pairs, Fp2* host, uint64_t out_id,
                 size_t out_off) {
    const Fp2 *a = nullptr, *b = nullptr, *cc = nullptr;
    if (resolve_pairs_input(c, a_id, a_off, pairs, &a) || resolve_pairs_input(c, b_id, b_off, pairs, &b) ||
        resolve_pairs_input(c, c_id, c_off, pairs, &cc))
        return -1;
    Fp2* dev = nullptr;
    if (!host) {
        void* p = nullptr;
        if (region_elems(c, out_id, out_off, 3, sizeof(Fp2), &p)) return -1;
        dev = static_cast<Fp2*>(p);
    }
    const MsgOut o = msg_out(c, dev, host, 3);
    if (op_begin(c) || op_mark(c, 1)) return -1;
    if (launch_reduce_wide<3>(c, TripleEval{a, b, cc}, pairs, store_epi<3>(o), 8)) return -1;
    return finish_msg(c, kOpGemm, o);
}

int logup_round(Context* c, const Fp2* p0, const Fp2* p1, const Fp2* q0, const Fp2* q1,
                const Fp2* s, size_t pairs, const MsgOut& o) {
    return launch_reduce_wide<4>(c, LogupEval{p0, p1, q0, q1, s}, pairs, store_epi<4>(o));
}

int resolve_logup_inputs(Context* c, uint64_t p0_id, size_t p0_off, uint64_t p1_id, size_t p1_off,
                         uint64_t q0_id, size_t q0_off, uint64_t q1_id, size_t q1_off,
                         uint64_t s_id, size_t s_off, size_t pairs, const Fp2** v) {
    void* s = nullptr;
    if (resolve_pairs_input(c, p0_id, p0_off, pairs, &v[0]) ||
        resolve_pairs_input(c, p1_id, p1_off, pairs, &v[1]) ||
        resolve_pairs_input(c, q0_id, q0_off, pairs, &v[2]) ||
        resolve_pairs_input(c, q1_id, q1_off, pairs, &v[3]) ||
        region_elems(c, s_id, s_off, pairs, sizeof(Fp2), &s))
        return -1;
    v[4] = static_cast<const Fp2*>(s);
    return 0;
}

int launch_fold_rows(Context* c, const Fp2* in, Fp2* out, size_t rows, size_t pairs, Fp2 r) {
    const size_t total = rows * pairs;
    fold_rows_kernel<<<grid_for(c, total, 256), 256, 0, c->stream>>>(in, out, rows, pairs, r);
    VZB_LAUNCHED(c);
    return 0;
}

}  // namespace

extern "C" int volta_cuda_reserve_fp2_product_round_workspace(void* raw, size_t max_pairs) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !max_pairs) return reject(c, "invalid product-round workspace reservation");
    if (c->coarse || c->active_record != kRingSize)
        return reject(c, "cannot reserve product-round workspace during active timing");
    // The single-launch reduction needs only the fixed per-block partials
    // allocated at context creation; nothing grows with max_pairs.
    return 0;
}

extern "C" int volta_cuda_reserve_logup_round_workspace(void* raw, size_t max_pairs) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !max_pairs) return reject(c, "invalid LogUp round workspace reservation");
    if (c->coarse || c->active_record != kRingSize)
        return reject(c, "cannot reserve LogUp round workspace during active timing");
    return 0;
}

extern "C" int volta_cuda_fp2_product_round_device(void* raw, uint64_t a_id, size_t a_off,
                                                   uint64_t b_id, size_t b_off, size_t pairs,
                                                   Fp2* output) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !pairs || !output) return fail_message(c, "invalid resident product-round geometry");
    return product_round(c, a_id, a_off, b_id, b_off, pairs, output, 0, 0, false, Fp2{1, 0});
}

extern "C" int volta_cuda_fp2_product_round_into_device(void* raw, uint64_t a_id, size_t a_off,
                                                        uint64_t b_id, size_t b_off, size_t pairs,
                                                        uint64_t out_id, size_t out_off) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !pairs) return fail_message(c, "invalid resident product-round mailbox geometry");
    return product_round(c, a_id, a_off, b_id, b_off, pairs, nullptr, out_id, out_off, false, Fp2{1, 0});
}

extern "C" int volta_cuda_fp2_product_round_scaled_into_device(void* raw, uint64_t a_id,
                                                               size_t a_off, uint64_t b_id,
                                                               size_t b_off, size_t pairs,
                                                               Fp2 scale, uint64_t out_id,
                                                               size_t out_off) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !pairs)
        return fail_message(c, "invalid resident scaled product-round mailbox geometry");
    return product_round(c, a_id, a_off, b_id, b_off, pairs, nullptr, out_id, out_off, true, scale);
}

extern "C" int volta_cuda_fp2_triple_product_round_device(void* raw, uint64_t a_id, size_t a_off,
                                                          uint64_t b_id, size_t b_off,
                                                          uint64_t c_id, size_t c_off,
                                                          size_t pairs, Fp2* output) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !pairs || !output) return fail_message(c, "invalid resident triple-product geometry");
    return triple_round(c, a_id, a_off, b_id, b_off, c_id, c_off, pairs, output, 0, 0);
}

extern "C" int volta_cuda_fp2_triple_product_round_into_device(void* raw, uint64_t a_id,
                                                               size_t a_off, uint64_t b_id,
                                                               size_t b_off, uint64_t c_id,
                                                               size_t c_off, size_t pairs,
                                                               uint64_t out_id, size_t out_off) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !pairs) return fail_message(c, "invalid resident triple-product mailbox geometry");
    return triple_round(c, a_id, a_off, b_id, b_off, c_id, c_off, pairs, nullptr, out_id, out_off);
}

extern "C" int volta_cuda_logup_general_round(void* raw, const Fp2* p0, const Fp2* p1,
                                              const Fp2* q0, const Fp2* q1, const Fp2* suffix,
                                              size_t pairs, Fp2* output) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !p0 || !p1 || !q0 || !q1 || !suffix || !output || !pairs) return -1;
    const size_t vb = 2 * pairs * sizeof(Fp2), sb = pairs * sizeof(Fp2);
    const int slots[5] = {kWsStageA, kWsStageB, kWsStageC, kWsStageD, kWsStageE};
    for (int i = 0; i < 5; ++i)
        if (ensure_ws(c, slots[i], i == 4 ? sb : vb)) return -1;
    if (op_begin(c)) return -1;
    const Fp2* src[5] = {p0, p1, q0, q1, suffix};
    for (int i = 0; i < 5; ++i)
        VZB_CUDA(c, cudaMemcpyAsync(c->ws[slots[i]].ptr, src[i], i == 4 ? sb : vb,
                                    cudaMemcpyHostToDevice, c->stream));
    if (op_mark(c, 1)) return -1;
    const MsgOut o = msg_out(c, nullptr, output, 4);
    if (logup_round(c, ws<Fp2>(c, kWsStageA), ws<Fp2>(c, kWsStageB), ws<Fp2>(c, kWsStageC),
                    ws<Fp2>(c, kWsStageD), ws<Fp2>(c, kWsStageE), pairs, o))
        return -1;
    if (op_mark(c, 2)) return -1;
    if (op_finish(c, kOpLogup, 4 * vb + sb, 4 * sizeof(Fp2))) return -1;
    std::memcpy(output, c->host_mailbox, 4 * sizeof(Fp2));
    return 0;
}

extern "C" int volta_cuda_logup_general_round_device(void* raw, uint64_t p0_id, size_t p0_off,
                                                     uint64_t p1_id, size_t p1_off,
                                                     uint64_t q0_id, size_t q0_off,
                                                     uint64_t q1_id, size_t q1_off,
                                                     uint64_t s_id, size_t s_off, size_t pairs,
                                                     Fp2* output) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !pairs || !output) return fail_message(c, "invalid resident LogUp round geometry");
    const Fp2* v[5];
    if (resolve_logup_inputs(c, p0_id, p0_off, p1_id, p1_off, q0_id, q0_off, q1_id, q1_off, s_id,
                             s_off, pairs, v))
        return -1;
    const MsgOut o = msg_out(c, nullptr, output, 4);
    if (op_begin(c) || op_mark(c, 1)) return -1;
    if (logup_round(c, v[0], v[1], v[2], v[3], v[4], pairs, o)) return -1;
    return finish_msg(c, kOpLogup, o);
}

extern "C" int volta_cuda_logup_general_round_into_device(void* raw, uint64_t p0_id, size_t p0_off,
                                                          uint64_t p1_id, size_t p1_off,
                                                          uint64_t q0_id, size_t q0_off,
                                                          uint64_t q1_id, size_t q1_off,
                                                          uint64_t s_id, size_t s_off,
                                                          size_t pairs, uint64_t out_id,
                                                          size_t out_off) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !pairs) return fail_message(c, "invalid resident LogUp round mailbox geometry");
    const Fp2* v[5];
    void* out = nullptr;
    if (resolve_logup_inputs(c, p0_id, p0_off, p1_id, p1_off, q0_id, q0_off, q1_id, q1_off, s_id,
                             s_off, pairs, v) ||
        region_elems(c, out_id, out_off, 4, sizeof(Fp2), &out))
        return -1;
    const MsgOut o = msg_out(c, static_cast<Fp2*>(out), nullptr, 4);
    if (op_begin(c) || op_mark(c, 1)) return -1;
    if (logup_round(c, v[0], v[1], v[2], v[3], v[4], pairs, o)) return -1;
    return finish_msg(c, kOpLogup, o);
}

extern "C" int volta_cuda_logup_fold4(void* raw, const Fp2* p0, const Fp2* p1, const Fp2* q0,
                                      const Fp2* q1, size_t pairs, Fp2 r, Fp2* o0, Fp2* o1,
                                      Fp2* o2, Fp2* o3) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !p0 || !p1 || !q0 || !q1 || !o0 || !o1 || !o2 || !o3 || !pairs) return -1;
    const size_t ib = 2 * pairs * sizeof(Fp2), ob = pairs * sizeof(Fp2);
    const int in_slots[4] = {kWsStageA, kWsStageB, kWsStageC, kWsStageD};
    const int out_slots[4] = {kWsStageE, kWsStageF, kWsStageG, kWsStageH};
    for (int i = 0; i < 4; ++i)
        if (ensure_ws(c, in_slots[i], ib) || ensure_ws(c, out_slots[i], ob)) return -1;
    if (op_begin(c)) return -1;
    const Fp2* src[4] = {p0, p1, q0, q1};
    for (int i = 0; i < 4; ++i)
        VZB_CUDA(c, cudaMemcpyAsync(c->ws[in_slots[i]].ptr, src[i], ib, cudaMemcpyHostToDevice, c->stream));
    if (op_mark(c, 1)) return -1;
    Quad q{};
    for (int i = 0; i < 4; ++i) {
        q.in[i] = ws<Fp2>(c, in_slots[i]);
        q.out[i] = ws<Fp2>(c, out_slots[i]);
    }
    fold4_kernel<<<grid_for(c, pairs, 256), 256, 0, c->stream>>>(q, pairs, r);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    Fp2* dst[4] = {o0, o1, o2, o3};
    for (int i = 0; i < 4; ++i)
        VZB_CUDA(c, cudaMemcpyAsync(dst[i], q.out[i], ob, cudaMemcpyDeviceToHost, c->stream));
    return op_finish(c, kOpLogup, 4 * ib, 4 * ob);
}

extern "C" int volta_cuda_logup_fold4_device(void* raw, uint64_t p0_id, size_t p0_off,
                                             uint64_t p1_id, size_t p1_off, uint64_t q0_id,
                                             size_t q0_off, uint64_t q1_id, size_t q1_off,
                                             size_t pairs, Fp2 r, uint64_t o0_id, size_t o0_off,
                                             uint64_t o1_id, size_t o1_off, uint64_t o2_id,
                                             size_t o2_off, uint64_t o3_id, size_t o3_off) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !pairs) return fail_message(c, "invalid resident LogUp fold geometry");
    const uint64_t ii[4] = {p0_id, p1_id, q0_id, q1_id};
    const size_t io[4] = {p0_off, p1_off, q0_off, q1_off};
    const uint64_t oi[4] = {o0_id, o1_id, o2_id, o3_id};
    const size_t oo[4] = {o0_off, o1_off, o2_off, o3_off};
    Quad q{};
    for (int i = 0; i < 4; ++i) {
        void* out = nullptr;
        if (resolve_pairs_input(c, ii[i], io[i], pairs, &q.in[i]) ||
            region_elems(c, oi[i], oo[i], pairs, sizeof(Fp2), &out))
            return -1;
        q.out[i] = static_cast<Fp2*>(out);
    }
    if (op_begin(c) || op_mark(c, 1)) return -1;
    fold4_kernel<<<grid_for(c, pairs, 256), 256, 0, c->stream>>>(q, pairs, r);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpLogup, 0, 0);
}

extern "C" int volta_cuda_fp2_deinterleave_device(void* raw, uint64_t in_id, size_t in_off,
                                                  size_t pairs, uint64_t even_id, size_t even_off,
                                                  uint64_t odd_id, size_t odd_off) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !pairs) return fail_message(c, "invalid resident deinterleave geometry");
    const Fp2* in = nullptr;
    void *even = nullptr, *odd = nullptr;
    if (resolve_pairs_input(c, in_id, in_off, pairs, &in) ||
        region_elems(c, even_id, even_off, pairs, sizeof(Fp2), &even) ||
        region_elems(c, odd_id, odd_off, pairs, sizeof(Fp2), &odd))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    deinterleave_kernel<<<grid_for(c, pairs, 256), 256, 0, c->stream>>>(
        in, static_cast<Fp2*>(even), static_cast<Fp2*>(odd), pairs);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpLogup, 0, 0);
}

// Suffix tables: table k (2^k entries, eq over the last k coordinates) at
// offset 2^k - 1, k = 0 .. L-1 (logup.rs:284-305).
extern "C" int volta_cuda_logup_suffix_eq_device(void* raw, uint64_t points_id, size_t points_off,
                                                 size_t point_len, uint64_t out_id, size_t out_off) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !point_len || point_len >= 63) return fail_message(c, "invalid resident suffix-eq geometry");
    const size_t total = (size_t{1} << point_len) - 1;
    void *pts = nullptr, *out = nullptr;
    if (region_elems(c, points_id, points_off, point_len, sizeof(Fp2), &pts) ||
        region_elems(c, out_id, out_off, total, sizeof(Fp2), &out))
        return -1;
    const Fp2* point = static_cast<const Fp2*>(pts);
    Fp2* o = static_cast<Fp2*>(out);
    const int L = static_cast<int>(point_len);
    // tables with k <= 12 come from one multi-job launch; larger tables are
    // outer products of their low 12 coordinates and the table k - 12.
    size_t tmp_entries = 0;
    for (int k = kEqTileBits + 1; k < L; ++k) tmp_entries += kEqTile;
    if (tmp_entries && ensure_ws(c, kWsScratch, tmp_entries * sizeof(Fp2))) return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    EqJobs jobs{};
    for (int k = 0; k < L && k <= kEqTileBits; ++k) {
        jobs.job[jobs.count++] = EqJob{point + (L - k), k, Fp2{1, 0}, o + ((size_t{1} << k) - 1), nullptr};
    }
    Fp2* lows = ws<Fp2>(c, kWsScratch);
    for (int k = kEqTileBits + 1; k < L; ++k) {
        if (jobs.count == kMaxEqJobs) return fail_message(c, "suffix-eq job table overflow");
        jobs.job[jobs.count++] =
            EqJob{point + (L - k), kEqTileBits, Fp2{1, 0}, lows + static_cast<size_t>(k - kEqTileBits - 1) * kEqTile, nullptr};
    }
    eq_small_kernel<<<jobs.count, 256, 0, c->stream>>>(jobs);
    VZB_LAUNCHED(c);
    // one launch per band of 11 tables: table k is the outer product of its
    // low 11 coordinates and table k - 11, which an earlier band (or the
    // small-table launch) completed
    for (int band = kEqTileBits + 1; band < L; band += kEqTileBits) {
        OuterTables t{};
        for (int k = band; k < L && k < band + kEqTileBits; ++k) {
            const size_t entries = size_t{1} << k;
            t.lo[t.count] = lows + static_cast<size_t>(k - kEqTileBits - 1) * kEqTile;
            t.hi[t.count] = o + ((size_t{1} << (k - kEqTileBits)) - 1);
            t.out[t.count] = o + (entries - 1);
            t.first[t.count + 1] = t.first[t.count] + entries;
            ++t.count;
        }
        eq_outer_multi_kernel<<<grid_for(c, t.first[t.count], 256), 256, 0, c->stream>>>(t);
        VZB_LAUNCHED(c);
    }
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpLogup, 0, 0);
}

// Outer-product tables of several layers in one launch: table t (entries
// 2^bits) is out_t[i] = lo_t[i & (2^11 - 1)] * hi_t[i >> 11]; its CTAs are
// [block0, block0 + blocks), in proportion to its size.
constexpr int kMaxOuterBatch = 256;
struct OuterJob {
    const Fp2* lo;
    const Fp2* hi;
    Fp2* out;
    size_t entries;
    uint32_t block0, blocks;
};
struct OuterBatch {
    OuterJob t[kMaxOuterBatch];
    int count;
};

__global__ void __launch_bounds__(256) eq_outer_batch_kernel(const __grid_constant__ OuterBatch b) {
    int lo = 0, hi = b.count - 1;  // last table whose first CTA is <= blockIdx.x
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (b.t[mid].block0 <= blockIdx.x) lo = mid;
        else hi = mid - 1;
    }
    const OuterJob& t = b.t[lo];
    const size_t stride = static_cast<size_t>(t.blocks) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x - t.block0) * blockDim.x + threadIdx.x; i < t.entries; i += stride)
        st2(t.out + i, d2mul(ldg2(t.lo + (i & (kEqTile - 1))), ldg2(t.hi + (i >> kEqTileBits))));
}

extern "C" int volta_b200_logup_suffix_eq_batch_device(void* raw, const vzb_suffix_job* jobs, size_t count) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !jobs || !count) return fail_message(c, "invalid suffix-eq batch");
    std::vector<const Fp2*> pts(count);
    std::vector<Fp2*> outs(count);
    std::vector<size_t> low_base(count, 0);
    size_t lows_total = 0;
    int max_len = 0;
    for (size_t j = 0; j < count; ++j) {
        const vzb_suffix_job& q = jobs[j];
        if (!q.point_len || q.point_len >= 63) return fail_message(c, "invalid resident suffix-eq geometry");
        void *p = nullptr, *o = nullptr;
        if (region_elems(c, q.points_id, q.points_offset, q.point_len, sizeof(Fp2), &p) ||
            region_elems(c, q.out_id, q.out_offset, (size_t{1} << q.point_len) - 1, sizeof(Fp2), &o))
            return -1;
        pts[j] = static_cast<const Fp2*>(p);
        outs[j] = static_cast<Fp2*>(o);
        const int L = static_cast<int>(q.point_len);
        low_base[j] = lows_total;
        if (L > kEqTileBits + 1) lows_total += static_cast<size_t>(L - kEqTileBits - 1) * kEqTile;
        max_len = std::max(max_len, L);
    }
    if (lows_total && ensure_ws(c, kWsScratch, lows_total * sizeof(Fp2))) return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    Fp2* lows = lows_total ? ws<Fp2>(c, kWsScratch) : nullptr;
    // tables of <= 11 coordinates and the 11-coordinate low factors of the
    // larger ones, one CTA each, kMaxEqJobs per launch
    EqJobs small{};
    auto flush_small = [&]() -> int {
        if (!small.count) return 0;
        eq_small_kernel<<<small.count, 256, 0, c->stream>>>(small);
        VZB_LAUNCHED(c);
        small.count = 0;
        return 0;
    };
    for (size_t j = 0; j < count; ++j) {
        const int L = static_cast<int>(jobs[j].point_len);
        const Fp2* point = pts[j];
        for (int k = 0; k < L; ++k) {
            if (small.count == kMaxEqJobs && flush_small()) return -1;
            if (k <= kEqTileBits)
                small.job[small.count++] = EqJob{point + (L - k), k, Fp2{1, 0}, outs[j] + ((size_t{1} << k) - 1), nullptr};
            else
                small.job[small.count++] = EqJob{point + (L - k), kEqTileBits, Fp2{1, 0},
                                                 lows + low_base[j] + static_cast<size_t>(k - kEqTileBits - 1) * kEqTile,
                                                 nullptr};
        }
    }
    if (flush_small()) return -1;
    // bands of 11 table sizes across all jobs: table k is the outer product
    // of its low factor and table k - 11 (complete after the previous band)
    for (int band = kEqTileBits + 1; band < max_len; band += kEqTileBits) {
        OuterBatch ob{};
        size_t total = 0;
        for (size_t j = 0; j < count; ++j) {
            const int L = static_cast<int>(jobs[j].point_len);
            for (int k = band; k < L && k < band + kEqTileBits; ++k) {
                if (ob.count == kMaxOuterBatch) return fail_message(c, "suffix-eq batch has too many large tables");
                OuterJob& t = ob.t[ob.count++];
                t.lo = lows + low_base[j] + static_cast<size_t>(k - kEqTileBits - 1) * kEqTile;
                t.hi = outs[j] + ((size_t{1} << (k - kEqTileBits)) - 1);
                t.out = outs[j] + ((size_t{1} << k) - 1);
                t.entries = size_t{1} << k;
                total += t.entries;
            }
        }
        if (!ob.count) continue;
        const size_t target = static_cast<size_t>(c->sm_count) * 8;
        uint32_t next = 0;
        for (int i = 0; i < ob.count; ++i) {
            OuterJob& t = ob.t[i];
            const size_t need = (t.entries + 255) / 256;
            size_t share = (target * t.entries + total - 1) / total;
            if (share < 1) share = 1;
            t.block0 = next;
            t.blocks = static_cast<uint32_t>(std::min(need, share));
            next += t.blocks;
        }
        eq_outer_batch_kernel<<<next, 256, 0, c->stream>>>(ob);
        VZB_LAUNCHED(c);
    }
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpLogup, 0, 0);
}

extern "C" int volta_cuda_fp2_fold_rows_device(void* raw, uint64_t in_id, size_t in_off,
                                               size_t rows, size_t len, Fp2 r, uint64_t out_id,
                                               size_t out_off) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !rows || len < 2 || (len & 1)) return fail_message(c, "invalid resident row-fold geometry");
    const size_t pairs = len / 2;
    size_t n_in = 0, n_out = 0;
    if (!mul_ok(rows, len, &n_in) || !mul_ok(rows, pairs, &n_out))
        return fail_message(c, "resident row-fold geometry overflows size_t");
    void *in = nullptr, *out = nullptr;
    if (region_elems(c, in_id, in_off, n_in, sizeof(Fp2), &in) ||
        region_elems(c, out_id, out_off, n_out, sizeof(Fp2), &out))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    if (launch_fold_rows(c, static_cast<const Fp2*>(in), static_cast<Fp2*>(out), rows, pairs, r)) return -1;
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpLogup, 0, 0);
}

extern "C" int volta_cuda_logup_eq_rows_device(void* raw, uint64_t points_id, size_t points_off,
                                               size_t rows, size_t dims, uint64_t out_id,
                                               size_t out_off) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !rows || dims >= 63 || (dims && !points_id))
        return fail_message(c, "invalid resident eq-row geometry");
    const size_t width = size_t{1} << dims;
    size_t total = 0;
    if (!mul_ok(rows, width, &total)) return fail_message(c, "resident eq-row geometry overflows size_t");
    void *pts = nullptr, *out = nullptr;
    if ((dims && region_elems(c, points_id, points_off, rows * dims, sizeof(Fp2), &pts)) ||
        region_elems(c, out_id, out_off, total, sizeof(Fp2), &out))
        return -1;
    const Fp2* point = static_cast<const Fp2*>(pts);
    Fp2* o = static_cast<Fp2*>(out);
    const size_t tmp = eq_tmp_entries(static_cast<int>(dims));
    if (tmp && ensure_ws(c, kWsScratch, tmp * sizeof(Fp2))) return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    if (dims <= static_cast<size_t>(kEqTileBits)) {
        for (size_t r0 = 0; r0 < rows; r0 += kMaxEqJobs) {
            EqJobs jobs{};
            for (size_t r = r0; r < rows && jobs.count < kMaxEqJobs; ++r)
                jobs.job[jobs.count++] = EqJob{point + r * dims, static_cast<int>(dims), Fp2{1, 0}, o + r * width, nullptr};
            eq_small_kernel<<<jobs.count, 256, 0, c->stream>>>(jobs);
            VZB_LAUNCHED(c);
        }
    } else {
        for (size_t r = 0; r < rows; ++r)
            if (eq_table(c, point + r * dims, static_cast<int>(dims), Fp2{1, 0}, o + r * width,
                         ws<Fp2>(c, kWsScratch)))
                return -1;
    }
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpLogup, 0, 0);
}

namespace {

int aux_round(Context* c, uint64_t q0_id, size_t q0_off, uint64_t q1_id, size_t q1_off,
              uint64_t s_id, size_t s_off, uint64_t col_id, size_t col_off, uint64_t eq_id,
              size_t eq_off, uint64_t cc_id, size_t cc_off, uint64_t w_id, size_t w_off,
              size_t column_count, size_t claim_count, size_t vector_len, Fp2 lambda, Fp2 cpref,
              Fp2 point, Fp2* host, uint64_t out_id, size_t out_off) {
    const size_t pairs = vector_len / 2;
    void *q0 = nullptr, *q1 = nullptr, *s = nullptr, *cols = nullptr;
    void *eq = nullptr, *cc = nullptr, *w = nullptr;
    size_t col_n = 0, eq_n = 0;
    if (!mul_ok(column_count, vector_len, &col_n) || !mul_ok(col_n, 2, &col_n) ||
        !mul_ok(claim_count, vector_len, &eq_n))
        return fail_message(c, "resident aux-round geometry overflows size_t");
    if (region_elems(c, q0_id, q0_off, vector_len, sizeof(Fp2), &q0) ||
        region_elems(c, q1_id, q1_off, vector_len, sizeof(Fp2), &q1) ||
        region_elems(c, s_id, s_off, pairs, sizeof(Fp2), &s) ||
        region_elems(c, col_id, col_off, col_n, sizeof(Fp2), &cols))
        return -1;
    if (claim_count &&
        (region_elems(c, eq_id, eq_off, eq_n, sizeof(Fp2), &eq) ||
         region_elems(c, cc_id, cc_off, claim_count, sizeof(uint32_t), &cc) ||
         region_elems(c, w_id, w_off, 2 * claim_count, sizeof(Fp2), &w)))
        return -1;
    Fp2* dev = nullptr;
    if (!host) {
        void* p = nullptr;
        if (region_elems(c, out_id, out_off, 3, sizeof(Fp2), &p)) return -1;
        dev = static_cast<Fp2*>(p);
    }
    const MsgOut o = msg_out(c, dev, host, 3);
    if (op_begin(c) || op_mark(c, 1)) return -1;
    AuxEval ev{static_cast<const Fp2*>(q0), static_cast<const Fp2*>(q1), static_cast<const Fp2*>(s),
               static_cast<const Fp2*>(cols), static_cast<const Fp2*>(eq), static_cast<const Fp2*>(w),
               static_cast<const uint32_t*>(cc), column_count, claim_count, vector_len};
    if (launch_reduce<9>(c, ev, pairs, AuxEpi{o.dev, lambda, cpref, point}, 2)) return -1;
    return finish_msg(c, kOpLogup, o, false);
}

}  // namespace

extern "C" int volta_cuda_logup_aux_round_device(
    void* raw, uint64_t q0_id, size_t q0_off, uint64_t q1_id, size_t q1_off, uint64_t s_id,
    size_t s_off, uint64_t col_id, size_t col_off, uint64_t eq_id, size_t eq_off, uint64_t cc_id,
    size_t cc_off, uint64_t w_id, size_t w_off, size_t column_count, size_t claim_count,
    size_t vector_len, Fp2 lambda, Fp2 cpref, Fp2 point, Fp2* output) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !output || !column_count || vector_len < 2 || (vector_len & 1))
        return fail_message(c, "invalid resident aux-round geometry");
    return aux_round(c, q0_id, q0_off, q1_id, q1_off, s_id, s_off, col_id, col_off, eq_id, eq_off,
                     cc_id, cc_off, w_id, w_off, column_count, claim_count, vector_len, lambda,
                     cpref, point, output, 0, 0);
}

extern "C" int volta_cuda_logup_aux_round_into_device(
    void* raw, uint64_t q0_id, size_t q0_off, uint64_t q1_id, size_t q1_off, uint64_t s_id,
    size_t s_off, uint64_t col_id, size_t col_off, uint64_t eq_id, size_t eq_off, uint64_t cc_id,
    size_t cc_off, uint64_t w_id, size_t w_off, size_t column_count, size_t claim_count,
    size_t vector_len, Fp2 lambda, Fp2 cpref, Fp2 point, uint64_t out_id, size_t out_off) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !column_count || vector_len < 2 || (vector_len & 1))
        return fail_message(c, "invalid resident aux-round mailbox geometry");
    return aux_round(c, q0_id, q0_off, q1_id, q1_off, s_id, s_off, col_id, col_off, eq_id, eq_off,
                     cc_id, cc_off, w_id, w_off, column_count, claim_count, vector_len, lambda,
                     cpref, point, nullptr, out_id, out_off);
}

extern "C" int volta_cuda_fp2_dot_device(void* raw, uint64_t a_id, size_t a_off, uint64_t b_id,
                                         size_t b_off, size_t n, Fp2* output) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !n || !output) return fail_message(c, "invalid resident Fp2 dot geometry");
    void *a = nullptr, *b = nullptr;
    if (region_elems(c, a_id, a_off, n, sizeof(Fp2), &a) || region_elems(c, b_id, b_off, n, sizeof(Fp2), &b))
        return -1;
    const MsgOut o = msg_out(c, nullptr, output, 1);
    if (op_begin(c) || op_mark(c, 1)) return -1;
    if (launch_reduce_wide<1>(c, DotEval{static_cast<const Fp2*>(a), static_cast<const Fp2*>(b)}, n,
                         store_epi<1>(o)))
        return -1;
    return finish_msg(c, kOpGemm, o);
}

extern "C" int volta_cuda_fp2_dot_scaled_pair_into_device(void* raw, uint64_t a_id, size_t a_off,
                                                          uint64_t b_id, size_t b_off, size_t n,
                                                          Fp2 scale, uint64_t out_id,
                                                          size_t out_off) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !n) return fail_message(c, "invalid X4d scaled-dot geometry");
    void *a = nullptr, *b = nullptr, *out = nullptr;
    if (region_elems(c, a_id, a_off, n, sizeof(Fp2), &a) || region_elems(c, b_id, b_off, n, sizeof(Fp2), &b) ||
        region_elems(c, out_id, out_off, 2, sizeof(Fp2), &out))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    if (launch_reduce_wide<1>(c, DotEval{static_cast<const Fp2*>(a), static_cast<const Fp2*>(b)}, n,
                         ScaledPairEpi{static_cast<Fp2*>(out), scale}))
        return -1;
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpGemm, 0, 0);
}

extern "C" int volta_cuda_fp2_pair_sum_device(void* raw, uint64_t in_id, size_t in_off, size_t pairs,
                                              Fp2* output) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !pairs || !output) return fail_message(c, "invalid X4d pair-mailbox geometry");
    size_t off = 0;
    if (!mul_ok(in_off, 2, &off)) return fail_message(c, "X4d pair geometry overflows size_t");
    const Fp2* in = nullptr;
    if (resolve_pairs_input(c, in_id, off, pairs, &in)) return -1;
    const MsgOut o = msg_out(c, nullptr, output, 2);
    if (op_begin(c) || op_mark(c, 1)) return -1;
    if (launch_reduce<2>(c, PairSumEval{in}, pairs, store_epi<2>(o))) return -1;
    return finish_msg(c, kOpGemm, o);
}

extern "C" int volta_cuda_claim_reduce_f_two_into_device(
    void* raw, uint64_t points_id, size_t points_off, size_t n_vars, uint64_t out_id,
    size_t out_off, uint64_t s1_id, size_t s1_off, uint64_t s2_id, size_t s2_off, uint64_t s3_id,
    size_t s3_off) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !n_vars || n_vars > 30) return fail_message(c, "invalid ClaimReduce F geometry");
    const size_t len = size_t{1} << n_vars;
    void *pts = nullptr, *out = nullptr, *s1 = nullptr, *s2 = nullptr, *s3 = nullptr;
    if (region_elems(c, points_id, points_off, 2 * n_vars + 2, sizeof(Fp2), &pts) ||
        region_elems(c, out_id, out_off, len, sizeof(Fp2), &out) ||
        region_elems(c, s1_id, s1_off, len, sizeof(Fp2), &s1) ||
        region_elems(c, s2_id, s2_off, len, sizeof(Fp2), &s2) ||
        region_elems(c, s3_id, s3_off, len, sizeof(Fp2), &s3))
        return -1;
    const Fp2* p = static_cast<const Fp2*>(pts);
    // out = s1 * eq(p[0..n)) + s2 * eq(p[n..2n)); the scales p[2n], p[2n+1]
    // stay on the device and are read inside the table kernels.
    const size_t tmp = eq_tmp_entries(static_cast<int>(n_vars));
    if (tmp && ensure_ws(c, kWsScratch, tmp * sizeof(Fp2))) return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    Fp2* second = static_cast<Fp2*>(s2);
    if (eq_table(c, p + n_vars, static_cast<int>(n_vars), Fp2{1, 0}, second, ws<Fp2>(c, kWsScratch),
                 nullptr, p + 2 * n_vars + 1))
        return -1;
    if (n_vars <= static_cast<size_t>(kEqTileBits)) {
        if (eq_table(c, p, static_cast<int>(n_vars), Fp2{1, 0}, static_cast<Fp2*>(s1),
                     ws<Fp2>(c, kWsScratch), nullptr, p + 2 * n_vars))
            return -1;
        add_inplace_kernel<<<1, 256, 0, c->stream>>>(static_cast<Fp2*>(s1), second, len);
        VZB_LAUNCHED(c);
        VZB_CUDA(c, cudaMemcpyAsync(out, s1, len * sizeof(Fp2), cudaMemcpyDeviceToDevice, c->stream));
    } else if (eq_table(c, p, static_cast<int>(n_vars), Fp2{1, 0}, static_cast<Fp2*>(out),
                        ws<Fp2>(c, kWsScratch), second, p + 2 * n_vars)) {
        return -1;
    }
    (void)s3;
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpGemm, 0, 0);
}

extern "C" int volta_cuda_x4d_link_eq_accumulate_device(void* raw, uint64_t point_id,
                                                        size_t point_off, size_t n_vars,
                                                        uint64_t target_id, size_t target_off,
                                                        uint64_t s1_id, size_t s1_off,
                                                        uint64_t s2_id, size_t s2_off,
                                                        int initialize) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !n_vars || n_vars > 30 || (initialize != 0 && initialize != 1))
        return fail_message(c, "invalid X4d link-equality geometry");
    const size_t len = size_t{1} << n_vars;
    void *pt = nullptr, *target = nullptr, *s1 = nullptr, *s2 = nullptr;
    if (region_elems(c, point_id, point_off, n_vars + 1, sizeof(Fp2), &pt) ||
        region_elems(c, target_id, target_off, len, sizeof(Fp2), &target) ||
        region_elems(c, s1_id, s1_off, len, sizeof(Fp2), &s1) ||
        region_elems(c, s2_id, s2_off, len, sizeof(Fp2), &s2))
        return -1;
    const Fp2* p = static_cast<const Fp2*>(pt);
    const size_t tmp = eq_tmp_entries(static_cast<int>(n_vars));
    if (tmp && ensure_ws(c, kWsScratch, tmp * sizeof(Fp2))) return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    const Fp2 scale{1, 0};
    Fp2* contrib = static_cast<Fp2*>(s1);
    if (eq_table(c, p, static_cast<int>(n_vars), scale, contrib, ws<Fp2>(c, kWsScratch), nullptr,
                 p + n_vars))
        return -1;
    if (initialize) {
        VZB_CUDA(c, cudaMemcpyAsync(target, contrib, len * sizeof(Fp2), cudaMemcpyDeviceToDevice, c->stream));
    } else {
        add_inplace_kernel<<<grid_for(c, len, 256), 256, 0, c->stream>>>(static_cast<Fp2*>(target), contrib, len);
        VZB_LAUNCHED(c);
    }
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpGemm, 0, 0);
}

extern "C" int volta_cuda_fp2_add_inplace_device(void* raw, uint64_t t_id, size_t t_off,
                                                 uint64_t a_id, size_t a_off, size_t n) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !n) return fail_message(c, "invalid resident Fp2 add");
    void *t = nullptr, *a = nullptr;
    if (region_elems(c, t_id, t_off, n, sizeof(Fp2), &t) || region_elems(c, a_id, a_off, n, sizeof(Fp2), &a))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    add_inplace_kernel<<<grid_for(c, n, 256), 256, 0, c->stream>>>(static_cast<Fp2*>(t),
                                                                   static_cast<const Fp2*>(a), n);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpPcsRows, 0, 0);
}

extern "C" int volta_cuda_fp2_mobius_inverse_inplace_device(void* raw, uint64_t v_id, size_t v_off,
                                                            size_t n) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !n || (n & (n - 1))) return fail_message(c, "invalid resident Fp2 Mobius inverse");
    void* v = nullptr;
    if (region_elems(c, v_id, v_off, n, sizeof(Fp2), &v)) return -1;
    Fp2* values = static_cast<Fp2*>(v);
    if (op_begin(c) || op_mark(c, 1)) return -1;
    if (n > 1) {
        const size_t tile = n < kEqTile ? n : kEqTile;
        mobius_tile_kernel<<<static_cast<unsigned>(n / tile), 256, 0, c->stream>>>(values, n);
        VZB_LAUNCHED(c);
        for (size_t stride = tile; stride < n; stride <<= 1) {
            mobius_stage_kernel<<<grid_for(c, n / 2, 256), 256, 0, c->stream>>>(values, n / 2, stride);
            VZB_LAUNCHED(c);
        }
    }
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpPcsRows, 0, 0);
}

extern "C" int volta_cuda_fp2_affine_eq_weights_inplace_device(void* raw, uint64_t v_id, size_t n,
                                                               size_t source_count,
                                                               uint64_t point_id, size_t point_off,
                                                               size_t point_len, uint64_t rho_c0,
                                                               uint64_t rho_c1, uint64_t gamma_c0,
                                                               uint64_t gamma_c1) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !n || (n & (n - 1)) || !point_len || point_len >= 8 * sizeof(size_t) ||
        n != (size_t{1} << point_len) || source_count > n)
        return fail_message(c, "invalid resident Fp2 affine equality weights");
    void *v = nullptr, *pt = nullptr;
    if (region(c, v_id, 0, n * sizeof(Fp2), &v) ||
        region_elems(c, point_id, point_off, point_len, sizeof(Fp2), &pt))
        return -1;
    const size_t tmp = eq_tmp_entries(static_cast<int>(point_len)) + n;
    if (ensure_ws(c, kWsScratch2, tmp * sizeof(Fp2))) return -1;
    Fp2* eqv = ws<Fp2>(c, kWsScratch2);
    if (op_begin(c) || op_mark(c, 1)) return -1;
    if (eq_table(c, static_cast<const Fp2*>(pt), static_cast<int>(point_len), Fp2{1, 0}, eqv, eqv + n)) return -1;
    affine_eq_kernel<<<grid_for(c, n, 256), 256, 0, c->stream>>>(static_cast<Fp2*>(v), eqv, n, source_count,
                                                                 Fp2{rho_c0, rho_c1}, Fp2{gamma_c0, gamma_c1});
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpPcsRows, 0, 0);
}

extern "C" int volta_cuda_fp2_row_dots_device(void* raw, uint64_t a_id, size_t a_off, size_t a_stride,
                                              uint64_t b_id, size_t b_off, size_t b_stride,
                                              uint64_t out_id, size_t out_off, size_t rows,
                                              size_t len) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !rows || !len || a_stride < len || b_stride < len)
        return fail_message(c, "invalid Fp2 row-dot geometry");
    size_t aob = 0, asb = 0, bob = 0, bsb = 0, oob = 0, ob = 0, rb = 0;
    if (!mul_ok(a_off, sizeof(Fp2), &aob) || !mul_ok(a_stride, sizeof(Fp2), &asb) ||
        !mul_ok(b_off, sizeof(Fp2), &bob) || !mul_ok(b_stride, sizeof(Fp2), &bsb) ||
        !mul_ok(out_off, sizeof(Fp2), &oob) || !mul_ok(len, sizeof(Fp2), &rb) ||
        !mul_ok(rows, sizeof(Fp2), &ob))
        return fail_message(c, "Fp2 row-dot geometry overflows size_t");
    void *a = nullptr, *b = nullptr, *out = nullptr;
    size_t aspan = 0, bspan = 0;
    if (strided_region(c, a_id, aob, asb, rb, rows, &a, &aspan) ||
        strided_region(c, b_id, bob, bsb, rb, rows, &b, &bspan) || region(c, out_id, oob, ob, &out))
        return -1;
    size_t oe = 0, ae = 0, be = 0;
    if (!add_ok(oob, ob, &oe) || !add_ok(aob, aspan, &ae) || !add_ok(bob, bspan, &be))
        return fail_message(c, "Fp2 row-dot envelope overflows size_t");
    if ((out_id == a_id && oob < ae && aob < oe) || (out_id == b_id && oob < be && bob < oe))
        return fail_message(c, "Fp2 row-dot output overlaps an input");
    if (op_begin(c) || op_mark(c, 1)) return -1;
    const unsigned blocks = static_cast<unsigned>(std::min<size_t>(rows, 65535));
    row_dots_kernel<<<blocks, 256, 0, c->stream>>>(static_cast<const Fp2*>(a), a_stride,
                                                   static_cast<const Fp2*>(b), b_stride,
                                                   static_cast<Fp2*>(out), rows, len);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpPcsRows, 0, 0);
}

extern "C" int volta_cuda_fp2_powers_device(void* raw, uint64_t base_c0, uint64_t base_c1,
                                            uint64_t out_id, size_t out_off, size_t count) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !count || base_c0 >= kP || base_c1 >= kP) return fail_message(c, "invalid Fp2 powers input");
    void* out = nullptr;
    if (region_elems(c, out_id, out_off, count, sizeof(Fp2), &out)) return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    powers_kernel<<<grid_for(c, count, 256), 256, 0, c->stream>>>(Fp2{base_c0, base_c1},
                                                                  static_cast<Fp2*>(out), count);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpPcsRows, 0, 0, 0, 0, count * sizeof(Fp2));
}

// ===========================================================================
// Extensions (include/volta_b200_ext.h): fused fold + next round
// ===========================================================================

static int triple_fold_round(Context* c, uint64_t a_id, uint64_t b_id, uint64_t c_id, size_t len, Fp2 r,
                             uint64_t ao_id, uint64_t bo_id, uint64_t co_id, Fp2* host, uint64_t out_id,
                             size_t out_off) {
    if (!c || (!host && !out_id) || len < 4 || (len & 3))
        return fail_message(c, "invalid fused triple fold-round geometry");
    void *a = nullptr, *b = nullptr, *cc = nullptr, *ao = nullptr, *bo = nullptr, *co = nullptr, *dev = nullptr;
    if (region_elems(c, a_id, 0, len, sizeof(Fp2), &a) || region_elems(c, b_id, 0, len, sizeof(Fp2), &b) ||
        region_elems(c, c_id, 0, len, sizeof(Fp2), &cc) || region_elems(c, ao_id, 0, len / 2, sizeof(Fp2), &ao) ||
        region_elems(c, bo_id, 0, len / 2, sizeof(Fp2), &bo) || region_elems(c, co_id, 0, len / 2, sizeof(Fp2), &co))
        return -1;
    if (!host && region_elems(c, out_id, out_off, 3, sizeof(Fp2), &dev)) return -1;
    const MsgOut o = msg_out(c, static_cast<Fp2*>(dev), host, 3);
    if (op_begin(c) || op_mark(c, 1)) return -1;
    TripleFoldEval ev{static_cast<const Fp2*>(a), static_cast<const Fp2*>(b), static_cast<const Fp2*>(cc),
                      static_cast<Fp2*>(ao), static_cast<Fp2*>(bo), static_cast<Fp2*>(co), r};
    if (launch_reduce_wide<3>(c, ev, len / 4, store_epi<3>(o), 8)) return -1;
    return finish_msg(c, kOpGemm, o);
}

static int logup_fold_round(Context* c, const uint64_t in_ids[4], size_t len, Fp2 r, const uint64_t out_ids[4],
                            uint64_t s_id, size_t s_off, Fp2* host, uint64_t out_id, size_t out_off) {
    if (!c || (!host && !out_id) || len < 4 || (len & 3))
        return fail_message(c, "invalid fused LogUp fold-round geometry");
    void* in[4];
    void* out[4];
    void *s = nullptr, *dev = nullptr;
    for (int k = 0; k < 4; ++k)
        if (region_elems(c, in_ids[k], 0, len, sizeof(Fp2), &in[k]) ||
            region_elems(c, out_ids[k], 0, len / 2, sizeof(Fp2), &out[k]))
            return -1;
    if (region_elems(c, s_id, s_off, len / 4, sizeof(Fp2), &s)) return -1;
    if (!host && region_elems(c, out_id, out_off, 4, sizeof(Fp2), &dev)) return -1;
    const MsgOut o = msg_out(c, static_cast<Fp2*>(dev), host, 4);
    if (op_begin(c) || op_mark(c, 1)) return -1;
    LogupFoldEval ev{static_cast<const Fp2*>(in[0]), static_cast<const Fp2*>(in[1]), static_cast<const Fp2*>(in[2]),
                     static_cast<const Fp2*>(in[3]), static_cast<const Fp2*>(s), static_cast<Fp2*>(out[0]),
                     static_cast<Fp2*>(out[1]), static_cast<Fp2*>(out[2]), static_cast<Fp2*>(out[3]), r};
    if (launch_reduce_wide<4>(c, ev, len / 4, store_epi<4>(o))) return -1;
    return finish_msg(c, kOpLogup, o);
}

extern "C" int volta_b200_triple_fold_round_device(void* raw, uint64_t a_id, uint64_t b_id, uint64_t c_id,
                                                   size_t len, Fp2 r, uint64_t ao_id, uint64_t bo_id,
                                                   uint64_t co_id, Fp2* output) {
    Context* c = static_cast<Context*>(raw);
    if (!output) return fail_message(c, "invalid fused triple fold-round geometry");
    return triple_fold_round(c, a_id, b_id, c_id, len, r, ao_id, bo_id, co_id, output, 0, 0);
}

extern "C" int volta_b200_triple_fold_round_into_device(void* raw, uint64_t a_id, uint64_t b_id, uint64_t c_id,
                                                        size_t len, Fp2 r, uint64_t ao_id, uint64_t bo_id,
                                                        uint64_t co_id, uint64_t out_id, size_t out_offset) {
    return triple_fold_round(static_cast<Context*>(raw), a_id, b_id, c_id, len, r, ao_id, bo_id, co_id, nullptr,
                             out_id, out_offset);
}

extern "C" int volta_b200_product_fold_round_into_device(void* raw, uint64_t a_id, uint64_t b_id, size_t len, Fp2 r,
                                                         uint64_t ao_id, uint64_t bo_id, uint64_t out_id,
                                                         size_t out_offset) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !out_id || len < 4 || (len & 3)) return fail_message(c, "invalid fused product fold-round geometry");
    void *a = nullptr, *b = nullptr, *ao = nullptr, *bo = nullptr, *dev = nullptr;
    if (region_elems(c, a_id, 0, len, sizeof(Fp2), &a) || region_elems(c, b_id, 0, len, sizeof(Fp2), &b) ||
        region_elems(c, ao_id, 0, len / 2, sizeof(Fp2), &ao) || region_elems(c, bo_id, 0, len / 2, sizeof(Fp2), &bo) ||
        region_elems(c, out_id, out_offset, 2, sizeof(Fp2), &dev))
        return -1;
    const MsgOut o = msg_out(c, static_cast<Fp2*>(dev), nullptr, 2);
    if (op_begin(c) || op_mark(c, 1)) return -1;
    ProductFoldEval ev{static_cast<const Fp2*>(a), static_cast<const Fp2*>(b), static_cast<Fp2*>(ao),
                       static_cast<Fp2*>(bo), r};
    if (launch_reduce_wide<2>(c, ev, len / 4, store_epi<2>(o), 8)) return -1;
    return finish_msg(c, kOpGemm, o);
}

// Triple-product rounds on base-field tables (extensions).
extern "C" int volta_b200_triple_round_fp_into_device(void* raw, uint64_t a_id, uint64_t b_id, uint64_t c_id,
                                                      size_t pairs, uint64_t out_id, size_t out_offset) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !pairs) return fail_message(c, "invalid base-field triple round geometry");
    void *a = nullptr, *b = nullptr, *cc = nullptr, *dev = nullptr;
    if (region_elems(c, a_id, 0, 2 * pairs, sizeof(uint64_t), &a) ||
        region_elems(c, b_id, 0, 2 * pairs, sizeof(uint64_t), &b) ||
        region_elems(c, c_id, 0, 2 * pairs, sizeof(uint64_t), &cc) ||
        region_elems(c, out_id, out_offset, 3, sizeof(Fp2), &dev))
        return -1;
    const MsgOut o = msg_out(c, static_cast<Fp2*>(dev), nullptr, 3);
    if (op_begin(c) || op_mark(c, 1)) return -1;
    TripleEvalFp ev{static_cast<const uint64_t*>(a), static_cast<const uint64_t*>(b), static_cast<const uint64_t*>(cc)};
    if (launch_reduce_wide<3>(c, ev, pairs, store_epi<3>(o), 8)) return -1;
    return finish_msg(c, kOpGemm, o);
}

extern "C" int volta_b200_triple_fold_round_fp_into_device(void* raw, uint64_t a_id, uint64_t b_id, uint64_t c_id,
                                                           size_t len, Fp2 r, uint64_t ao_id, uint64_t bo_id,
                                                           uint64_t co_id, uint64_t out_id, size_t out_offset) {
    Context* c = static_cast<Context*>(raw);
    if (!c || len < 4 || (len & 3)) return fail_message(c, "invalid base-field triple fold-round geometry");
    if (r.c0 >= kP || r.c1 >= kP) return fail_message(c, "triple fold-round challenge is not canonical");
    void *a = nullptr, *b = nullptr, *cc = nullptr, *ao = nullptr, *bo = nullptr, *co = nullptr, *dev = nullptr;
    if (region_elems(c, a_id, 0, len, sizeof(uint64_t), &a) || region_elems(c, b_id, 0, len, sizeof(uint64_t), &b) ||
        region_elems(c, c_id, 0, len, sizeof(uint64_t), &cc) || region_elems(c, ao_id, 0, len / 2, sizeof(Fp2), &ao) ||
        region_elems(c, bo_id, 0, len / 2, sizeof(Fp2), &bo) || region_elems(c, co_id, 0, len / 2, sizeof(Fp2), &co) ||
        region_elems(c, out_id, out_offset, 3, sizeof(Fp2), &dev))
        return -1;
    const MsgOut o = msg_out(c, static_cast<Fp2*>(dev), nullptr, 3);
    if (op_begin(c) || op_mark(c, 1)) return -1;
    TripleFoldEvalFp ev{static_cast<const uint64_t*>(a), static_cast<const uint64_t*>(b),
                        static_cast<const uint64_t*>(cc), static_cast<Fp2*>(ao), static_cast<Fp2*>(bo),
                        static_cast<Fp2*>(co), r};
    if (launch_reduce_wide<3>(c, ev, len / 4, store_epi<3>(o), 8)) return -1;
    return finish_msg(c, kOpGemm, o);
}

extern "C" int volta_b200_logup_fold_round_device(void* raw, uint64_t p0_id, uint64_t p1_id, uint64_t q0_id,
                                                  uint64_t q1_id, size_t len, Fp2 r, uint64_t o0_id,
                                                  uint64_t o1_id, uint64_t o2_id, uint64_t o3_id,
                                                  uint64_t s_id, size_t s_off, Fp2* output) {
    Context* c = static_cast<Context*>(raw);
    if (!output) return fail_message(c, "invalid fused LogUp fold-round geometry");
    const uint64_t in[4] = {p0_id, p1_id, q0_id, q1_id}, out[4] = {o0_id, o1_id, o2_id, o3_id};
    return logup_fold_round(c, in, len, r, out, s_id, s_off, output, 0, 0);
}

extern "C" int volta_b200_logup_fold_round_into_device(void* raw, uint64_t p0_id, uint64_t p1_id, uint64_t q0_id,
                                                       uint64_t q1_id, size_t len, Fp2 r, uint64_t o0_id,
                                                       uint64_t o1_id, uint64_t o2_id, uint64_t o3_id,
                                                       uint64_t s_id, size_t s_off, uint64_t out_id,
                                                       size_t out_offset) {
    const uint64_t in[4] = {p0_id, p1_id, q0_id, q1_id}, out[4] = {o0_id, o1_id, o2_id, o3_id};
    return logup_fold_round(static_cast<Context*>(raw), in, len, r, out, s_id, s_off, nullptr, out_id,
                            out_offset);
}

// Every round of a general LogUp sumcheck with the challenges known in
// advance (the rounds of logup.rs:427-471 run_general_rounds; the GPU loop
// of cuda/p7_logup_blind_rounds.cu:403-431): round 0's message over the
// inputs, then per round j >= 1 one fused pass that folds level j-1 with
// r[j-1] into level j of the caller's ladder and reduces round j's message,
// and a last plain fold of the two-entry level into the four final values.
// log2(len) + 1 launches, no host wait; the message of round j reads the
// suffix table's first len >> (j + 1) entries.
extern "C" int volta_b200_logup_rounds_device(void* raw, uint64_t p0_id, uint64_t p1_id, uint64_t q0_id,
                                              uint64_t q1_id, size_t len, uint64_t s_id, size_t s_off,
                                              const Fp2* r, uint64_t l0_id, uint64_t l1_id, uint64_t l2_id,
                                              uint64_t l3_id, uint64_t out_id, size_t out_offset) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !r || len < 2 || (len & (len - 1))) return fail_message(c, "invalid LogUp rounds geometry");
    int L = 0;
    while ((size_t{1} << L) < len) ++L;
    for (int j = 0; j < L; ++j)
        if (r[j].c0 >= kP || r[j].c1 >= kP) return fail_message(c, "LogUp rounds challenge is not canonical");
    const uint64_t in_ids[4] = {p0_id, p1_id, q0_id, q1_id}, lad_ids[4] = {l0_id, l1_id, l2_id, l3_id};
    const Fp2* in[4];
    Fp2* lad[4] = {nullptr, nullptr, nullptr, nullptr};
    void *p = nullptr, *s = nullptr, *out = nullptr;
    for (int k = 0; k < 4; ++k) {
        if (region_elems(c, in_ids[k], 0, len, sizeof(Fp2), &p)) return -1;
        in[k] = static_cast<const Fp2*>(p);
        if (len > 2) {
            if (region_elems(c, lad_ids[k], 0, len - 2, sizeof(Fp2), &p)) return -1;
            lad[k] = static_cast<Fp2*>(p);
        }
    }
    if (region_elems(c, s_id, s_off, len / 2, sizeof(Fp2), &s) ||
        region_elems(c, out_id, out_offset, 4 * size_t(L) + 4, sizeof(Fp2), &out))
        return -1;
    Fp2* msg = static_cast<Fp2*>(out);
    const Fp2* suffix = static_cast<const Fp2*>(s);
    if (op_begin(c) || op_mark(c, 1)) return -1;
    if (logup_round(c, in[0], in[1], in[2], in[3], suffix, len / 2, msg_out(c, msg, nullptr, 4))) return -1;
    const Fp2* src[4] = {in[0], in[1], in[2], in[3]};
    for (int j = 1; j < L; ++j) {
        const size_t cur = len >> (j - 1), at = len - 2 * (len >> j);  // level j at ladder offset `at`
        Fp2* dst[4];
        for (int k = 0; k < 4; ++k) dst[k] = lad[k] + at;
        LogupFoldEval ev{src[0], src[1], src[2], src[3], suffix, dst[0], dst[1], dst[2], dst[3], r[j - 1]};
        if (launch_reduce_wide<4>(c, ev, cur / 4, store_epi<4>(msg_out(c, msg + 4 * j, nullptr, 4)))) return -1;
        for (int k = 0; k < 4; ++k) src[k] = dst[k];
    }
    Quad q{};
    for (int k = 0; k < 4; ++k) {
        q.in[k] = src[k];
        q.out[k] = msg + 4 * L + k;
    }
    fold4_kernel<<<1, 32, 0, c->stream>>>(q, 1, r[L - 1]);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpLogup, 0, 0);
}

// ===========================================================================
// Extensions: LogUp layer rounds straight from interleaved tree children
// ===========================================================================

extern "C" int volta_b200_logup_round_il_into_device(void* raw, uint64_t p_id, uint64_t q_id, size_t child_offset,
                                                     size_t vector_len, uint64_t s_id, size_t s_off, uint64_t out_id,
                                                     size_t out_offset) {
    Context* c = static_cast<Context*>(raw);
    if (!c || vector_len < 2 || (vector_len & 1)) return fail_message(c, "invalid interleaved LogUp round geometry");
    void *P = nullptr, *Q = nullptr, *S = nullptr, *dev = nullptr;
    if (region_elems(c, p_id, child_offset, 2 * vector_len, sizeof(Fp2), &P) ||
        region_elems(c, q_id, child_offset, 2 * vector_len, sizeof(Fp2), &Q) ||
        region_elems(c, s_id, s_off, vector_len / 2, sizeof(Fp2), &S) ||
        region_elems(c, out_id, out_offset, 4, sizeof(Fp2), &dev))
        return -1;
    const MsgOut o = msg_out(c, static_cast<Fp2*>(dev), nullptr, 4);
    if (op_begin(c) || op_mark(c, 1)) return -1;
    LogupEvalIL ev{static_cast<const Fp2*>(P), static_cast<const Fp2*>(Q), static_cast<const Fp2*>(S)};
    if (launch_reduce_wide<4>(c, ev, vector_len / 2, store_epi<4>(o))) return -1;
    return finish_msg(c, kOpLogup, o);
}

extern "C" int volta_b200_logup_fold_round_il_into_device(void* raw, uint64_t p_id, uint64_t q_id,
                                                          size_t child_offset, size_t vector_len, Fp2 r,
                                                          uint64_t o0_id, uint64_t o1_id, uint64_t o2_id,
                                                          uint64_t o3_id, uint64_t s_id, size_t s_off,
                                                          uint64_t out_id, size_t out_offset) {
    Context* c = static_cast<Context*>(raw);
    if (!c || vector_len < 4 || (vector_len & 3))
        return fail_message(c, "invalid interleaved LogUp fold-round geometry");
    void *P = nullptr, *Q = nullptr, *S = nullptr, *dev = nullptr;
    void* o[4];
    const uint64_t oid[4] = {o0_id, o1_id, o2_id, o3_id};
    if (region_elems(c, p_id, child_offset, 2 * vector_len, sizeof(Fp2), &P) ||
        region_elems(c, q_id, child_offset, 2 * vector_len, sizeof(Fp2), &Q) ||
        region_elems(c, s_id, s_off, vector_len / 4, sizeof(Fp2), &S) ||
        region_elems(c, out_id, out_offset, 4, sizeof(Fp2), &dev))
        return -1;
    for (int k = 0; k < 4; ++k)
        if (region_elems(c, oid[k], 0, vector_len / 2, sizeof(Fp2), &o[k])) return -1;
    const MsgOut m = msg_out(c, static_cast<Fp2*>(dev), nullptr, 4);
    if (op_begin(c) || op_mark(c, 1)) return -1;
    LogupFoldEvalIL ev{static_cast<const Fp2*>(P), static_cast<const Fp2*>(Q), static_cast<const Fp2*>(S),
                       static_cast<Fp2*>(o[0]), static_cast<Fp2*>(o[1]), static_cast<Fp2*>(o[2]),
                       static_cast<Fp2*>(o[3]), r};
    if (launch_reduce_wide<4>(c, ev, vector_len / 4, store_epi<4>(m))) return -1;
    return finish_msg(c, kOpLogup, m);
}

// ===========================================================================
// Extension: round steps of several fraction-tree layers in one launch
// ===========================================================================

// Round terms when every numerator entry is 1 (a = b = 1 at every point):
// a d + b c = c + d, so the two inner products per point disappear.
// c0, c1, d0, d1 canonical.
__device__ __forceinline__ void q_round_terms(Fp2 c0, Fp2 c1, Fp2 d0, Fp2 d1, Fp2 si, Fp2W* w) {
    const Fp2 t0 = d2add(c0, d0), t1 = d2add(c1, d1);
    const Fp2 t2 = d2add_weak(t1, d2sub(t1, t0));  // (c2 + d2) = 2 (c1 + d1) - (c0 + d0)
    const Fp2 c2 = d2add_weak(c1, d2sub(c1, c0)), d2 = d2add_weak(d1, d2sub(d1, d0));
    f2w_mac(w[0], si, t0);
    f2w_mac(w[1], si, t2);
    f2w_mac(w[2], si, d2mul(c0, d0));
    f2w_mac(w[3], si, d2mul(c2, d2));
}

// kind 0 with all-one numerators: only the Q children are read
struct QEvalIL {
    const Fp2 *Q, *s;
    __device__ __forceinline__ void operator()(size_t i, Fp2W* w) const {
        const Fp2 c0 = ldcs2(Q + 4 * i), d0 = ldcs2(Q + 4 * i + 1), c1 = ldcs2(Q + 4 * i + 2), d1 = ldcs2(Q + 4 * i + 3);
        q_round_terms(c0, c1, d0, d1, ldg2(s + i), w);
    }
};

// kind 1 with all-one numerators: folds and writes q0, q1 only
struct QFoldEvalIL {
    const Fp2 *Q, *s;
    Fp2 *o2, *o3;
    Fp2 r;
    __device__ __forceinline__ void operator()(size_t i, Fp2W* w) const {
        Fp2 y[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) y[k] = ldcs2(Q + 8 * i + k);
        const Fp2 c0 = d2fold(y[0], y[2], r), c1 = d2fold(y[4], y[6], r);
        const Fp2 d0 = d2fold(y[1], y[3], r), d1 = d2fold(y[5], y[7], r);
        st2(o2 + 2 * i, c0);
        st2(o2 + 2 * i + 1, c1);
        st2(o3 + 2 * i, d0);
        st2(o3 + 2 * i + 1, d1);
        q_round_terms(c0, c1, d0, d1, ldg2(s + i), w);
    }
};

// kind 0 with the parents given: the t = 0 terms a0 d0 + b0 c0 and c0 d0 of
// pair i are the parent node 2 i's p and q (its tree level PP, PQ).
struct LogupEvalILPar {
    const Fp2 *P, *Q, *s, *PP, *PQ;
    __device__ __forceinline__ void operator()(size_t i, Fp2W* w) const {
        const Fp2 a0 = ldcs2(P + 4 * i), b0 = ldcs2(P + 4 * i + 1), a1 = ldcs2(P + 4 * i + 2), b1 = ldcs2(P + 4 * i + 3);
        const Fp2 c0 = ldcs2(Q + 4 * i), d0 = ldcs2(Q + 4 * i + 1), c1 = ldcs2(Q + 4 * i + 2), d1 = ldcs2(Q + 4 * i + 3);
        const Fp2 si = ldg2(s + i), pp = ldcs2(PP + 2 * i), pq = ldcs2(PQ + 2 * i);
        const Fp2 a2 = d2add_weak(a1, d2sub(a1, a0)), b2 = d2add_weak(b1, d2sub(b1, b0));
        const Fp2 c2 = d2add_weak(c1, d2sub(c1, c0)), d2 = d2add_weak(d1, d2sub(d1, d0));
        Fp2W t;
        f2w_zero(t);
        f2w_mac(t, a2, d2);
        f2w_mac(t, b2, c2);
        f2w_mac(w[0], si, pp);
        f2w_mac(w[1], si, f2w_reduce(t));
        f2w_mac(w[2], si, pq);
        f2w_mac(w[3], si, d2mul(c2, d2));
    }
};

// Leaf-layer children read from the query column: child j's denominator is
// (a0 - f_j, a1).  The product of two such values is
// (x y + 7 a1^2, a1 (x + y)): two base products instead of an Fp2 product.
__device__ __forceinline__ Fp2 leaf_q_mul(uint64_t x, uint64_t y, uint64_t a1, uint64_t w7a1sq) {
    return Fp2{dadd(dmul(x, y), w7a1sq), dmul(a1, dadd(x, y))};
}

// kind 0, all-one numerators, children from the query column
struct QColEvalIL {
    const uint64_t* f;
    const Fp2* s;
    uint64_t a0, a1, w7a1sq;
    __device__ __forceinline__ void operator()(size_t i, Fp2W* w) const {
        const uint64_t x0 = dsub(a0, __ldcs(f + 4 * i)), x1 = dsub(a0, __ldcs(f + 4 * i + 1));
        const uint64_t x2 = dsub(a0, __ldcs(f + 4 * i + 2)), x3 = dsub(a0, __ldcs(f + 4 * i + 3));
        // c = q0 = (x0, x2), d = q1 = (x1, x3); every c1 part is a1, every t c1 part 2 a1
        const uint64_t two_a1 = dadd(a1, a1);
        const uint64_t t0 = dadd(x0, x1), t1 = dadd(x2, x3);
        const uint64_t t2 = dadd(t1, dsub(t1, t0));
        const uint64_t c2 = dadd(x2, dsub(x2, x0)), d2 = dadd(x3, dsub(x3, x1));
        const Fp2 si = ldg2(s + i);
        f2w_mac(w[0], si, Fp2{t0, two_a1});
        f2w_mac(w[1], si, Fp2{t2, two_a1});
        f2w_mac(w[2], si, leaf_q_mul(x0, x1, a1, w7a1sq));
        f2w_mac(w[3], si, leaf_q_mul(c2, d2, a1, w7a1sq));
    }
};

// kind 1, all-one numerators, children from the query column: the folds of
// (xa, a1), (xb, a1) are (xa + r.c0 d, a1 + r.c1 d), d = xb - xa in Fp
struct QColFoldEvalIL {
    const uint64_t* f;
    const Fp2* s;
    Fp2 *o2, *o3;
    Fp2 r;
    uint64_t a0, a1;
    __device__ __forceinline__ Fp2 fold(uint64_t xa, uint64_t xb) const {
        const uint64_t d = dsub(xb, xa);
        return Fp2{dadd(xa, dmul(r.c0, d)), dadd(a1, dmul(r.c1, d))};
    }
    __device__ __forceinline__ void operator()(size_t i, Fp2W* w) const {
        uint64_t x[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) x[k] = dsub(a0, __ldcs(f + 8 * i + k));
        const Fp2 c0 = fold(x[0], x[2]), c1 = fold(x[4], x[6]);
        const Fp2 d0 = fold(x[1], x[3]), d1 = fold(x[5], x[7]);
        st2(o2 + 2 * i, c0);
        st2(o2 + 2 * i + 1, c1);
        st2(o3 + 2 * i, d0);
        st2(o3 + 2 * i + 1, d1);
        q_round_terms(c0, c1, d0, d1, ldg2(s + i), w);
    }
};

// kind 2 with all-one numerators
struct QFoldEval {
    const Fp2 *q0, *q1, *s;
    Fp2 *o2, *o3;
    Fp2 r;
    __device__ __forceinline__ void operator()(size_t i, Fp2W* w) const {
        Fp2 c0, c1, d0, d1;
        fold4_pair(q0, o2, i, r, c0, c1);
        fold4_pair(q1, o3, i, r, d0, d1);
        q_round_terms(c0, c1, d0, d1, ldg2(s + i), w);
    }
};

namespace {

constexpr int kBatchJobs = 24;
constexpr unsigned kBatchCounterBase = 64;  // per-job counters in the counter workspace

enum BatchKind : uint32_t { kBatchRoundIL = 0, kBatchFoldRoundIL = 1, kBatchFoldRound = 2, kBatchFold = 3 };

struct BatchJob {
    uint32_t kind;
    uint32_t p_one;           // numerators all 1: not read, not written (kind 3 writes ones)
    uint32_t q_col;           // children are (a0 - f_j, a1) from the column `col`
    uint32_t parents;         // kind 0: the parent level is given (pp, pq)
    const Fp2 *pp, *pq;
    const uint64_t* col;
    uint64_t a0, a1, w7a1sq;
    uint32_t block0, blocks;  // CTA range [block0, block0 + blocks)
    size_t items;
    const Fp2 *in0, *in1, *in2, *in3;
    Fp2 *out0, *out1, *out2, *out3;
    const Fp2* s;
    Fp2 r;
    Fp2* msg;
};

struct RoundBatch {
    BatchJob job[kBatchJobs];
    uint32_t count;
};

// Grid reduction over the `blocks` CTAs of one job (bidx = this CTA's index
// within the job): the same last-CTA-finishes scheme as grid_finish.
template <int K, class Epi>
__device__ __forceinline__ void job_finish(Acc<K> a, Fp2* partials, unsigned* counter, unsigned blocks,
                                           unsigned bidx, const Epi& epi) {
    a = block_sum<K>(a);
    if (blocks == 1) {
        if (threadIdx.x == 0) epi(a);
        return;
    }
    __shared__ bool last;
    if (threadIdx.x == 0) {
#pragma unroll
        for (int k = 0; k < K; ++k) st2(partials + static_cast<size_t>(bidx) * K + k, a.v[k]);
        __threadfence();
        last = atomicAdd(counter, 1u) == blocks - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    Acc<K> t;
    t.zero();
    for (unsigned b = threadIdx.x; b < blocks; b += blockDim.x) {
#pragma unroll
        for (int k = 0; k < K; ++k) {
            const ulonglong2 v = __ldcg(reinterpret_cast<const ulonglong2*>(partials + static_cast<size_t>(b) * K + k));
            t.v[k] = f2add(t.v[k], Fp2{v.x, v.y});
        }
    }
    t = block_sum<K>(t);
    if (threadIdx.x == 0) {
        epi(t);
        *counter = 0;
    }
}

struct MsgStoreEpi {
    Fp2* out;
    __device__ __forceinline__ void operator()(const Acc<4>& a) const {
#pragma unroll
        for (int k = 0; k < 4; ++k) out[k] = a.v[k];
    }
};

// CTA b runs the job whose range holds b: a grid-stride loop over that
// job's items with the job's own CTA count as the stride, then the job's
// grid reduction.  Fold-only jobs skip the reduction.  One instantiation per
// job class, so that each class gets its own register allocation:
//   kBatchRound0   kind 0 (round 0 on interleaved children); its evaluators
//                  fit 96 registers, so five 128-thread CTAs (20 warps)
//                  share an SM;
//   kBatchFoldIL   kind 1 (fold 0 + round 1 on interleaved children);
//   kBatchFoldRun  kinds 2 and 3 (fold j + round j + 1, fold only).
enum BatchClass : int { kBatchRound0 = 0, kBatchFoldIL = 1, kBatchFoldRun = 2 };
constexpr unsigned kRound0Threads = 128;
constexpr unsigned kRound0Ctas = 5;

__host__ __device__ constexpr int batch_class(uint32_t kind) {
    return kind == kBatchRoundIL ? kBatchRound0 : kind == kBatchFoldRoundIL ? kBatchFoldIL : kBatchFoldRun;
}

template <int kClass>
__global__ void __launch_bounds__(kClass == kBatchRound0 ? kRound0Threads : kReduceThreads,
                                  kClass == kBatchRound0 ? kRound0Ctas : 2)
    logup_round_batch_kernel(const __grid_constant__ RoundBatch batch, Fp2* partials, unsigned* counters) {
    unsigned j = 0;
    while (j + 1 < batch.count && blockIdx.x >= batch.job[j + 1].block0) ++j;
    const BatchJob& jb = batch.job[j];
    const unsigned bidx = blockIdx.x - jb.block0;
    const size_t stride = static_cast<size_t>(jb.blocks) * blockDim.x;
    const size_t first = static_cast<size_t>(bidx) * blockDim.x + threadIdx.x;
    if (kClass == kBatchFoldRun && jb.kind == kBatchFold) {
        for (size_t i = first; i < jb.items; i += stride) {
            Fp2 x0, x1;
            if (jb.p_one) {
                const Fp2 one{1, 0};
                st2(jb.out0 + 2 * i, one);
                st2(jb.out0 + 2 * i + 1, one);
                st2(jb.out1 + 2 * i, one);
                st2(jb.out1 + 2 * i + 1, one);
            } else {
                fold4_pair(jb.in0, jb.out0, i, jb.r, x0, x1);
                fold4_pair(jb.in1, jb.out1, i, jb.r, x0, x1);
            }
            fold4_pair(jb.in2, jb.out2, i, jb.r, x0, x1);
            fold4_pair(jb.in3, jb.out3, i, jb.r, x0, x1);
        }
        return;
    }
    Fp2W w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) f2w_zero(w[k]);
    if (kClass == kBatchRound0) {
        if (jb.q_col) {
            const QColEvalIL ev{jb.col, jb.s, jb.a0, jb.a1, jb.w7a1sq};
            for (size_t i = first; i < jb.items; i += stride) ev(i, w);
        } else if (jb.p_one) {
            const QEvalIL ev{jb.in1, jb.s};
            for (size_t i = first; i < jb.items; i += stride) ev(i, w);
        } else if (jb.parents) {
            const LogupEvalILPar ev{jb.in0, jb.in1, jb.s, jb.pp, jb.pq};
            for (size_t i = first; i < jb.items; i += stride) ev(i, w);
        } else {
            const LogupEvalIL ev{jb.in0, jb.in1, jb.s};
            for (size_t i = first; i < jb.items; i += stride) ev(i, w);
        }
    } else if (kClass == kBatchFoldIL) {
        if (jb.q_col) {
            const QColFoldEvalIL ev{jb.col, jb.s, jb.out2, jb.out3, jb.r, jb.a0, jb.a1};
            for (size_t i = first; i < jb.items; i += stride) ev(i, w);
        } else if (jb.p_one) {
            const QFoldEvalIL ev{jb.in1, jb.s, jb.out2, jb.out3, jb.r};
            for (size_t i = first; i < jb.items; i += stride) ev(i, w);
        } else {
            const LogupFoldEvalIL ev{jb.in0, jb.in1, jb.s, jb.out0, jb.out1, jb.out2, jb.out3, jb.r};
            for (size_t i = first; i < jb.items; i += stride) ev(i, w);
        }
    } else if (jb.p_one) {
        const QFoldEval ev{jb.in2, jb.in3, jb.s, jb.out2, jb.out3, jb.r};
        for (size_t i = first; i < jb.items; i += stride) ev(i, w);
    } else {
        const LogupFoldEval ev{jb.in0, jb.in1, jb.in2, jb.in3, jb.s, jb.out0, jb.out1, jb.out2, jb.out3, jb.r};
        for (size_t i = first; i < jb.items; i += stride) ev(i, w);
    }
    Acc<4> acc;
#pragma unroll
    for (int k = 0; k < 4; ++k) acc.v[k] = f2w_reduce(w[k]);
    job_finish<4>(acc, partials + static_cast<size_t>(jb.block0) * 4, counters + j, jb.blocks, bidx,
                  MsgStoreEpi{jb.msg});
}

// One launch of the jobs of one class: CTAs in proportion to the items (at
// least one per job, at most one per thread block of items), two waves of
// the resident CTAs in all.
int launch_round_batch(Context* c, RoundBatch& batch, int cls) {
    size_t total = 0;
    for (uint32_t j = 0; j < batch.count; ++j) total += batch.job[j].items;
    const unsigned threads = cls == kBatchRound0 ? kRound0Threads : kReduceThreads;
    const size_t target = static_cast<size_t>(c->sm_count) * (cls == kBatchRound0 ? 2 * kRound0Ctas : 4);
    uint32_t next = 0;
    for (uint32_t j = 0; j < batch.count; ++j) {
        BatchJob& d = batch.job[j];
        const size_t need = (d.items + threads - 1) / threads;
        size_t share = (target * d.items + total - 1) / total;
        if (share < 1) share = 1;
        d.block0 = next;
        d.blocks = static_cast<uint32_t>(need < share ? need : share);
        next += d.blocks;
    }
    // partials: 4 Fp2 per CTA within the workspace (SMs x 8 CTAs x 9 Fp2)
    if (static_cast<size_t>(next) * 4 > static_cast<size_t>(c->sm_count) * 8 * 9)
        return fail_message(c, "LogUp round batch exceeds the reduction workspace");
    Fp2* partials = ws<Fp2>(c, kWsPartials);
    unsigned* counters = ws<unsigned>(c, kWsCounter) + kBatchCounterBase;
    if (cls == kBatchRound0)
        logup_round_batch_kernel<kBatchRound0><<<next, threads, 0, c->stream>>>(batch, partials, counters);
    else if (cls == kBatchFoldIL)
        logup_round_batch_kernel<kBatchFoldIL><<<next, threads, 0, c->stream>>>(batch, partials, counters);
    else
        logup_round_batch_kernel<kBatchFoldRun><<<next, threads, 0, c->stream>>>(batch, partials, counters);
    VZB_LAUNCHED(c);
    return 0;
}

}  // namespace

extern "C" int volta_b200_logup_round_batch_device(void* raw, const vzb_round_job* jobs, size_t count) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !jobs || !count || count > static_cast<size_t>(kBatchJobs))
        return fail_message(c, "invalid LogUp round batch (1 to 24 jobs)");
    RoundBatch batch{};
    batch.count = static_cast<uint32_t>(count);
    for (size_t j = 0; j < count; ++j) {
        const vzb_round_job& q = jobs[j];
        BatchJob& d = batch.job[j];
        const size_t len = q.len;
        d.kind = q.kind;
        if (q.kind > kBatchFold) return fail_message(c, "invalid LogUp round batch job kind");
        if (q.flags & ~(VZB_ROUND_P_ONE | VZB_ROUND_Q_COLUMN | VZB_ROUND_PARENTS))
            return fail_message(c, "invalid LogUp round batch job flags");
        if ((q.flags & VZB_ROUND_PARENTS) && (q.kind != kBatchRoundIL || (q.flags & VZB_ROUND_P_ONE)))
            return fail_message(c, "LogUp round batch: parents need kind 0 without all-one numerators");
        const bool one = (q.flags & VZB_ROUND_P_ONE) != 0;
        const bool qcol = (q.flags & VZB_ROUND_Q_COLUMN) != 0;
        if (qcol && (!one || q.kind > kBatchFoldRoundIL))
            return fail_message(c, "LogUp round batch: column children need all-one numerators and kind 0 or 1");
        if (qcol && (q.q_alpha[0] >= kP || q.q_alpha[1] >= kP))
            return fail_message(c, "LogUp round batch: leaf constants are not canonical");
        d.p_one = one ? 1u : 0u;
        d.q_col = qcol ? 1u : 0u;
        const bool il = q.kind <= kBatchFoldRoundIL, fold = q.kind != kBatchRoundIL;
        if (len < (fold ? 4u : 2u) || (len & (fold ? 3 : 1)))
            return fail_message(c, "invalid LogUp round batch job length");
        if (q.r[0] >= kP || q.r[1] >= kP) return fail_message(c, "LogUp round batch challenge is not canonical");
        d.r = Fp2{q.r[0], q.r[1]};
        void* p[4] = {nullptr, nullptr, nullptr, nullptr};
        // with all-one numerators P (kinds 0, 1) or p0, p1 (kinds 2, 3) are not read
        if (qcol) {  // the query column: 2 len u64 values (the children)
            void* col = nullptr;
            if (region_elems(c, q.in_id[1], q.in_offset[0], 2 * len, sizeof(uint64_t), &col)) return -1;
            d.col = static_cast<const uint64_t*>(col);
            d.a0 = q.q_alpha[0];
            d.a1 = q.q_alpha[1];
            d.w7a1sq = fmul7(fmul(q.q_alpha[1], q.q_alpha[1]));
        } else if (il) {
            for (int k = one ? 1 : 0; k < 2; ++k)
                if (region_elems(c, q.in_id[k], q.in_offset[0], 2 * len, sizeof(Fp2), &p[k])) return -1;
        } else {
            for (int k = one ? 2 : 0; k < 4; ++k)
                if (region_elems(c, q.in_id[k], q.in_offset[k], len, sizeof(Fp2), &p[k])) return -1;
        }
        d.in0 = static_cast<const Fp2*>(p[0]);
        d.in1 = static_cast<const Fp2*>(p[1]);
        d.in2 = static_cast<const Fp2*>(p[2]);
        d.in3 = static_cast<const Fp2*>(p[3]);
        if (fold) {
            void* o[4] = {nullptr, nullptr, nullptr, nullptr};
            // the numerator outputs are written only by kind 3 (ones)
            const int k0 = (one && q.kind != kBatchFold) ? 2 : 0;
            for (int k = k0; k < 4; ++k)
                if (region_elems(c, q.out_id[k], q.out_offset[k], len / 2, sizeof(Fp2), &o[k])) return -1;
            d.out0 = static_cast<Fp2*>(o[0]);
            d.out1 = static_cast<Fp2*>(o[1]);
            d.out2 = static_cast<Fp2*>(o[2]);
            d.out3 = static_cast<Fp2*>(o[3]);
        }
        d.items = fold ? len / 4 : len / 2;
        if (q.flags & VZB_ROUND_PARENTS) {
            void *pp = nullptr, *pq = nullptr;
            if (region_elems(c, q.out_id[0], q.out_offset[0], len, sizeof(Fp2), &pp) ||
                region_elems(c, q.out_id[1], q.out_offset[0], len, sizeof(Fp2), &pq))
                return -1;
            d.parents = 1;
            d.pp = static_cast<const Fp2*>(pp);
            d.pq = static_cast<const Fp2*>(pq);
        }
        if (q.kind != kBatchFold) {
            void *sv = nullptr, *mv = nullptr;
            if (region_elems(c, q.s_id, q.s_offset, d.items, sizeof(Fp2), &sv) ||
                region_elems(c, q.msg_id, q.msg_offset, 4, sizeof(Fp2), &mv))
                return -1;
            d.s = static_cast<const Fp2*>(sv);
            d.msg = static_cast<Fp2*>(mv);
        }
    }
    // one launch per job class present, in class order (a step of the
    // scheduled drivers holds one class, or kinds 2 and 3 together); the
    // launches run in stream order, so they share the partials and counters
    if (op_begin(c) || op_mark(c, 1)) return -1;
    for (int cls = kBatchRound0; cls <= kBatchFoldRun; ++cls) {
        RoundBatch sub{};
        for (uint32_t j = 0; j < batch.count; ++j)
            if (batch_class(batch.job[j].kind) == cls) sub.job[sub.count++] = batch.job[j];
        if (sub.count && launch_round_batch(c, sub, cls)) return -1;
    }
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpLogup, 0, 0);
}
