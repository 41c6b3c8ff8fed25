// Protocol drivers above the seam (clear sinks), restating the reference's
// resident callers call for call:
//   triple-product sumcheck  rust/volta-proto/src/hadamard.rs:186-260
//   LogUp prove              rust/volta-proto/src/logup.rs:1760-1771 (logup_prove)
//   resident engine          logup.rs:995-1090 (prove_engine_resident_from_device_leaves)
//   resident layer           logup.rs:1335-1470 (layer_general_resident)
//   clear sink               logup.rs:1601-1622 (lambda, per-round r, split t)
#include <utility>

#include "api.hpp"
#include "accel.hpp"
#include "protocol.hpp"

namespace vzh {


using vzb::f2add;
using vzb::f2mul;

namespace {

// layer_general_resident: children at (tree_p, tree_q)[child_offset ..
// child_offset + child_len), claim point of length L = log2(child_len) - 1.
std::pair<std::vector<Fp2>, std::vector<Fp2>> layer_general_resident(
    Backend& b, uint64_t tree_p, uint64_t tree_q, size_t child_offset, size_t child_len,
    const std::vector<Fp2>& point, FpStream& chal, std::vector<Fp2>& proof) {
    const Api& A = b.api();
    void* ctx = b.ctx();
    const size_t vector_len = child_len / 2;
    Owned own(b);
    uint64_t v[4];
    v[0] = own.add(b.alloc(vector_len * sizeof(Fp2)));
    v[1] = own.add(b.alloc(vector_len * sizeof(Fp2)));
    v[2] = own.add(b.alloc(vector_len * sizeof(Fp2)));
    v[3] = own.add(b.alloc(vector_len * sizeof(Fp2)));
    b.check(A.volta_cuda_fp2_deinterleave_device(ctx, tree_p, child_offset, vector_len, v[0], 0, v[1], 0),
            "fp2_deinterleave_device");
    b.check(A.volta_cuda_fp2_deinterleave_device(ctx, tree_q, child_offset, vector_len, v[2], 0, v[3], 0),
            "fp2_deinterleave_device");
    const Fp2 lambda = chal.next_fp2();
    Fp2 cpref{1, 0};
    std::vector<Fp2> rprime;
    const size_t L = point.size();
    uint64_t suffix = 0;
    if (L) {
        const uint64_t pts = own.add(b.alloc(L * sizeof(Fp2)));
        b.upload(pts, 0, point.data(), L * sizeof(Fp2));
        suffix = own.add(b.alloc(((size_t{1} << L) - 1) * sizeof(Fp2)));
        b.check(A.volta_cuda_logup_suffix_eq_device(ctx, pts, 0, L, suffix, 0), "logup_suffix_eq_device");
    }
    size_t len = vector_len;
    auto fold4 = [&](Fp2 r, size_t half, uint64_t* nv) {
        b.check(A.volta_cuda_logup_fold4_device(ctx, v[0], 0, v[1], 0, v[2], 0, v[3], 0, half, r, nv[0], 0,
                                                nv[1], 0, nv[2], 0, nv[3], 0),
                "logup_fold4_device");
    };
    const auto fused = b.ext().logup_fold_round;
    Fp2 acc[4];
    Fp2 pending{0, 0};  // challenge of the previous round, not yet folded in
    for (size_t j = 0; j < L; ++j) {
        const size_t half = len / 2;
        const size_t soff = (size_t{1} << (L - 1 - j)) - 1;
        if (j == 0 || !fused) {
            b.check(A.volta_cuda_logup_general_round_device(ctx, v[0], 0, v[1], 0, v[2], 0, v[3], 0, suffix,
                                                            soff, half, acc),
                    "logup_general_round_device");
        } else {
            // v still holds 2 * len entries: fold the previous round's
            // challenge and evaluate this round in one pass
            uint64_t nv[4];
            for (int k = 0; k < 4; ++k) nv[k] = own.add(b.alloc(len * sizeof(Fp2)));
            b.check(fused(ctx, v[0], v[1], v[2], v[3], 2 * len, pending, nv[0], nv[1], nv[2], nv[3], suffix,
                          soff, acc),
                    "volta_b200_logup_fold_round_device");
            for (int k = 0; k < 4; ++k) {
                own.release(v[k]);
                v[k] = nv[k];
            }
        }
        const Fp2 h0 = f2mul(cpref, f2add(f2mul(lambda, acc[0]), acc[2]));
        const Fp2 h2 = f2mul(cpref, f2add(f2mul(lambda, acc[1]), acc[3]));
        proof.push_back(h0);
        proof.push_back(h2);
        const Fp2 r = chal.next_fp2();
        if (!fused || j + 1 == L) {
            uint64_t nv[4];
            for (int k = 0; k < 4; ++k) nv[k] = own.add(b.alloc(half * sizeof(Fp2)));
            fold4(r, half, nv);
            for (int k = 0; k < 4; ++k) {
                own.release(v[k]);
                v[k] = nv[k];
            }
        } else {
            pending = r;
        }
        cpref = eq_step(cpref, point[j], r);
        rprime.push_back(r);
        len = half;
    }
    std::vector<Fp2> splits = b.download_fp2_segments({{v[0], 0}, {v[1], 0}, {v[2], 0}, {v[3], 0}});
    return {rprime, splits};
}

void prove_frac_tree_resident(Backend& b, uint64_t leaf, uint64_t mult, size_t n, uint64_t alpha1,
                              FpStream& chal, std::vector<Fp2>& proof) {
    const Api& A = b.api();
    void* ctx = b.ctx();
    int depth = 0;
    while ((size_t{1} << depth) < n) ++depth;
    Owned own(b);
    const uint64_t tp = own.add(b.alloc((n - 1) * sizeof(Fp2)));
    const uint64_t tq = own.add(b.alloc((n - 1) * sizeof(Fp2)));
    b.check(A.volta_cuda_logup_tree_device(ctx, leaf, 0, mult, 0, n, alpha1, mult ? 1 : 0, tp, 0, tq, 0),
            "logup_tree_device");
    std::vector<Fp2> root = b.download_fp2_segments({{tp, 0}, {tq, 0}});
    proof.push_back(root[0]);
    proof.push_back(root[1]);
    std::vector<Fp2> point;
    for (int l = 0; l < depth; ++l) {
        const bool leaf_layer = l + 1 == depth;
        std::pair<std::vector<Fp2>, std::vector<Fp2>> res;
        if (leaf_layer) {
            Owned leaves(b);
            const uint64_t lp = leaves.add(b.alloc(n * sizeof(Fp2)));
            const uint64_t lq = leaves.add(b.alloc(n * sizeof(Fp2)));
            b.check(A.volta_cuda_logup_materialize_leaves_device(ctx, leaf, 0, mult, 0, n, alpha1, mult ? 1 : 0,
                                                                 lp, 0, lq, 0),
                    "logup_materialize_leaves_device");
            res = layer_general_resident(b, lp, lq, 0, n, point, chal, proof);
        } else {
            const size_t child_len = size_t{1} << (l + 1);
            res = layer_general_resident(b, tp, tq, child_len - 1, child_len, point, chal, proof);
        }
        for (const Fp2& s : res.second) proof.push_back(s);
        const Fp2 t = chal.next_fp2();
        std::vector<Fp2> np;
        np.reserve(res.first.size() + 1);
        np.push_back(t);
        for (const Fp2& r : res.first) np.push_back(r);
        point.swap(np);
    }
}

}  // namespace

namespace {

TripleResult triple_sumcheck_rounds(Backend& b, uint64_t a, uint64_t bb, uint64_t c, size_t n, FpStream& tx) {
    const Api& A = b.api();
    void* ctx = b.ctx();
    TripleResult out;
    Owned own(b);
    uint64_t cur[3] = {a, bb, c};
    bool owned = false;  // the caller's inputs are never folded in place
    size_t len = n;
    const auto fused = b.ext().triple_fold_round;
    Fp2 g[3];
    if (len > 1)
        b.check(A.volta_cuda_fp2_triple_product_round_device(ctx, cur[0], 0, cur[1], 0, cur[2], 0, len / 2, g),
                "fp2_triple_product_round_device");
    while (len > 1) {
        const size_t pairs = len / 2;
        out.messages.insert(out.messages.end(), g, g + 3);
        const Fp2 r = tx.next_fp2();
        uint64_t nxt[3];
        for (int k = 0; k < 3; ++k) nxt[k] = own.add(b.alloc(pairs * sizeof(Fp2)));
        if (fused && pairs > 1) {
            // fold with r and produce the next round's message in one pass
            b.check(fused(ctx, cur[0], cur[1], cur[2], len, r, nxt[0], nxt[1], nxt[2], g),
                    "volta_b200_triple_fold_round_device");
        } else {
            for (int k = 0; k < 3; ++k)
                b.check(A.volta_cuda_fp2_fold_rows_device(ctx, cur[k], 0, 1, len, r, nxt[k], 0),
                        "fp2_fold_rows_device");
            if (pairs > 1)
                b.check(A.volta_cuda_fp2_triple_product_round_device(ctx, nxt[0], 0, nxt[1], 0, nxt[2], 0,
                                                                     pairs / 2, g),
                        "fp2_triple_product_round_device");
        }
        for (int k = 0; k < 3; ++k) {
            if (owned) own.release(cur[k]);
            cur[k] = nxt[k];
        }
        owned = true;
        len = pairs;
    }
    std::vector<Fp2> fin = b.download_fp2_segments({{cur[0], 0}, {cur[1], 0}, {cur[2], 0}});
    for (int k = 0; k < 3; ++k) out.finals[k] = fin[k];
    return out;
}

}  // namespace

using SideProver = void (*)(Backend&, uint64_t, uint64_t, size_t, uint64_t, FpStream&, std::vector<Fp2>&);

TripleResult triple_sumcheck_resident(Backend& b, uint64_t a, uint64_t bb, uint64_t c, size_t n,
                                      FpStream& tx) {
    return b.scheduled() ? triple_sumcheck_scheduled(b, a, bb, c, n, tx) : triple_sumcheck_rounds(b, a, bb, c, n, tx);
}

TripleResult triple_sumcheck_resident_fp(Backend& b, uint64_t a, uint64_t bb, uint64_t c, size_t n,
                                         FpStream& tx, const HostColumns* host) {
    const ExtApi& X = b.ext();
    if (b.scheduled() && X.triple_round_fp && X.triple_fold_round_fp && n >= 4)
        return triple_sumcheck_scheduled(b, a, bb, c, n, tx, true, host);
    Owned own(b);
    uint64_t lifted[3];
    const uint64_t cols[3] = {a, bb, c};
    if (host)
        for (int t = 0; t < 3; ++t) b.upload(cols[t], 0, host->col[t], n * sizeof(uint64_t));
    for (int t = 0; t < 3; ++t) {
        lifted[t] = own.add(b.alloc(n * sizeof(Fp2)));
        b.check(b.api().volta_cuda_base_broadcast_fp2_device(b.ctx(), cols[t], 0, lifted[t], 0, n, 1, 2),
                "base_broadcast_fp2_device");
    }
    return triple_sumcheck_resident(b, lifted[0], lifted[1], lifted[2], n, tx);
}

std::vector<Fp2> logup_prove_resident(Backend& b, uint64_t f_col, size_t n_f, uint64_t t_col,
                                      size_t n_t, uint64_t mult, FpStream& chal) {
    if (b.scheduled()) return logup_prove_scheduled(b, f_col, n_f, t_col, n_t, mult, chal);
    const SideProver side_prover = prove_frac_tree_resident;
    const Api& A = b.api();
    void* ctx = b.ctx();
    std::vector<Fp2> proof;
    const Fp2 alpha = chal.next_fp2();
    proof.push_back(alpha);
    Owned own(b);
    const uint32_t zero_shift = 0;
    const uint64_t shifts = own.add(b.alloc(sizeof(uint32_t)));
    b.upload(shifts, 0, &zero_shift, sizeof(zero_shift));
    // lookup side: leaf a_i = alpha0 - f_i, numerators 1
    {
        Owned side(b);
        const uint64_t leaf = side.add(b.alloc(n_f * sizeof(uint64_t)));
        b.check(A.volta_cuda_pack_lookup_leaf_device(ctx, f_col, 0, shifts, 0, leaf, 0, 1, n_f, alpha.c0),
                "pack_lookup_leaf_device");
        side_prover(b, leaf, 0, n_f, alpha.c1, chal, proof);
    }
    // table side: numerators -mult
    {
        Owned side(b);
        const uint64_t leaf = side.add(b.alloc(n_t * sizeof(uint64_t)));
        b.check(A.volta_cuda_pack_lookup_leaf_device(ctx, t_col, 0, shifts, 0, leaf, 0, 1, n_t, alpha.c0),
                "pack_lookup_leaf_device");
        side_prover(b, leaf, mult, n_t, alpha.c1, chal, proof);
    }
    return proof;
}

}  // namespace vzh
