// GPT-2 small prefill proof schedule over the resident witness of a
// Gpt2Session (see gpt2.hpp).
//
// Per layer, in the reference's reverse dataflow order (FFN chain, then
// attention chain; rust/volta-proto/src/block_proof.rs:10246-10390
// prove_layer_phase1/phase2, 3825-4200 prove_ffn_*, prove_attn_block), the
// schedule proves with the seam's kernels:
//   * boundary authentication of x_in, k, v, attn_block_out, ffn_block_out:
//     VOLE-MAC masks (mock_correlation_sub_masks, domain (tag << 32) | row,
//     gemm.rs:135-138) and corrections x - mask (auth_matrix_rows_p,
//     block_proof.rs:1235);
//   * the 14 lookup instances of layer_lookups (block_proof.rs:9853-9876),
//     each a LogUp proof (logup.rs:1760-1771) of its query column against its
//     table with the instance's multiplicities: requant remainders on
//     Range(s) (range_cols_padded / range_mult, 2359-2408) and packed pairs
//     in + 2^k out on the pair tables (pair_cols_padded / pair_table,
//     2482-2520), padded to the reference's instance sizes (T_pad x 2^10 or
//     2^12, the 16 x T_pad x T_pad attention rectangle, 16 x T_pad, T_pad);
//   * the four weight GEMMs (gemm_proof.rs:685-760
//     prove_gemm_committed_chained): the claim acc~(r_i, r_j) at a transcript
//     point, the Thaler folds of X over eq(r_i) and of W over eq(r_j), and
//     the product sumcheck over k;
//   * the attention contractions Q.K^T (sumcheck over heads x head_dim of
//     Q_r, K_r, eq(r_h)) and A.V (over heads x key positions of the folded
//     weights and values and eq(r_h)), the softmax-norm product exp * recip
//     (triple sumcheck of the exp, reciprocal and real-entry columns over the
//     attention rectangle) and the two LayerNorm products (x - mu) * (r g)
//     (ln_hadamard_factors; prove_ln_chain, 3038-3180).
// After the layers, the Ligero PCS commitment of every weight (GPT2_FULL
// shape: 8192 rows x 2^14 int16 + 512 ChaCha8 pads, RS code 2^15, BLAKE3
// column tree; ligero.rs:59-60, 465-505).
//
// Each sub-proof draws its claim point and challenges from its own private
// transcript FpStream(seed, domain(layer, site)); claim points are not
// carried from one sub-proof into the next (each GEMM, contraction and
// product claim is evaluated from the witness at its own point), and the
// weight claims are not opened against the commitment.  Everything is
// enqueued with device-side message slots and nothing waits on the device
// until the words of all layers come home at the end.
#include <algorithm>
#include <chrono>
#include <cstring>

#include "gpt2.hpp"
#include "protocol.hpp"

namespace vzh {
namespace {

constexpr size_t kHeadPad = 16;
constexpr size_t kRecipBits = 18;       // luts.rs C62_SOFTMAX_RECIP_BITS
constexpr uint64_t kRecipPadInput = 256;  // block_proof.rs C62_RECIP_PAD_INPUT

size_t pow2_at_least(size_t n) {
    size_t p = 1;
    while (p < n) p <<= 1;
    return p;
}

size_t log2_exact(size_t n) {
    size_t k = 0;
    while ((size_t{1} << k) < n) ++k;
    return k;
}

uint64_t fp_from_i64(int64_t v) { return vzb::ffrom_i64(v); }

// LSB-first eq table of a point (mle.rs eq_vec), on the host
std::vector<Fp2> eq_host(const std::vector<Fp2>& pt) {
    std::vector<Fp2> t{Fp2{1, 0}};
    for (const Fp2& r : pt) {
        const size_t n = t.size();
        t.resize(2 * n);
        for (size_t i = 0; i < n; ++i) {
            const Fp2 hi = f2mul(t[i], r);
            t[n + i] = hi;
            t[i] = f2sub(t[i], hi);
        }
    }
    return t;
}

std::vector<Fp2> draw(FpStream& tx, size_t n) {
    std::vector<Fp2> v(n);
    for (auto& x : v) x = tx.next_fp2();
    return v;
}

}  // namespace

uint64_t gpt2_site_domain(size_t layer, int site, size_t chunk) {
    return 0x7000000000000000ull | (static_cast<uint64_t>(chunk) << 32) | (static_cast<uint64_t>(layer) << 16) |
           (static_cast<uint64_t>(site) << 8);
}

Gpt2Prover::Gpt2Prover(Gpt2Session& s) : s_(s), b_(s.backend()) {
    const Gpt2Shape& sh = s.shape();
    if (!sh.shifts.row_shift) throw AccelError("the GPT-2 proof needs the row-shifted (stable) softmax");
    // the attention sumchecks pad heads to 16 and draw 4 head variables
    if (sh.heads > kHeadPad || pow2_at_least(sh.d) / sh.head_dim > kHeadPad)
        throw AccelError("the GPT-2 proof supports at most 16 heads (padded model width / head_dim <= 16)");
    try {
        auto up = [&](const void* src, size_t bytes) {
            const uint64_t id = own(b_.alloc(bytes));
            b_.upload(id, 0, src, bytes);
            return id;
        };
        // Range(s) tables 0 .. 2^s - 1 (block_proof.rs:2504-2509)
        for (uint32_t s : {10u, 12u, 14u, 16u}) {
            std::vector<uint64_t> t(size_t{1} << s);
            for (size_t u = 0; u < t.size(); ++u) t[u] = u;
            range_[s] = up(t.data(), t.size() * 8);
        }
        // pair tables in(u) + 2^k out(u) (block_proof.rs:2511-2520)
        const std::vector<int16_t>& exp = s.lut_host(1);
        const std::vector<int16_t>& recip = s.lut_host(2);
        const std::vector<int16_t>& gelu = s.lut_host(3);
        const std::vector<int16_t>& rsqrt = s.lut_host(0);
        auto pair = [&](size_t len, unsigned k, bool signed_in, auto out_of) {
            std::vector<uint64_t> t(len);
            const uint64_t scale = uint64_t{1} << k;
            for (size_t u = 0; u < len; ++u) {
                const int64_t in = signed_in ? static_cast<int16_t>(static_cast<uint16_t>(u)) : static_cast<int64_t>(u);
                t[u] = vzb::fadd(fp_from_i64(in), vzb::fmul(fp_from_i64(out_of(u)), scale));
            }
            return up(t.data(), len * 8);
        };
        gelu_pairs_ = pair(1 << 16, 16, true, [&](size_t u) { return int64_t{gelu[u]}; });
        rsqrt_pairs_ = pair(1 << 16, 16, false, [&](size_t u) { return int64_t{rsqrt[u]}; });
        // ExpGap (luts.rs:188-206): exp of -gap for gap <= 2^15, else 0
        if (exp[0x8000] != 0) throw AccelError("softmax lower exp boundary is not zero");
        auto gap_exp = [&](size_t u) -> int64_t {
            return u <= 0x8000 ? exp[static_cast<uint16_t>(static_cast<int16_t>(-static_cast<int32_t>(u)))] : 0;
        };
        exp_pad_out_ = fp_from_i64(gap_exp(0));
        expgap_pairs_ = pair(1 << 16, 16, false, gap_exp);
        // the 18-bit reciprocal domain (luts.rs:208-226)
        const Gpt2Shifts& f = sh.shifts;
        auto recip18 = [&](size_t u) -> int64_t {
            if (u < (size_t{1} << 16)) return recip[u];
            const uint64_t den = (static_cast<uint64_t>(u) << f.recip_den) + (uint64_t{1} << (f.recip_den - 1));
            const uint64_t v = ((uint64_t{1} << f.recip_log2) + den / 2) / den;
            return static_cast<int64_t>(std::min<uint64_t>(v, 32767));
        };
        recip_pad_out_ = fp_from_i64(recip18(kRecipPadInput));
        recip_pairs_ = pair(size_t{1} << kRecipBits, kRecipBits, false, recip18);
        // pack shifts: {0, 16} at 0, {0, 18} at 2, {0} at 4
        const uint32_t shifts[5] = {0, 16, 0, kRecipBits, 0};
        shifts_ = up(shifts, sizeof(shifts));
        // the committed weight matrix: every layer's c_attn, attn_proj,
        // ffn_up, ffn_down, ln gains and biases, then wte, wpe, final LN,
        // row-major into rows of 2^14 int16 (zero past the weights)
        const size_t cols = size_t{1} << kPcsColBits;
        size_t total = 0;
        std::vector<std::pair<uint64_t, size_t>> parts;
        const size_t d = sh.d, dff = sh.dff;
        const size_t lsz[8] = {d * 3 * d, d * d, d * dff, dff * d, d, d, d, d};
        for (size_t l = 0; l < sh.layers; ++l)
            for (int k = 0; k < 8; ++k) parts.emplace_back(s.weight(l, k), lsz[k]);
        parts.emplace_back(s.wte(), sh.vocab * d);
        parts.emplace_back(s.wpe(), sh.positions * d);
        parts.emplace_back(s.lnf(0), d);
        parts.emplace_back(s.lnf(1), d);
        for (const auto& p : parts) total += p.second;
        pcs_rows_ = pcs_rows_for(total);
        wmat_ = own(b_.alloc(pcs_rows_ * cols * sizeof(int16_t)));
        b_.check(b_.api().volta_cuda_resident_zero(b_.ctx(), wmat_, 0, pcs_rows_ * cols * sizeof(int16_t)),
                 "resident_zero");
        size_t at = 0;
        for (const auto& p : parts) {
            b_.check(b_.api().volta_cuda_resident_copy_rows(b_.ctx(), p.first, 0, p.second * 2, wmat_, at * 2,
                                                            p.second * 2, 1, p.second * 2),
                     "resident_copy_rows");
            at += p.second;
        }
        pads_ = own(b_.alloc(pcs_rows_ * kPcsPad * sizeof(uint64_t)));
        code_ = own(b_.alloc(pcs_rows_ * (size_t{1} << kPcsCodeBits) * sizeof(uint64_t)));
        tree_ = own(b_.alloc(((size_t{2} << kPcsCodeBits) - 1) * 32));
        err_ = own(b_.alloc(sizeof(uint32_t)));
    } catch (...) {
        for (uint64_t id : owned_) b_.api().volta_cuda_resident_free(b_.ctx(), id);
        throw;
    }
}

Gpt2Prover::~Gpt2Prover() {
    for (uint64_t id : owned_) b_.api().volta_cuda_resident_free(b_.ctx(), id);
    for (const auto& l : corrections_)
        for (uint64_t id : l.second) b_.api().volta_cuda_resident_free(b_.ctx(), id);
}

namespace {

// ---- the sub-proof drivers ---------------------------------------------------

// Product sumcheck of two resident Fp2 vectors of n = 2^k entries
// (sumcheck_clear.rs:23-70 / hadamard.rs:190-260 with two factors): per round
// the seam's [g(0), g(2)] at msgs[off + 2 j], then the fold with r_j; the two
// final values at msgs[off + 2 k], msgs[off + 2 k + 1].  Challenges: the
// next k draws of tx.  Rounds on more than 2^11 entries run as one fused
// fold + next-round launch each; the rest run in one CTA.
constexpr size_t kProductTail = 2048;

void product_rounds(Backend& b, Owned& own, uint64_t a, uint64_t bb, size_t n, FpStream& tx, uint64_t msgs,
                    size_t off) {
    const Api& A = b.api();
    const ExtApi& X = b.ext();
    void* ctx = b.ctx();
    const size_t k = log2_exact(n);
    const std::vector<Fp2> r = draw(tx, k);
    if (!k) {
        for (int t = 0; t < 2; ++t)
            b.check(A.volta_cuda_resident_copy_rows(ctx, t ? bb : a, 0, sizeof(Fp2), msgs, (off + t) * sizeof(Fp2),
                                                    sizeof(Fp2), 1, sizeof(Fp2)),
                    "resident_copy_rows");
        return;
    }
    const uint64_t rdev = own.add(b.alloc(k * sizeof(Fp2)));
    b.upload(rdev, 0, r.data(), k * sizeof(Fp2));
    uint64_t cur[2] = {a, bb};
    size_t len = n, j = 0;
    if (len > kProductTail)
        b.check(A.volta_cuda_fp2_product_round_into_device(ctx, a, 0, bb, 0, len / 2, msgs, off),
                "fp2_product_round_into_device");
    while (len > kProductTail) {
        uint64_t nxt[2];
        for (int t = 0; t < 2; ++t) nxt[t] = own.add(b.alloc((len / 2) * sizeof(Fp2)));
        const vz_fp2 rj{r[j].c0, r[j].c1};
        if (len / 2 > kProductTail) {  // fold with r_j and round j + 1's message in one pass
            b.check(X.product_fold_round(ctx, cur[0], cur[1], len, rj, nxt[0], nxt[1], msgs, off + 2 * (j + 1)),
                    "volta_b200_product_fold_round_into_device");
        } else {  // the tail computes round j + 1 itself
            for (int t = 0; t < 2; ++t)
                b.check(A.volta_cuda_fp2_fold_rows_device(ctx, cur[t], 0, 1, len, rj, nxt[t], 0),
                        "fp2_fold_rows_device");
        }
        cur[0] = nxt[0];
        cur[1] = nxt[1];
        len /= 2;
        ++j;
    }
    b.check(X.product_tail(ctx, cur[0], cur[1], len, rdev, j, msgs, off + 2 * j), "volta_b200_product_tail_device");
}

// LogUp proof of one lookup instance: query side from `qcols` (one Fp
// column, or two packed as col0 + 2^k col1 with the pack shifts at
// shifts_off), table side from the table column with `mult`; the draw order
// and words of logup_prove_resident.
PendingLogup lookup_enqueue(Backend& b, Owned& own, uint64_t qcols, size_t qcount, uint64_t shifts,
                            size_t shifts_off, size_t n_f, uint64_t t_col, size_t n_t, uint64_t mult,
                            FpStream& chal) {
    const Api& A = b.api();
    PendingLogup pl;
    pl.alpha = chal.next_fp2();
    uint64_t leaf = 0;
    if (qcount == 2) {
        leaf = own.add(b.alloc(n_f * sizeof(uint64_t)));
        b.check(A.volta_cuda_pack_lookup_leaf_device(b.ctx(), qcols, 0, shifts, shifts_off, leaf, 0, 2, n_f,
                                                     pl.alpha.c0),
                "pack_lookup_leaf_device");
    }
    pl.sch[0] = draw_side_schedule(chal, log2_exact(n_f));
    pl.side[0] = frac_side_enqueue(b, own, leaf, 0, n_f, pl.alpha.c1, 0, pl.sch[0], leaf ? 0 : qcols, pl.alpha.c0);
    const uint64_t tleaf = own.add(b.alloc(n_t * sizeof(uint64_t)));
    b.check(A.volta_cuda_pack_lookup_leaf_device(b.ctx(), t_col, 0, shifts, 4, tleaf, 0, 1, n_t, pl.alpha.c0),
            "pack_lookup_leaf_device");
    pl.sch[1] = draw_side_schedule(chal, log2_exact(n_t));
    pl.side[1] = frac_side_enqueue(b, own, tleaf, mult, n_t, pl.alpha.c1, 0, pl.sch[1]);
    return pl;
}

}  // namespace

// One layer: enqueue every sub-proof (nothing is downloaded); returns the
// pending message slots in proof order.
std::vector<Gpt2Prover::Slot> Gpt2Prover::enqueue_layer(size_t l, Owned& own, const uint8_t seed[32],
                                                        const uint8_t mac_seed[32], const Gpt2Band* band,
                                                        size_t chunk, uint32_t mask) {
    const Api& A = b_.api();
    void* ctx = b_.ctx();
    const Gpt2Shape& sh = s_.shape();
    const Gpt2Shifts& f = sh.shifts;
    // rows t of the proof (the band's q, or the prefill's t) at positions
    // t0 .. t0 + t - 1, attending over the session's `keys` = t0 + t rows
    // (BandShape: q, s = t0 + q; the prefill is the square band t0 = 0)
    const size_t keys = sh.t, t0 = band ? band->t0() : 0, t = keys - t0;
    const size_t d = sh.d, dff = sh.dff, h = sh.heads;
    const size_t tp = pow2_at_least(t), sp = pow2_at_least(keys), rect = kHeadPad * tp * sp;
    const size_t d_pad = pow2_at_least(d), q_pad = pow2_at_least(3 * d), f_pad = pow2_at_least(dff);
    const size_t packed = h * (t * t0 + t * (t + 1) / 2);  // causal-packed attention entries (band packing)
    struct Wire {
        uint64_t id;
        size_t off;  // elements
    };
    auto W = [&](int w) -> Wire {
        if (!band) return Wire{s_.wire(l, w), 0};
        const auto bw = band->wire(l, w);
        return Wire{bw.first, bw.second};
    };
    auto alloc = [&](size_t bytes) { return own.add(b_.alloc(bytes)); };
    auto on = [&](int site) { return ((mask >> site) & 1u) != 0; };  // this unit proves the site
    std::vector<Slot> slots;

    // ---- boundary authentication --------------------------------------------
    const int boundary[5] = {kXin, kK, kV, kAttnOut, kFfnOut};
    std::vector<uint64_t> corr(5);
    for (int w = 0; w < 5 && on(kSiteCorrections); ++w) {
        // one mask domain per (chunk, layer, wire), row r at (tag << 32) | r
        const uint64_t tag = (static_cast<uint64_t>(chunk) << 16) | (l * 8 + w);
        const uint64_t masks = alloc(t * d * sizeof(uint64_t));
        b_.check(A.volta_cuda_mock_correlation_sub_masks_device(ctx, masks, 0, mac_seed, tag << 32, t, d),
                 "mock_correlation_sub_masks_device");
        corr[w] = b_.alloc(t * d * sizeof(uint64_t));
        const Wire x = W(boundary[w]);
        b_.check(A.volta_cuda_subfield_corrections_device(ctx, x.id, x.off, masks, 0, corr[w], 0, t * d, 0),
                 "subfield_corrections_device");
    }
    if (on(kSiteCorrections)) {
        corrections_[l] = corr;
        if (sink_) {
            if (!b_.ext().download_async) throw AccelError("backend lacks asynchronous downloads");
            for (int w = 0; w < 5; ++w)
                b_.check(b_.ext().download_async(ctx, corr[w], 0, sink_ + (l * 5 + w) * t * d,
                                                 t * d * sizeof(uint64_t)),
                         "volta_b200_download_async");
        }
    }

    // ---- the 14 lookup instances --------------------------------------------
    std::vector<PendingSide*> sides;
    std::vector<std::unique_ptr<PendingLogup>> logups;
    auto add_logup = [&](int site, uint64_t qcols, size_t qcount, size_t shifts_off, size_t n_f, uint64_t t_col,
                         size_t n_t, uint64_t mult) {
        FpStream chal(seed, gpt2_site_domain(l, site, chunk));
        logups.push_back(std::make_unique<PendingLogup>(
            lookup_enqueue(b_, own, qcols, qcount, shifts_, shifts_off, n_f, t_col, n_t, mult, chal)));
        sides.push_back(&logups.back()->side[0]);
        sides.push_back(&logups.back()->side[1]);
        Slot sl;
        sl.logup = logups.back().get();
        sl.site = site;
        slots.push_back(sl);
    };
    // a requant site: remainders of (acc, out) padded to row_pad x col_pad
    auto range_site = [&](int site, Wire acc, Wire out, size_t rows, size_t cols, size_t row_pad, size_t col_pad,
                          uint32_t shift) {
        if (!on(site)) return;
        const size_t n = row_pad * col_pad;
        const uint64_t cc = alloc(2 * n * sizeof(uint64_t));
        b_.check(A.volta_cuda_requant_columns_device(ctx, acc.id, acc.off, out.id, out.off, cc, 0, err_, 0, rows,
                                                     cols, row_pad, col_pad, 1, shift),
                 "requant_columns_device");
        const uint64_t mult = alloc((size_t{1} << shift) * sizeof(uint32_t));  // the histograms clear it
        b_.check(A.volta_cuda_histogram_fp_device(ctx, cc, 0, mult, 0, n, size_t{1} << shift),
                 "histogram_fp_device");
        add_logup(site, cc, 1, 0, n, range_.at(shift), size_t{1} << shift, mult);
    };
    // a pair site: (in, out) padded, packed in + 2^16 out
    auto pair_site = [&](int site, Wire in, int in_kind, Wire out, size_t rows, size_t cols, size_t row_pad,
                         size_t col_pad, uint64_t pad_in, uint64_t pad_out, uint64_t table, bool signed_in) {
        if (!on(site)) return;
        const size_t n = row_pad * col_pad;
        const uint64_t cc = alloc(2 * n * sizeof(uint64_t));
        b_.check(A.volta_cuda_pair_columns_device(ctx, in.id, in.off, out.id, out.off, cc, 0, rows, cols, row_pad,
                                                  col_pad, pad_in, pad_out, in_kind, 0),
                 "pair_columns_device");
        const uint64_t mult = alloc((size_t{1} << 16) * sizeof(uint32_t));
        if (signed_in)
            b_.check(A.volta_cuda_histogram_lut_device(ctx, cc, 0, mult, 0, n, 1), "histogram_lut_device");
        else
            b_.check(A.volta_cuda_histogram_fp_device(ctx, cc, 0, mult, 0, n, size_t{1} << 16),
                     "histogram_fp_device");
        // one query column in + 2^16 out: the column path of the LogUp driver
        const uint64_t q = alloc(n * sizeof(uint64_t));
        b_.check(b_.ext().pack_pair_column(ctx, cc, 0, n, 16, q, 0), "volta_b200_pack_pair_column_device");
        add_logup(site, q, 1, 0, n, table, size_t{1} << 16, mult);
    };
    const std::vector<int16_t>& gelu = s_.lut_host(3);
    const std::vector<int16_t>& rsqrt = s_.lut_host(0);
    // FFN chain
    range_site(kSiteDownRange, W(kDownAcc), W(kDownQ), t, d, tp, d_pad, f.ffn_down);
    pair_site(kSiteGelu, W(kUpQ), 0, W(kGelu), t, dff, tp, f_pad, 0, fp_from_i64(gelu[0]), gelu_pairs_, true);
    range_site(kSiteUpRange, W(kUpAcc), W(kUpQ), t, dff, tp, f_pad, f.ffn_up);
    range_site(kSiteLn2Norm, W(kLn2Acc), W(kLn2Out), t, d, tp, d_pad, f.ln_norm);
    pair_site(kSiteLn2Rsqrt, W(kLn2Rin), 1, W(kLn2Rout), 1, t, 1, tp, 0, fp_from_i64(rsqrt[0]), rsqrt_pairs_, false);
    // attention chain
    range_site(kSiteProjRange, W(kProjAcc), W(kProjQ), t, d, tp, d_pad, f.attn_proj);
    range_site(kSiteAvRange, W(kAvAcc), W(kAvQ), t, d, tp, d_pad, f.av);
    // softmax columns: [0] gap, [1] packed (gap, exp), [2] exp, [3] norm
    // remainders, [4] reciprocals, [5] mask; [6] reciprocal inputs, [7] packed
    // (input, reciprocal)
    uint64_t sm[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (on(kSiteNormRange) || on(kSiteExp) || on(kSiteRecip) || on(kSiteNormHad)) {
        for (int k = 0; k < 8; ++k) sm[k] = alloc((k < 6 ? rect : kHeadPad * tp) * sizeof(uint64_t));
        const Wire sq = W(kScoresQ), rs = W(kRowShift), ex = W(kExpOut), dn = W(kDenoms), rc = W(kRecips),
                   wt = W(kWeights);
        if (!b_.ext().softmax_lookup_columns_band) throw AccelError("backend lacks the band softmax columns");
        b_.check(b_.ext().softmax_lookup_columns_band(ctx, sq.id, sq.off, rs.id, rs.off, ex.id, ex.off, dn.id, dn.off,
                                                      rc.id, rc.off, wt.id, wt.off, sm, err_, 0, t, t0, h, rect,
                                                      kHeadPad, tp, exp_pad_out_, f.softmax_norm, f.recip_den,
                                                      kRecipPadInput, recip_pad_out_),
                 "volta_b200_softmax_lookup_columns_band_device");
    }
    if (on(kSiteNormRange)) {  // softmax norm remainders on Range(14)
        const uint64_t mult = alloc((size_t{1} << f.softmax_norm) * sizeof(uint32_t));
        b_.check(A.volta_cuda_histogram_fp_device(ctx, sm[3], 0, mult, 0, rect, size_t{1} << f.softmax_norm),
                 "histogram_fp_device");
        add_logup(kSiteNormRange, sm[3], 1, 0, rect, range_.at(f.softmax_norm), size_t{1} << f.softmax_norm, mult);
    }
    if (on(kSiteExp)) {  // (gap, exp) pairs on the ExpGap table
        const uint64_t mult = alloc((size_t{1} << 16) * sizeof(uint32_t));
        b_.check(A.volta_cuda_histogram_fp_device(ctx, sm[0], 0, mult, 0, rect, size_t{1} << 16),
                 "histogram_fp_device");
        add_logup(kSiteExp, sm[1], 1, 0, rect, expgap_pairs_, size_t{1} << 16, mult);
    }
    if (on(kSiteRecip)) {  // (denom >> den_shift, rc) pairs on the 18-bit reciprocal table
        const size_t n = kHeadPad * tp;
        const uint64_t mult = alloc((size_t{1} << kRecipBits) * sizeof(uint32_t));
        b_.check(A.volta_cuda_histogram_fp_device(ctx, sm[6], 0, mult, 0, n, size_t{1} << kRecipBits),
                 "histogram_fp_device");
        add_logup(kSiteRecip, sm[7], 1, 0, n, recip_pairs_, size_t{1} << kRecipBits, mult);
    }
    range_site(kSiteScoresRange, W(kScoresAcc), W(kScoresQ), 1, packed, 1, rect, f.scores);
    range_site(kSiteQkvRange, W(kQkvAcc), W(kQkvQ), t, 3 * d, tp, q_pad, f.qkv);
    range_site(kSiteLn1Norm, W(kLn1Acc), W(kLn1Out), t, d, tp, d_pad, f.ln_norm);
    pair_site(kSiteLn1Rsqrt, W(kLn1Rin), 1, W(kLn1Rout), 1, t, 1, tp, 0, fp_from_i64(rsqrt[0]), rsqrt_pairs_, false);
    // every instance's batched rounds share launches
    if (!sides.empty()) launch_side_work(b_, sides);
    pending_logups_.push_back(std::move(logups));

    // ---- sumchecks ------------------------------------------------------------
    auto slot_buffer = [&](int site, size_t words) {
        Slot sl;
        sl.msgs = alloc(words * sizeof(Fp2));
        sl.words = words;
        sl.site = site;
        slots.push_back(sl);
        return sl.msgs;
    };
    auto eq_table = [&](const std::vector<Fp2>& pt) {
        const uint64_t p = alloc(std::max<size_t>(pt.size(), 1) * sizeof(Fp2));
        if (!pt.empty()) b_.upload(p, 0, pt.data(), pt.size() * sizeof(Fp2));
        const uint64_t eq = alloc((size_t{1} << pt.size()) * sizeof(Fp2));
        b_.check(A.volta_cuda_logup_eq_rows_device(ctx, p, 0, 1, pt.size(), eq, 0), "logup_eq_rows_device");
        return eq;
    };
    // weight GEMM: claim acc~(r_i, r_j), folds, product sumcheck over k
    auto gemm = [&](int site, Wire x, uint64_t w, Wire acc, size_t m, size_t k, size_t n) {
        if (!on(site)) return;
        FpStream tx(seed, gpt2_site_domain(l, site, chunk));
        const size_t m_pad = pow2_at_least(m), n_pad = pow2_at_least(n), k_pad = pow2_at_least(k);
        const std::vector<Fp2> rj = draw(tx, log2_exact(n_pad)), ri = draw(tx, log2_exact(m_pad));
        const uint64_t eq_j = eq_table(rj), eq_i = eq_table(ri);
        const size_t kb = log2_exact(k_pad);
        const uint64_t msgs = slot_buffer(site, 1 + 2 * kb + 2);
        const uint64_t acc_r = alloc(n_pad * sizeof(Fp2));
        b_.check(A.volta_cuda_matrix_fold_device(ctx, acc.id, acc.off, eq_i, 0, acc_r, 0, m, n, 0, n, n_pad, 1, 0),
                 "matrix_fold_device");
        b_.check(A.volta_cuda_fp2_row_dots_device(ctx, acc_r, 0, n_pad, eq_j, 0, n_pad, msgs, 0, 1, n_pad),
                 "fp2_row_dots_device");
        const uint64_t av = alloc(k_pad * sizeof(Fp2)), bv = alloc(k_pad * sizeof(Fp2));
        b_.check(A.volta_cuda_matrix_fold_device(ctx, x.id, x.off, eq_i, 0, av, 0, m, k, 0, k, k_pad, 0, 0),
                 "matrix_fold_device");
        b_.check(A.volta_cuda_matrix_fold_device(ctx, w, 0, eq_j, 0, bv, 0, k, n, 0, n, k_pad, 0, 1),
                 "matrix_fold_device");
        product_rounds(b_, own, av, bv, k_pad, tx, msgs, 1);
    };
    // LayerNorm product (x - mu) * (r g) over t_pad x d_pad
    auto ln_product = [&](int site, int x, int mean, int rout, int gain) {
        if (!on(site)) return;
        FpStream tx(seed, gpt2_site_domain(l, site, chunk));
        const uint64_t mu = alloc(tp * sizeof(uint64_t)), rs = alloc(tp * sizeof(uint64_t));
        const Wire wm = W(mean), wr = W(rout), wx = W(x);
        b_.check(A.volta_cuda_pad_base_vector_device(ctx, wm.id, wm.off, mu, 0, t, tp, 0, 1), "pad_base_vector_device");
        b_.check(A.volta_cuda_pad_base_vector_device(ctx, wr.id, wr.off, rs, 0, t, tp, 0, 0), "pad_base_vector_device");
        const size_t n = tp * d_pad;
        const uint64_t cen = alloc(n * sizeof(Fp2)), sc = alloc(n * sizeof(Fp2));
        b_.check(A.volta_cuda_ln_hadamard_factors_device(ctx, wx.id, wx.off, mu, 0, rs, 0, s_.weight(l, gain), 0, cen,
                                                         0, sc, 0, t, d, tp, d_pad),
                 "ln_hadamard_factors_device");
        const uint64_t msgs = slot_buffer(site, 2 * log2_exact(n) + 2);
        product_rounds(b_, own, cen, sc, n, tx, msgs, 0);
    };
    auto triple = [&](int site, uint64_t a, uint64_t bb, uint64_t c, size_t n, FpStream& tx, bool base) {
        size_t k = 0;
        Slot sl;
        sl.site = site;
        sl.msgs = triple_enqueue(b_, own, a, bb, c, n, tx, base, k);
        sl.words = 3 * k + 3;
        slots.push_back(sl);
    };
    gemm(kSiteGemmDown, W(kGelu), s_.weight(l, 3), W(kDownAcc), t, dff, d);
    gemm(kSiteGemmUp, W(kLn2Out), s_.weight(l, 2), W(kUpAcc), t, d, dff);
    ln_product(kSiteLn2Had, kAttnOut, kLn2Mean, kLn2Rout, 6);
    gemm(kSiteGemmProj, W(kAvQ), s_.weight(l, 1), W(kProjAcc), t, d, d);
    if (on(kSiteAv)) {  // A.V over (head, key position)
        FpStream tx(seed, gpt2_site_domain(l, kSiteAv, chunk));
        const std::vector<Fp2> rc = draw(tx, log2_exact(sh.head_dim)), rh = draw(tx, 4), ri = draw(tx, log2_exact(tp));
        const uint64_t eq_c = eq_table(rc), eq_h = eq_table(rh), eq_i = eq_table(ri);
        const size_t n = kHeadPad * sp;  // (head, key position)
        const uint64_t parts[3] = {alloc(n * sizeof(Fp2)), alloc(n * sizeof(Fp2)), alloc(n * sizeof(Fp2))};
        const Wire wt = W(kWeights);
        if (!b_.ext().av_factors_band) throw AccelError("backend lacks the band A.V factors");
        // V over every cached row 0 .. keys - 1 (the session's rows)
        b_.check(b_.ext().av_factors_band(ctx, wt.id, wt.off, s_.wire(l, kV), 0, eq_i, 0, eq_c, 0, eq_h, 0, parts, t,
                                          t0, h, sh.head_dim, kHeadPad, tp, sp),
                 "volta_b200_av_factors_band_device");
        triple(kSiteAv, parts[0], parts[1], parts[2], n, tx, false);
    }
    if (on(kSiteNormHad)) {  // softmax norm product over the attention rectangle (Fp columns: exp, reciprocal, mask)
        FpStream tx(seed, gpt2_site_domain(l, kSiteNormHad, chunk));
        triple(kSiteNormHad, sm[2], sm[4], sm[5], rect, tx, true);
    }
    if (on(kSiteQk)) {  // Q.K^T over (head, dimension)
        FpStream tx(seed, gpt2_site_domain(l, kSiteQk, chunk));
        const std::vector<Fp2> rj = draw(tx, log2_exact(sp)), ri = draw(tx, log2_exact(tp)), rh = draw(tx, 4);
        const uint64_t eq_i = eq_table(ri), eq_j = eq_table(rj);
        const std::vector<Fp2> eh = eq_host(rh);
        std::vector<Fp2> c(d_pad, Fp2{0, 0});
        for (size_t x = 0; x < d_pad; ++x) c[x] = eh[x / sh.head_dim];
        const uint64_t cid = alloc(d_pad * sizeof(Fp2));
        b_.upload(cid, 0, c.data(), d_pad * sizeof(Fp2));
        const uint64_t qr = alloc(d_pad * sizeof(Fp2)), kr = alloc(d_pad * sizeof(Fp2));
        const Wire wq = W(kQ);
        b_.check(A.volta_cuda_matrix_fold_device(ctx, wq.id, wq.off, eq_i, 0, qr, 0, t, d, 0, d, d_pad, 0, 0),
                 "matrix_fold_device");
        // K over every cached row 0 .. keys - 1
        b_.check(A.volta_cuda_matrix_fold_device(ctx, s_.wire(l, kK), 0, eq_j, 0, kr, 0, keys, d, 0, d, d_pad, 0, 0),
                 "matrix_fold_device");
        triple(kSiteQk, qr, kr, cid, d_pad, tx, false);
    }
    gemm(kSiteGemmQkv, W(kLn1Out), s_.weight(l, 0), W(kQkvAcc), t, d, 3 * d);
    ln_product(kSiteLn1Had, kXin, kLn1Mean, kLn1Rout, 4);
    return slots;
}

Gpt2Proof Gpt2Prover::prove(const uint8_t seed[32], const uint8_t mac_seed[32], const uint8_t pad_seed[32]) {
    return prove_layers(seed, mac_seed, pad_seed, 0, 1, true);
}

namespace {
std::vector<Gpt2Unit> layer_units(size_t layers, size_t first, size_t stride) {
    if (!stride) throw AccelError("GPT-2 proof layer stride must be positive");
    std::vector<Gpt2Unit> u;
    for (size_t l = first; l < layers; l += stride) u.push_back(Gpt2Unit{l, kGpt2AllSites});
    return u;
}
}  // namespace

Gpt2Proof Gpt2Prover::prove_layers(const uint8_t seed[32], const uint8_t mac_seed[32], const uint8_t pad_seed[32],
                                   size_t first, size_t stride, bool with_pcs) {
    return run(seed, mac_seed, pad_seed, layer_units(s_.shape().layers, first, stride), with_pcs, nullptr, 0);
}

Gpt2Proof Gpt2Prover::prove_units(const uint8_t seed[32], const uint8_t mac_seed[32], const uint8_t pad_seed[32],
                                  const std::vector<Gpt2Unit>& units, bool with_pcs) {
    return run(seed, mac_seed, pad_seed, units, with_pcs, nullptr, 0);
}

void Gpt2Prover::commit_rows(const uint8_t pad_seed[32], size_t row0, size_t rows, uint8_t* cvs) {
    const Api& A = b_.api();
    void* ctx = b_.ctx();
    const size_t code_len = size_t{1} << kPcsCodeBits, cols = size_t{1} << kPcsColBits;
    if (!rows || rows % 128 || ((rows / 128) & (rows / 128 - 1)) || row0 % rows || row0 + rows > pcs_rows_)
        throw AccelError("commitment row block must be 128 * 2^k rows at a multiple of its size inside the matrix");
    if (!cvs_) cvs_ = own(b_.alloc(code_len * 32));
    // row r's pads come from ChaCha8 stream r, as in the whole commitment
    b_.check(A.volta_cuda_chacha8_prover_secret_fp_rows_device(ctx, pads_, 0, pad_seed, row0, rows, kPcsPad),
             "chacha8_prover_secret_fp_rows_device");
    b_.check(A.volta_cuda_pcs_messages_device(ctx, wmat_, row0 * cols, pads_, 0, rows, cols, kPcsPad, code_len, code_,
                                              0),
             "pcs_messages_device");
    b_.check(A.volta_cuda_ntt_fp_batch_device(ctx, code_, 0, rows, code_len, code_, 0), "ntt_fp_batch_device");
    if (!b_.ext().hash_fp_column_cvs) throw AccelError("backend lacks the column chaining values");
    b_.check(b_.ext().hash_fp_column_cvs(ctx, code_, 0, rows, code_len, row0 / 128, cvs_, 0),
             "volta_b200_hash_fp_column_cvs_device");
    b_.download(cvs_, 0, cvs, code_len * 32);
}

Gpt2Proof Gpt2Prover::prove_band(const Gpt2Band& band, size_t chunk, const uint8_t seed[32],
                                 const uint8_t mac_seed[32], size_t first, size_t stride) {
    if (&band.session() != &s_) throw AccelError("the band is not of this prover's session");
    if (!chunk || chunk >= (size_t{1} << 14)) throw AccelError("band chunk index must be in 1 .. 2^14 - 1");
    return run(seed, mac_seed, nullptr, layer_units(s_.shape().layers, first, stride), false, &band, chunk);
}

Gpt2Proof Gpt2Prover::run(const uint8_t seed[32], const uint8_t mac_seed[32], const uint8_t pad_seed[32],
                          const std::vector<Gpt2Unit>& units, bool with_pcs, const Gpt2Band* band, size_t chunk) {
    const Api& A = b_.api();
    void* ctx = b_.ctx();
    const Gpt2Shape& sh = s_.shape();
    for (const Gpt2Unit& u : units)
        if (u.layer >= sh.layers || !u.sites || (u.sites & ~kGpt2AllSites))
            throw AccelError("invalid GPT-2 proof unit (layer out of range or unknown sites)");
    const auto t_start = std::chrono::steady_clock::now();
    for (const auto& l : corrections_)
        for (uint64_t id : l.second) A.volta_cuda_resident_free(ctx, id);
    corrections_.clear();
    pending_logups_.clear();
    b_.check(A.volta_cuda_resident_zero(ctx, err_, 0, sizeof(uint32_t)), "resident_zero");
    // Each layer's raw messages are copied (device to device) into one buffer
    // per layer, so the layer's working buffers can be released as soon as
    // its work is enqueued (frees are stream-ordered) and the whole proof is
    // enqueued without waiting on the device; the words come home at the end.
    Owned keep(b_);
    struct LayerRaw {
        uint64_t buf = 0;
        size_t total = 0;
        std::vector<Slot> slots;
    };
    std::vector<LayerRaw> raw;
    for (const Gpt2Unit& u : units) {
        Owned lay(b_);
        raw.emplace_back();
        LayerRaw& lr = raw.back();
        lr.slots = enqueue_layer(u.layer, lay, seed, mac_seed, band, chunk, u.sites);
        for (Slot& sl : lr.slots) {
            sl.at = lr.total;
            lr.total += sl.logup ? sl.logup->side[0].msg_total + sl.logup->side[1].msg_total : sl.words;
        }
        lr.buf = keep.add(b_.alloc(std::max<size_t>(lr.total, 1) * sizeof(Fp2)));  // (a corrections-only unit has no words)
        std::vector<vzb_copy_seg> segs;  // every slot's messages into the layer buffer, one batched copy
        auto copy = [&](uint64_t src, size_t words, size_t at) {
            segs.push_back(vzb_copy_seg{src, 0, lr.buf, at * sizeof(Fp2), words * sizeof(Fp2)});
        };
        for (const Slot& sl : lr.slots) {
            if (sl.logup) {
                copy(sl.logup->side[0].msgs, sl.logup->side[0].msg_total, sl.at);
                copy(sl.logup->side[1].msgs, sl.logup->side[1].msg_total, sl.at + sl.logup->side[0].msg_total);
            } else {
                copy(sl.msgs, sl.words, sl.at);
            }
        }
        if (b_.ext().copy_segments && !segs.empty()) {
            b_.check(b_.ext().copy_segments(ctx, segs.data(), segs.size()), "copy_segments_device");
        } else {
            for (const vzb_copy_seg& g : segs)
                b_.check(A.volta_cuda_resident_copy_rows(ctx, g.src_id, 0, g.bytes, g.dst_id, g.dst_offset, g.bytes, 1,
                                                         g.bytes),
                         "resident_copy_rows");
        }
    }
    // Ligero commitment of the weights
    const size_t code_len = size_t{1} << kPcsCodeBits, cols = size_t{1} << kPcsColBits;
    if (with_pcs) {
        b_.check(A.volta_cuda_chacha8_prover_secret_fp_rows_device(ctx, pads_, 0, pad_seed, 0, pcs_rows_, kPcsPad),
                 "chacha8_prover_secret_fp_rows_device");
        b_.check(A.volta_cuda_pcs_messages_device(ctx, wmat_, 0, pads_, 0, pcs_rows_, cols, kPcsPad, code_len, code_,
                                                  0),
                 "pcs_messages_device");
        b_.check(A.volta_cuda_ntt_fp_batch_device(ctx, code_, 0, pcs_rows_, code_len, code_, 0), "ntt_fp_batch_device");
        b_.check(A.volta_cuda_hash_fp_tree_device(ctx, code_, 0, pcs_rows_, code_len, tree_, 0),
                 "hash_fp_tree_device");
    }
    const auto t_enqueued = std::chrono::steady_clock::now();
    // the words: one download per layer, LogUp accumulators turned into
    // round messages exactly as the resident LogUp driver does
    Gpt2Proof out;
    for (const LayerRaw& lr : raw) {
        std::vector<Fp2> host(lr.total);
        if (lr.total) b_.download(lr.buf, 0, host.data(), lr.total * sizeof(Fp2));
        std::vector<Fp2> words;
        std::vector<std::pair<int, size_t>> sites;
        for (const Slot& sl : lr.slots) {
            const size_t before = words.size();
            if (sl.logup)
                logup_proof_words(*sl.logup, host.data() + sl.at, host.data() + sl.at + sl.logup->side[0].msg_total,
                                  words);
            else
                words.insert(words.end(), host.begin() + sl.at, host.begin() + sl.at + sl.words);
            sites.emplace_back(sl.site, words.size() - before);
        }
        out.layer_words.push_back(std::move(words));
        out.unit_sites.push_back(std::move(sites));
    }
    pending_logups_.clear();
    if (with_pcs) b_.download(tree_, (2 * code_len - 2) * 32, out.pcs_root, 32);
    uint32_t e = 0;
    b_.download(err_, 0, &e, sizeof(e));
    if (sink_) b_.check(b_.ext().wait_downloads(ctx), "volta_b200_wait_downloads");
    const auto t_done = std::chrono::steady_clock::now();
    host_enqueue_ms_ = std::chrono::duration<double, std::milli>(t_enqueued - t_start).count();
    host_total_ms_ = std::chrono::duration<double, std::milli>(t_done - t_start).count();
    if (e) throw AccelError("GPT-2 proof witness columns out of their lookup domains");
    return out;
}

}  // namespace vzh
