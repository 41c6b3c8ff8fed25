// Scheduled protocol drivers.
//
// In the clear sink (logup.rs:1601-1622) and the private transcript
// (transcript.rs:84-103: FpStream(seed, u64::MAX)) every challenge is the next
// draw of a seeded stream that never absorbs a message.  The challenge
// sequence, every claim point and every suffix-eq table are therefore known
// before the first kernel runs.  These drivers draw them first, in the exact
// order of the round-by-round callers (hadamard.rs:186-260, logup.rs:995-1470),
// enqueue every round on the context's stream with its message written to a
// device slot (the *_into_device entry points), and bring all messages home in
// one download.  The host then forms the proof words (h0, h2 = cpref (lambda pq
// + qq), logup.rs:452-453) exactly as the round-by-round driver does.
//
// Nothing waits on the GPU between rounds, so the GPU runs the rounds back to
// back instead of idling for a host round trip per round.
#include <algorithm>
#include <cstring>

#include "protocol.hpp"

namespace vzh {

// Vectors at most this long finish in one CTA (volta_b200_*_tail / layers).
constexpr size_t kTailLen = 2048;
// Jobs per volta_b200_logup_round_batch_device call.
constexpr size_t kRoundBatchMax = 24;
// Entries per tile of volta_b200_triple_local_device (13 rounds per pass).
constexpr size_t kLocalTile = 8192;
constexpr size_t kLocalRounds = 13;
constexpr size_t kLocalAccBytes = kLocalRounds * 3 * 4 * sizeof(uint64_t);
// Entries per column and upload chunk when host columns stream in (3 x 16 MiB;
// 2^20 and 2^22 measured within 1 % of it on a 2^24 proof with two lanes).
constexpr size_t kDefaultUploadChunk = size_t{1} << 21;

uint64_t triple_enqueue(Backend& b, Owned& own, uint64_t a, uint64_t bb, uint64_t c, size_t n, FpStream& tx,
                        bool base, size_t& k_out, const HostColumns* host) {
    const Api& A = b.api();
    const ExtApi& X = b.ext();
    void* ctx = b.ctx();
    size_t k = 0;
    while ((size_t{1} << k) < n) ++k;
    if ((size_t{1} << k) != n) throw AccelError("triple sumcheck needs a power-of-two table length");
    k_out = k;
    std::vector<Fp2> r(k);
    for (auto& x : r) x = tx.next_fp2();
    // slots: 3 per round message, then the 3 final openings
    const uint64_t msgs = own.add(b.alloc((3 * k + 3) * sizeof(Fp2)));
    const bool local = X.triple_local && X.triple_flush && X.triple_tail;
    uint64_t rdev = 0;
    if ((X.triple_tail || local) && k) {
        rdev = own.add(b.alloc(k * sizeof(Fp2)));
        b.upload(rdev, 0, r.data(), k * sizeof(Fp2));
    }
    uint64_t cur[3] = {a, bb, c};
    bool owned = false, finals = false;
    size_t len = n, j = 0;
    const bool stream_in = host && local && base && n >= kLocalTile && n > kTailLen;
    if (host) {
        if (!base) throw AccelError("host columns need the base-field driver");
        if (!X.upload_async || !X.wait_uploads) throw AccelError("asynchronous uploads unavailable");
        if (!stream_in) {  // everything lands before the first round
            for (int t = 0; t < 3; ++t)
                b.check(X.upload_async(ctx, cur[t], 0, host->col[t], n * sizeof(uint64_t)), "volta_b200_upload_async");
            b.check(X.wait_uploads(ctx), "volta_b200_wait_uploads");
        }
    }
    // on-chip passes: 13 rounds per launch while the tables are longer than
    // the tail takes and hold whole tiles
    uint64_t acc = 0;
    while (local && len >= kLocalTile && len > kTailLen) {
        if (!acc) {
            acc = own.add(b.alloc(kLocalAccBytes));
            b.check(A.volta_cuda_resident_zero(ctx, acc, 0, kLocalAccBytes), "resident_zero");
        }
        const size_t tiles = len / kLocalTile;
        uint64_t nxt[3];
        for (int t = 0; t < 3; ++t) nxt[t] = own.add(b.alloc(tiles * sizeof(Fp2)));
        // one launch over all tiles, or (first pass over host columns) one per
        // uploaded chunk, each waiting for its own chunk only
        size_t per = tiles;
        if (stream_in && j == 0) {
            const size_t want = host->chunk ? host->chunk : kDefaultUploadChunk;
            per = std::max<size_t>(1, want / kLocalTile);
        }
        for (size_t t0 = 0; t0 < tiles; t0 += per) {
            const size_t cnt = std::min(per, tiles - t0);
            if (stream_in && j == 0) {
                const size_t off = t0 * kLocalTile, m = cnt * kLocalTile;
                for (int t = 0; t < 3; ++t)
                    b.check(X.upload_async(ctx, cur[t], off * sizeof(uint64_t), host->col[t] + off,
                                           m * sizeof(uint64_t)),
                            "volta_b200_upload_async");
                b.check(X.wait_uploads(ctx), "volta_b200_wait_uploads");
            }
            b.check(X.triple_local(ctx, base && j == 0, cur[0], cur[1], cur[2], len, t0, cnt, rdev, j, acc,
                                   nxt[0], nxt[1], nxt[2]),
                    "volta_b200_triple_local_device");
        }
        b.check(X.triple_flush(ctx, acc, msgs, 3 * j), "volta_b200_triple_flush_device");
        for (int t = 0; t < 3; ++t) {
            if (owned) own.release(cur[t]);
            cur[t] = nxt[t];
        }
        owned = true;
        len = tiles;
        j += kLocalRounds;
    }
    if (j) {
        // round j's message on the folded tables, unless the tail takes them
        if (len > kTailLen)
            b.check(A.volta_cuda_fp2_triple_product_round_into_device(ctx, cur[0], 0, cur[1], 0, cur[2], 0, len / 2,
                                                                      msgs, 3 * j),
                    "fp2_triple_product_round_into_device");
    } else if (base) {
        // base-field columns (n >= 4): rounds 0 and 1 read them directly; the
        // fold with r[0] writes the Fp2 tables the later rounds use (when they
        // go to the tail, it recomputes round 1 with the same result)
        b.check(X.triple_round_fp(ctx, a, bb, c, n / 2, msgs, 0), "volta_b200_triple_round_fp_into_device");
        uint64_t nxt[3];
        for (int t = 0; t < 3; ++t) nxt[t] = own.add(b.alloc((n / 2) * sizeof(Fp2)));
        b.check(X.triple_fold_round_fp(ctx, a, bb, c, n, r[0], nxt[0], nxt[1], nxt[2], msgs, 3),
                "volta_b200_triple_fold_round_fp_into_device");
        for (int t = 0; t < 3; ++t) cur[t] = nxt[t];
        owned = true;
        len = n / 2;
        j = 1;
    } else if (k && (!X.triple_tail || n > kTailLen)) {
        // large rounds: one pass each (fold of the previous round fused with the next round)
        b.check(A.volta_cuda_fp2_triple_product_round_into_device(ctx, a, 0, bb, 0, c, 0, n / 2, msgs, 0),
                "fp2_triple_product_round_into_device");
    }
    while (j < k && (!X.triple_tail || len > kTailLen)) {
        const size_t pairs = len / 2;
        if (pairs == 1) {  // last fold: the openings land in their slots
            for (int t = 0; t < 3; ++t)
                b.check(A.volta_cuda_fp2_fold_rows_device(ctx, cur[t], 0, 1, 2, r[j], msgs, 3 * k + t),
                        "fp2_fold_rows_device");
            ++j;
            len = 1;
            finals = true;
            break;
        }
        uint64_t nxt[3];
        for (int t = 0; t < 3; ++t) nxt[t] = own.add(b.alloc(pairs * sizeof(Fp2)));
        const bool to_tail = X.triple_tail && pairs <= kTailLen;
        if (to_tail) {  // the remaining rounds run in the tail
            for (int t = 0; t < 3; ++t)
                b.check(A.volta_cuda_fp2_fold_rows_device(ctx, cur[t], 0, 1, len, r[j], nxt[t], 0),
                        "fp2_fold_rows_device");
        } else if (X.triple_fold_round_into) {
            b.check(X.triple_fold_round_into(ctx, cur[0], cur[1], cur[2], len, r[j], nxt[0], nxt[1], nxt[2], msgs,
                                             3 * (j + 1)),
                    "volta_b200_triple_fold_round_into_device");
        } else {
            for (int t = 0; t < 3; ++t)
                b.check(A.volta_cuda_fp2_fold_rows_device(ctx, cur[t], 0, 1, len, r[j], nxt[t], 0),
                        "fp2_fold_rows_device");
            b.check(A.volta_cuda_fp2_triple_product_round_into_device(ctx, nxt[0], 0, nxt[1], 0, nxt[2], 0,
                                                                      pairs / 2, msgs, 3 * (j + 1)),
                    "fp2_triple_product_round_into_device");
        }
        for (int t = 0; t < 3; ++t) {
            if (owned) own.release(cur[t]);
            cur[t] = nxt[t];
        }
        owned = true;
        len = pairs;
        ++j;
    }
    if (X.triple_tail && len <= kTailLen && !finals) {
        // rounds j..k-1 and the openings in one CTA
        b.check(X.triple_tail(ctx, cur[0], cur[1], cur[2], len, rdev, j, msgs, 3 * j), "volta_b200_triple_tail_device");
    } else if (!k) {  // a single entry: the openings are the inputs
        for (int t = 0; t < 3; ++t)
            b.check(A.volta_cuda_resident_copy_rows(ctx, cur[t], 0, sizeof(Fp2), msgs, t * sizeof(Fp2),
                                                    sizeof(Fp2), 1, sizeof(Fp2)),
                    "resident_copy_rows");
    }
    return msgs;
}

TripleResult triple_collect(Backend& b, uint64_t msgs, size_t k) {
    std::vector<Fp2> host(3 * k + 3);
    b.download(msgs, 0, host.data(), host.size() * sizeof(Fp2));
    TripleResult out;
    out.messages.assign(host.begin(), host.begin() + 3 * k);
    for (int t = 0; t < 3; ++t) out.finals[t] = host[3 * k + t];
    return out;
}

TripleResult triple_sumcheck_scheduled(Backend& b, uint64_t a, uint64_t bb, uint64_t c, size_t n, FpStream& tx,
                                       bool base, const HostColumns* host) {
    Owned own(b);
    size_t k = 0;
    const uint64_t msgs = triple_enqueue(b, own, a, bb, c, n, tx, base, k, host);
    return triple_collect(b, msgs, k);
}

SideSchedule draw_side_schedule(FpStream& chal, size_t depth) {
    SideSchedule s;
    s.lambda.resize(depth);
    s.t.resize(depth);
    s.r.resize(depth);
    s.point.resize(depth);
    for (size_t l = 0; l < depth; ++l) {
        s.lambda[l] = chal.next_fp2();
        s.r[l].resize(l);
        for (auto& x : s.r[l]) x = chal.next_fp2();
        s.t[l] = chal.next_fp2();
        if (l + 1 < depth) {  // claim point of the next layer: (t, r')
            s.point[l + 1].push_back(s.t[l]);
            s.point[l + 1].insert(s.point[l + 1].end(), s.r[l].begin(), s.r[l].end());
        }
    }
    return s;
}

// One shard of a fraction-tree side.  The shard holds leaves
// [g n_local, (g+1) n_local) of a side of depth log2(n_local) + shard_bits;
// its subtree is the slice of every global level below level shard_bits.
// For every global layer l >= shard_bits it runs the first l - shard_bits
// rounds on its slice (the rounds that only fold the shard's own index bits)
// with the suffix-eq tables of the truncated claim point, so each round
// accumulator is this shard's share of the global one up to the factor
// eq(top bits of the point, g), and keeps the four vector values left over.
// With shard_bits = 0 these are the whole rounds and the splits.
PendingSide frac_side_enqueue(Backend& b, Owned& own, uint64_t leaf, uint64_t mult, size_t n_local,
                              uint64_t alpha1, size_t shard_bits, const SideSchedule& sch, uint64_t col,
                              uint64_t alpha0) {
    const Api& A = b.api();
    const ExtApi& X = b.ext();
    void* ctx = b.ctx();
    size_t local_depth = 0;
    while ((size_t{1} << local_depth) < n_local) ++local_depth;
    if ((size_t{1} << local_depth) != n_local || !local_depth)
        throw AccelError("fraction-tree shards need a power-of-two length of at least 2");
    const size_t depth = local_depth + shard_bits;
    // truncated claim points of the sharded layers in one upload
    std::vector<size_t> pts_off(depth, 0);
    std::vector<Fp2> flat;
    for (size_t l = shard_bits; l < depth; ++l) {
        pts_off[l] = flat.size();
        const size_t Lp = l - shard_bits;
        flat.insert(flat.end(), sch.point[l].begin(), sch.point[l].begin() + Lp);
    }
    // With the cross-layer batches, the points and the jobs' challenges are
    // read only by launch_side_work's launches: their uploads go with it
    const bool defer = X.logup_layers && X.logup_round_batch && X.logup_suffix_eq_batch && X.upload_batch &&
                       b.batched() && flat.size() * sizeof(Fp2) <= (size_t{64} << 10);
    std::vector<std::pair<uint64_t, std::vector<Fp2>>> deferred;
    uint64_t pts = 0;
    if (!flat.empty()) {
        pts = own.add(b.alloc(flat.size() * sizeof(Fp2)));
        if (defer)
            deferred.emplace_back(pts, flat);
        else
            b.upload(pts, 0, flat.data(), flat.size() * sizeof(Fp2));
    }
    // message slots: local root, then per sharded layer its local round
    // accumulators (4 Fp2 each) and its 4 left-over values
    std::vector<size_t> moff(depth, 0);
    size_t msg_total = 2;
    for (size_t l = shard_bits; l < depth; ++l) {
        moff[l] = msg_total;
        msg_total += 4 * (l - shard_bits) + 4;
    }
    const uint64_t msgs = own.add(b.alloc(msg_total * sizeof(Fp2)));
    const uint64_t tp = own.add(b.alloc((n_local - 1) * sizeof(Fp2)));
    const uint64_t tq = own.add(b.alloc((n_local - 1) * sizeof(Fp2)));
    // A side without multiplicities given as its query column (leaf j = alpha0
    // - col_j) whose leaf layer runs as cross-layer batches: the tree and the
    // leaf layer's first two steps read the column, so the packed leaves and
    // the materialised leaf denominators are never stored.
    const bool col_path = col && !mult && X.logup_tree_column && X.logup_round_batch && b.batched() &&
                          X.logup_layers && n_local / 4 > kTailLen;
    if (col_path) {
        b.check(X.logup_tree_column(ctx, col, 0, alpha0, n_local, alpha1, tp, 0, tq, 0),
                "volta_b200_logup_tree_column_device");
    } else {
        if (!leaf) {  // pack the leaf column: alpha0 - col
            const uint32_t zero_shift = 0;
            const uint64_t shifts = own.add(b.alloc(sizeof(uint32_t)));
            b.upload(shifts, 0, &zero_shift, sizeof(zero_shift));
            leaf = own.add(b.alloc(n_local * sizeof(uint64_t)));
            b.check(A.volta_cuda_pack_lookup_leaf_device(ctx, col, 0, shifts, 0, leaf, 0, 1, n_local, alpha0),
                    "pack_lookup_leaf_device");
        }
        b.check(A.volta_cuda_logup_tree_device(ctx, leaf, 0, mult, 0, n_local, alpha1, mult ? 1 : 0, tp, 0, tq, 0),
                "logup_tree_device");
    }
    // the side's root (p, q) into its first message slots: gathered with the
    // other sides' roots into one batched copy by launch_side_work
    std::vector<vzb_copy_seg> root_copies = {vzb_copy_seg{tp, 0, msgs, 0, sizeof(Fp2)},
                                             vzb_copy_seg{tq, 0, msgs, sizeof(Fp2), sizeof(Fp2)}};
    // round challenges of the local rounds, for the one-CTA layer jobs
    const bool jobs_on = X.logup_layers != nullptr;
    std::vector<size_t> r_off(depth, 0);
    uint64_t rbuf = 0;
    if (jobs_on) {
        std::vector<Fp2> rflat;
        for (size_t l = shard_bits; l < depth; ++l) {
            r_off[l] = rflat.size();
            rflat.insert(rflat.end(), sch.r[l].begin(), sch.r[l].begin() + (l - shard_bits));
        }
        if (!rflat.empty()) {
            rbuf = own.add(b.alloc(rflat.size() * sizeof(Fp2)));
            if (defer && rflat.size() * sizeof(Fp2) <= (size_t{64} << 10))
                deferred.emplace_back(rbuf, std::move(rflat));
            else
                b.upload(rbuf, 0, rflat.data(), rflat.size() * sizeof(Fp2));
        }
    }
    std::vector<vzb_layer_job> jobs;  // launched together after every large round is enqueued
    // Cross-layer batches: with every claim point and challenge known, the
    // large layers are independent, so step t of every layer runs in one
    // launch (plan[layer][t]); the buffers they use live until the end.
    const bool batch_on = jobs_on && X.logup_round_batch && b.batched();
    std::vector<std::vector<vzb_round_job>> plan;
    std::vector<vzb_suffix_job> suffix_jobs;  // built together before the first batch
    auto tail_job = [&](const uint64_t v[4], size_t l, size_t j0) {
        vzb_layer_job jb{};
        for (int k = 0; k < 4; ++k) jb.v_id[k] = v[k];
        jb.rounds = (l - shard_bits) - j0;
        jb.point_id = pts;
        jb.point_offset = pts_off[l] + j0;
        jb.r_id = rbuf;
        jb.r_offset = r_off[l] + j0;
        jb.out_id = msgs;
        jb.out_offset = moff[l] + 4 * j0;
        jobs.push_back(jb);
    };
    for (size_t l = shard_bits; l < depth; ++l) {
        Owned layer(b);
        const size_t L = l - shard_bits;  // local rounds
        const size_t vector_len = size_t{1} << L, child_len = size_t{2} << L;
        const size_t split = moff[l] + 4 * L;
        uint64_t src_p = tp, src_q = tq;
        size_t child_off = child_len - 1;
        const bool small = jobs_on && vector_len <= kTailLen;
        if (l + 1 == depth && col_path) {  // the leaf layer's children come from the column
            src_p = 0;
            src_q = col;
            child_off = 0;
        } else if (l + 1 == depth) {  // the leaf layer's children are the materialised leaves
            Owned& keep = (small || batch_on) ? own : layer;  // a job or batch reads them after this loop
            src_p = keep.add(b.alloc(n_local * sizeof(Fp2)));
            src_q = keep.add(b.alloc(n_local * sizeof(Fp2)));
            b.check(A.volta_cuda_logup_materialize_leaves_device(ctx, leaf, 0, mult, 0, n_local, alpha1,
                                                                 mult ? 1 : 0, src_p, 0, src_q, 0),
                    "logup_materialize_leaves_device");
            child_off = 0;
        }
        if (small) {  // the whole layer in one CTA: deinterleave on load, all rounds, splits
            vzb_layer_job jb{};
            jb.il_p_id = src_p;
            jb.il_q_id = src_q;
            jb.il_offset = child_off;
            jb.rounds = L;
            jb.point_id = pts;
            jb.point_offset = pts_off[l];
            jb.r_id = rbuf;
            jb.r_offset = r_off[l];
            jb.out_id = msgs;
            jb.out_offset = moff[l];
            jobs.push_back(jb);
            continue;
        }
        if (L == 0) {  // no local rounds: the four values are the two child pairs
            b.check(A.volta_cuda_fp2_deinterleave_device(ctx, src_p, child_off, 1, msgs, split, msgs, split + 1),
                    "fp2_deinterleave_device");
            b.check(A.volta_cuda_fp2_deinterleave_device(ctx, src_q, child_off, 1, msgs, split + 2, msgs,
                                                         split + 3),
                    "fp2_deinterleave_device");
            continue;
        }
        const uint64_t suffix = (batch_on ? own : layer).add(b.alloc(((size_t{1} << L) - 1) * sizeof(Fp2)));
        if (batch_on && X.logup_suffix_eq_batch)
            suffix_jobs.push_back(vzb_suffix_job{pts, pts_off[l], L, suffix, 0});
        else
            b.check(A.volta_cuda_logup_suffix_eq_device(ctx, pts, pts_off[l], L, suffix, 0),
                    "logup_suffix_eq_device");
        if (batch_on) {  // vector_len > kTailLen here: L >= 12
            // the leaf layer of a side without multiplicities has all-one
            // numerators (materialize_leaves): its jobs skip them, except
            // that the fold feeding the one-CTA tail writes the ones
            const uint32_t flags =
                (l + 1 == depth && !mult && vector_len / 2 > kTailLen) ? VZB_ROUND_P_ONE : 0u;
            const bool from_col = l + 1 == depth && col_path;  // (col_path implies flags)
            std::vector<vzb_round_job> steps;
            auto challenge = [&](vzb_round_job& q, size_t j) {
                q.r[0] = sch.r[l][j].c0;
                q.r[1] = sch.r[l][j].c1;
            };
            // round 0 and (fold 0 + round 1) on the interleaved children
            vzb_round_job q{};
            q.kind = 0;
            q.flags = flags | (from_col ? VZB_ROUND_Q_COLUMN : 0u);
            q.q_alpha[0] = alpha0;
            q.q_alpha[1] = alpha1;
            q.in_id[0] = src_p;
            q.in_id[1] = src_q;
            q.in_offset[0] = child_off;
            q.len = vector_len;
            q.s_id = suffix;
            q.s_offset = (size_t{1} << (L - 1)) - 1;
            q.msg_id = msgs;
            q.msg_offset = moff[l];
            if (!flags) {  // round 0's t = 0 terms are the layer's own tree level (the children's parents)
                q.flags |= VZB_ROUND_PARENTS;
                q.out_id[0] = tp;
                q.out_id[1] = tq;
                q.out_offset[0] = vector_len - 1;
            }
            steps.push_back(q);
            q.flags &= ~VZB_ROUND_PARENTS;
            q.out_offset[0] = 0;
            size_t len = vector_len / 2;
            uint64_t v[4] = {0, 0, 0, 0};
            for (int k = flags ? 2 : 0; k < 4; ++k) v[k] = own.add(b.alloc(len * sizeof(Fp2)));
            q.kind = 1;
            challenge(q, 0);
            for (int k = 0; k < 4; ++k) q.out_id[k] = v[k];
            q.s_offset = (size_t{1} << (L - 2)) - 1;
            q.msg_offset = moff[l] + 4;
            steps.push_back(q);
            if (len <= kTailLen) {
                tail_job(v, l, 1);  // (the job rewrites the round-1 message)
            } else {
                for (size_t j = 1;; ++j) {  // fold j + round j + 1
                    const size_t half = len / 2;
                    const bool last = half <= kTailLen;  // fold only, then the one-CTA tail
                    uint64_t nv[4] = {0, 0, 0, 0};
                    for (int k = (flags && !last) ? 2 : 0; k < 4; ++k) nv[k] = own.add(b.alloc(half * sizeof(Fp2)));
                    vzb_round_job f{};
                    f.flags = flags;
                    for (int k = 0; k < 4; ++k) {
                        f.in_id[k] = v[k];
                        f.out_id[k] = nv[k];
                    }
                    f.len = len;
                    challenge(f, j);
                    if (last) {  // fold only; rounds j + 1 .. L - 1 in one CTA
                        f.kind = 3;
                        steps.push_back(f);
                        tail_job(nv, l, j + 1);
                        break;
                    }
                    f.kind = 2;
                    f.s_id = suffix;
                    f.s_offset = (size_t{1} << (L - 2 - j)) - 1;
                    f.msg_id = msgs;
                    f.msg_offset = moff[l] + 4 * (j + 1);
                    steps.push_back(f);
                    for (int k = 0; k < 4; ++k) v[k] = nv[k];
                    len = half;
                }
            }
            plan.push_back(std::move(steps));
            continue;
        }
        size_t len = vector_len;
        uint64_t v[4];
        size_t j_first = 0;
        if (X.logup_round_il && X.logup_fold_round_il && vector_len >= 4) {
            // rounds 0 and 1 read the interleaved children directly (no deinterleave pass)
            b.check(X.logup_round_il(ctx, src_p, src_q, child_off, vector_len, suffix, (size_t{1} << (L - 1)) - 1,
                                     msgs, moff[l]),
                    "volta_b200_logup_round_il_into_device");
            const size_t half = len / 2;
            const bool to_job = jobs_on && half <= kTailLen;
            Owned& keep = to_job ? own : layer;
            for (auto& x : v) x = keep.add(b.alloc(half * sizeof(Fp2)));
            // (when the rest goes to a job, the job rewrites this round-1 message)
            b.check(X.logup_fold_round_il(ctx, src_p, src_q, child_off, vector_len, sch.r[l][0], v[0], v[1], v[2],
                                          v[3], suffix, (size_t{1} << (L - 2)) - 1, msgs, moff[l] + 4),
                    "volta_b200_logup_fold_round_il_into_device");
            len = half;
            j_first = 1;
            if (to_job) {
                vzb_layer_job jb{};
                for (int k = 0; k < 4; ++k) jb.v_id[k] = v[k];
                jb.rounds = L - 1;
                jb.point_id = pts;
                jb.point_offset = pts_off[l] + 1;
                jb.r_id = rbuf;
                jb.r_offset = r_off[l] + 1;
                jb.out_id = msgs;
                jb.out_offset = moff[l] + 4;
                jobs.push_back(jb);
                continue;
            }
        } else {
            for (auto& x : v) x = layer.add(b.alloc(vector_len * sizeof(Fp2)));
            b.check(A.volta_cuda_fp2_deinterleave_device(ctx, src_p, child_off, vector_len, v[0], 0, v[1], 0),
                    "fp2_deinterleave_device");
            b.check(A.volta_cuda_fp2_deinterleave_device(ctx, src_q, child_off, vector_len, v[2], 0, v[3], 0),
                    "fp2_deinterleave_device");
            b.check(A.volta_cuda_logup_general_round_into_device(ctx, v[0], 0, v[1], 0, v[2], 0, v[3], 0, suffix,
                                                                 (size_t{1} << (L - 1)) - 1, len / 2, msgs,
                                                                 moff[l]),
                    "logup_general_round_into_device");
        }
        for (size_t j = j_first; j < L; ++j) {
            const Fp2 rj = sch.r[l][j];
            const size_t half = len / 2;
            if (half == 1) {  // last fold: the left-over values land in their slots
                b.check(A.volta_cuda_logup_fold4_device(ctx, v[0], 0, v[1], 0, v[2], 0, v[3], 0, 1, rj, msgs, split,
                                                        msgs, split + 1, msgs, split + 2, msgs, split + 3),
                        "logup_fold4_device");
                break;
            }
            const bool to_job = jobs_on && half <= kTailLen;
            Owned& keep = to_job ? own : layer;  // the job reads the folded vectors later
            uint64_t nv[4];
            for (auto& x : nv) x = keep.add(b.alloc(half * sizeof(Fp2)));
            const size_t soff = (size_t{1} << (L - 2 - j)) - 1;  // suffix table of round j + 1
            if (to_job) {
                b.check(A.volta_cuda_logup_fold4_device(ctx, v[0], 0, v[1], 0, v[2], 0, v[3], 0, half, rj, nv[0], 0,
                                                        nv[1], 0, nv[2], 0, nv[3], 0),
                        "logup_fold4_device");
                // rounds j + 1 .. L - 1 and the splits in one CTA
                vzb_layer_job jb{};
                for (int k = 0; k < 4; ++k) jb.v_id[k] = nv[k];
                jb.rounds = L - (j + 1);
                jb.point_id = pts;
                jb.point_offset = pts_off[l] + j + 1;
                jb.r_id = rbuf;
                jb.r_offset = r_off[l] + j + 1;
                jb.out_id = msgs;
                jb.out_offset = moff[l] + 4 * (j + 1);
                jobs.push_back(jb);
                break;
            }
            if (X.logup_fold_round_into) {
                b.check(X.logup_fold_round_into(ctx, v[0], v[1], v[2], v[3], len, rj, nv[0], nv[1], nv[2], nv[3],
                                                suffix, soff, msgs, moff[l] + 4 * (j + 1)),
                        "volta_b200_logup_fold_round_into_device");
            } else {
                b.check(A.volta_cuda_logup_fold4_device(ctx, v[0], 0, v[1], 0, v[2], 0, v[3], 0, half, rj, nv[0], 0,
                                                        nv[1], 0, nv[2], 0, nv[3], 0),
                        "logup_fold4_device");
                b.check(A.volta_cuda_logup_general_round_into_device(ctx, nv[0], 0, nv[1], 0, nv[2], 0, nv[3], 0,
                                                                     suffix, soff, half / 2, msgs,
                                                                     moff[l] + 4 * (j + 1)),
                        "logup_general_round_into_device");
            }
            for (int k = 0; k < 4; ++k) {
                layer.release(v[k]);
                v[k] = nv[k];
            }
            len = half;
        }
    }
    // the suffix tables, the round batches and the one-CTA jobs are launched
    // by launch_side_work, together with those of other sides
    PendingSide ps;
    ps.msgs = msgs;
    ps.msg_total = msg_total;
    ps.depth = depth;
    ps.shard_bits = shard_bits;
    ps.moff = std::move(moff);
    ps.suffix_jobs = std::move(suffix_jobs);
    ps.plan = std::move(plan);
    ps.jobs = std::move(jobs);
    ps.copies = std::move(root_copies);
    ps.uploads = std::move(deferred);
    return ps;
}

void launch_side_work(Backend& b, const std::vector<PendingSide*>& sides) {
    const ExtApi& X = b.ext();
    void* ctx = b.ctx();
    {   // every side's deferred uploads, before the launches that read them
        std::vector<vzb_upload> items;
        for (const PendingSide* ps : sides)
            for (const auto& u : ps->uploads)
                items.push_back(vzb_upload{u.first, 0, u.second.data(), u.second.size() * sizeof(Fp2)});
        if (!items.empty()) b.check(X.upload_batch(ctx, items.data(), items.size()), "upload_batch");
    }
    {   // every side's root copies (its tree is already enqueued)
        std::vector<vzb_copy_seg> copies;
        for (const PendingSide* ps : sides) copies.insert(copies.end(), ps->copies.begin(), ps->copies.end());
        if (X.copy_segments) {
            b.check(X.copy_segments(ctx, copies.data(), copies.size()), "copy_segments_device");
        } else {
            for (const vzb_copy_seg& g : copies)
                b.check(b.api().volta_cuda_resident_copy_rows(ctx, g.src_id, g.src_offset, g.bytes, g.dst_id,
                                                              g.dst_offset, g.bytes, 1, g.bytes),
                        "resident_copy_rows");
        }
    }
    std::vector<vzb_suffix_job> suffix_jobs;
    std::vector<vzb_layer_job> jobs;
    size_t steps_max = 0;
    for (const PendingSide* ps : sides) {
        suffix_jobs.insert(suffix_jobs.end(), ps->suffix_jobs.begin(), ps->suffix_jobs.end());
        jobs.insert(jobs.end(), ps->jobs.begin(), ps->jobs.end());
        for (const auto& st : ps->plan) steps_max = std::max(steps_max, st.size());
    }
    // one suffix-table batch per group of jobs whose large tables fit one
    // outer-product launch: a job of point length L has min(11, L - 12)
    // tables of 2^12 .. 2^22 entries in the first band, and no later band
    // has more
    constexpr size_t kOuterJobsPerLaunch = 256, kEqTileBits = 11;
    for (size_t at = 0; at < suffix_jobs.size();) {
        size_t end = at, large = 0;
        while (end < suffix_jobs.size()) {
            const size_t L = suffix_jobs[end].point_len;
            const size_t k = L > kEqTileBits + 1 ? std::min(kEqTileBits, L - kEqTileBits - 1) : 0;
            if (end > at && large + k > kOuterJobsPerLaunch) break;
            large += k;
            ++end;
        }
        b.check(X.logup_suffix_eq_batch(ctx, suffix_jobs.data() + at, end - at),
                "volta_b200_logup_suffix_eq_batch_device");
        at = end;
    }
    // step t of every large layer of every side in one launch (chunks of kRoundBatchMax)
    std::vector<vzb_round_job> batch;
    for (size_t t = 0; t < steps_max; ++t) {
        batch.clear();
        for (const PendingSide* ps : sides)
            for (const auto& st : ps->plan)
                if (t < st.size()) batch.push_back(st[t]);
        for (size_t o = 0; o < batch.size(); o += kRoundBatchMax)
            b.check(X.logup_round_batch(ctx, batch.data() + o, std::min(kRoundBatchMax, batch.size() - o)),
                    "volta_b200_logup_round_batch_device");
    }
    if (!jobs.empty()) b.check(X.logup_layers(ctx, jobs.data(), jobs.size()), "volta_b200_logup_layers_device");
}

LocalSide frac_side_collect(Backend& b, const PendingSide& ps) {
    std::vector<Fp2> m(ps.msg_total);
    b.download(ps.msgs, 0, m.data(), ps.msg_total * sizeof(Fp2));
    return frac_side_parse(ps, m.data());
}

LocalSide frac_side_parse(const PendingSide& ps, const Fp2* m) {
    LocalSide out;
    out.shard_bits = ps.shard_bits;
    out.root_p = m[0];
    out.root_q = m[1];
    for (size_t l = ps.shard_bits; l < ps.depth; ++l) {
        const size_t L = l - ps.shard_bits;
        out.accs.emplace_back(m + ps.moff[l], m + ps.moff[l] + 4 * L);
        out.leftover.emplace_back(m + ps.moff[l] + 4 * L, m + ps.moff[l] + 4 * L + 4);
    }
    return out;
}

LocalSide frac_side_local(Backend& b, uint64_t leaf, uint64_t mult, size_t n_local, uint64_t alpha1,
                          size_t shard_bits, const SideSchedule& sch) {
    Owned own(b);
    PendingSide ps = frac_side_enqueue(b, own, leaf, mult, n_local, alpha1, shard_bits, sch);
    launch_side_work(b, {&ps});
    return frac_side_collect(b, ps);
}

PendingLogup logup_local_enqueue(Backend& b, Owned& own, uint64_t f_col, size_t n_f_local, uint64_t t_col,
                                 size_t n_t_local, uint64_t mult, size_t shard_bits, FpStream& chal) {
    const Api& A = b.api();
    PendingLogup pl;
    pl.alpha = chal.next_fp2();
    const uint32_t zero_shift = 0;
    const uint64_t shifts = own.add(b.alloc(sizeof(uint32_t)));
    b.upload(shifts, 0, &zero_shift, sizeof(zero_shift));
    const uint64_t cols[2] = {f_col, t_col};
    const size_t ns[2] = {n_f_local, n_t_local};
    for (int side = 0; side < 2; ++side) {
        // the side without multiplicities passes its column: frac_side_enqueue
        // reads it directly where it can, else packs the leaves itself
        uint64_t leaf = 0;
        if (side == 1) {
            leaf = own.add(b.alloc(ns[side] * sizeof(uint64_t)));
            b.check(A.volta_cuda_pack_lookup_leaf_device(b.ctx(), cols[side], 0, shifts, 0, leaf, 0, 1, ns[side],
                                                         pl.alpha.c0),
                    "pack_lookup_leaf_device");
        }
        size_t local_depth = 0;
        while ((size_t{1} << local_depth) < ns[side]) ++local_depth;
        pl.sch[side] = draw_side_schedule(chal, local_depth + shard_bits);
        pl.side[side] = frac_side_enqueue(b, own, leaf, side ? mult : 0, ns[side], pl.alpha.c1, shard_bits,
                                          pl.sch[side], cols[side], pl.alpha.c0);
    }
    launch_side_work(b, {&pl.side[0], &pl.side[1]});  // both sides' batches share launches
    return pl;
}

std::vector<Fp2> logup_local_collect(Backend& b, const PendingLogup& pl) {
    std::vector<Fp2> words;
    words.push_back(pl.alpha);
    for (int side = 0; side < 2; ++side) {
        const LocalSide loc = frac_side_collect(b, pl.side[side]);
        words.push_back(loc.root_p);
        words.push_back(loc.root_q);
        for (size_t i = 0; i < loc.accs.size(); ++i) {
            words.insert(words.end(), loc.accs[i].begin(), loc.accs[i].end());
            words.insert(words.end(), loc.leftover[i].begin(), loc.leftover[i].end());
        }
    }
    return words;
}

// A whole side's proof words in the round-by-round order (h0, h2 =
// cpref (lambda pq + qq), logup.rs:452-453) from its raw accumulators.
static void append_side_proof(const SideSchedule& sch, const LocalSide& loc, std::vector<Fp2>& proof) {
    const size_t depth = sch.lambda.size();
    proof.push_back(loc.root_p);
    proof.push_back(loc.root_q);
    for (size_t l = 0; l < depth; ++l) {
        Fp2 cpref{1, 0};
        for (size_t j = 0; j < l; ++j) {
            const Fp2* acc = &loc.accs[l][4 * j];
            proof.push_back(f2mul(cpref, f2add(f2mul(sch.lambda[l], acc[0]), acc[2])));
            proof.push_back(f2mul(cpref, f2add(f2mul(sch.lambda[l], acc[1]), acc[3])));
            cpref = eq_step(cpref, sch.point[l][j], sch.r[l][j]);
        }
        for (int k = 0; k < 4; ++k) proof.push_back(loc.leftover[l][k]);
    }
}

void logup_proof_words(const PendingLogup& pl, const Fp2* raw0, const Fp2* raw1, std::vector<Fp2>& out) {
    out.push_back(pl.alpha);
    append_side_proof(pl.sch[0], frac_side_parse(pl.side[0], raw0), out);
    append_side_proof(pl.sch[1], frac_side_parse(pl.side[1], raw1), out);
}

std::vector<Fp2> logup_local_proof_words(Backend& b, const PendingLogup& pl) {
    std::vector<Fp2> proof;
    proof.push_back(pl.alpha);
    for (int side = 0; side < 2; ++side) append_side_proof(pl.sch[side], frac_side_collect(b, pl.side[side]), proof);
    return proof;
}

std::vector<Fp2> logup_prove_scheduled(Backend& b, uint64_t f_col, size_t n_f, uint64_t t_col, size_t n_t,
                                       uint64_t mult, FpStream& chal) {
    Owned own(b);
    const PendingLogup pl = logup_local_enqueue(b, own, f_col, n_f, t_col, n_t, mult, 0, chal);
    std::vector<Fp2> proof;
    proof.push_back(pl.alpha);
    for (int side = 0; side < 2; ++side) append_side_proof(pl.sch[side], frac_side_collect(b, pl.side[side]), proof);
    return proof;
}

void prove_frac_tree_scheduled(Backend& b, uint64_t leaf, uint64_t mult, size_t n, uint64_t alpha1,
                               FpStream& chal, std::vector<Fp2>& proof) {
    size_t depth = 0;
    while ((size_t{1} << depth) < n) ++depth;
    const SideSchedule sch = draw_side_schedule(chal, depth);
    const LocalSide loc = frac_side_local(b, leaf, mult, n, alpha1, 0, sch);
    append_side_proof(sch, loc, proof);
}

}  // namespace vzh
