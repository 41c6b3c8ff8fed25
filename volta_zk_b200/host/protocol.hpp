// Helpers shared by the protocol drivers (protocol.cpp, scheduled.cpp).
#pragma once

#include <vector>

#include "accel.hpp"
#include "api.hpp"

namespace vzh {

using vzb::f2add;
using vzb::f2mul;
using vzb::f2sub;

// eq(p, r) = 2pr - p - r + 1 (logup.rs:466-468)
inline Fp2 eq_step(Fp2 cpref, Fp2 p, Fp2 r) {
    const Fp2 pr = f2mul(p, r);
    return f2mul(cpref, f2add(f2sub(f2sub(f2add(pr, pr), p), r), Fp2{1, 0}));
}

// RAII list of arena ids freed on scope exit (mirrors the Rust guards).
struct Owned {
    Backend& b;
    std::vector<uint64_t> ids;
    explicit Owned(Backend& be) : b(be) {}
    uint64_t add(uint64_t id) {
        ids.push_back(id);
        return id;
    }
    void release(uint64_t id) {
        for (auto& x : ids)
            if (x == id) {
                x = 0;
                b.free(id);
                return;
            }
    }
    ~Owned() {
        for (uint64_t id : ids)
            if (id) b.api().volta_cuda_resident_free(b.ctx(), id);
    }
};

void prove_frac_tree_scheduled(Backend& b, uint64_t leaf, uint64_t mult, size_t n, uint64_t alpha1,
                               FpStream& chal, std::vector<Fp2>& proof);

// Every challenge of one fraction-tree side in the round-by-round order: per
// layer l the batching lambda, l round challenges and the split challenge t;
// point[l] is layer l's claim point (t, r' of layer l - 1).
struct SideSchedule {
    std::vector<Fp2> lambda, t;
    std::vector<std::vector<Fp2>> r, point;
};
SideSchedule draw_side_schedule(FpStream& chal, size_t depth);

// One shard's part of a side (scheduled.cpp): its subtree root and, per
// global layer l >= shard_bits, the raw accumulators of the first
// l - shard_bits rounds and the four left-over vector values.
struct LocalSide {
    size_t shard_bits = 0;
    Fp2 root_p, root_q;
    std::vector<std::vector<Fp2>> accs;      // [l - shard_bits][4 (l - shard_bits)]
    std::vector<std::vector<Fp2>> leftover;  // [l - shard_bits][4]
};
LocalSide frac_side_local(Backend& b, uint64_t leaf, uint64_t mult, size_t n_local, uint64_t alpha1,
                          size_t shard_bits, const SideSchedule& sch);
TripleResult triple_sumcheck_scheduled(Backend& b, uint64_t a, uint64_t bb, uint64_t c, size_t n,
                                       FpStream& tx, bool base = false, const HostColumns* host = nullptr);

// Enqueue / collect halves of the scheduled drivers: everything is enqueued
// on the context's stream with device-side message slots, and the collect
// call downloads them (the only synchronisation).  Buffers go to `own`,
// which must outlive the collect call.  Several enqueues may precede the
// first collect, so one proof's sumchecks run back to back on the GPU.
// With `host` set (base-field columns only), see HostColumns.
uint64_t triple_enqueue(Backend& b, Owned& own, uint64_t a, uint64_t bb, uint64_t c, size_t n, FpStream& tx,
                        bool base, size_t& k_out, const HostColumns* host = nullptr);
TripleResult triple_collect(Backend& b, uint64_t msgs, size_t k);
struct PendingSide {
    uint64_t msgs = 0;
    size_t msg_total = 0, depth = 0, shard_bits = 0;
    std::vector<size_t> moff;
    // launched by launch_side_work (suffix tables, round steps per layer, one-CTA jobs)
    std::vector<vzb_suffix_job> suffix_jobs;
    std::vector<std::vector<vzb_round_job>> plan;
    std::vector<vzb_layer_job> jobs;
    std::vector<vzb_copy_seg> copies;  // the root into the message slots
    // claim points and challenges read only by the batched launches, uploaded
    // together by launch_side_work
    std::vector<std::pair<uint64_t, std::vector<Fp2>>> uploads;
};
// leaf: the packed leaf column, or 0 with `col` and `alpha0` given (a side
// without multiplicities; leaf j = alpha0 - col_j).
PendingSide frac_side_enqueue(Backend& b, Owned& own, uint64_t leaf, uint64_t mult, size_t n_local,
                              uint64_t alpha1, size_t shard_bits, const SideSchedule& sch, uint64_t col = 0,
                              uint64_t alpha0 = 0);
// Launch the batched work of several sides together: one suffix-table batch,
// step t of every large layer of every side per launch, one launch of all
// one-CTA jobs.
void launch_side_work(Backend& b, const std::vector<PendingSide*>& sides);
LocalSide frac_side_collect(Backend& b, const PendingSide& ps);
// The same from the side's raw message slots already on the host.
LocalSide frac_side_parse(const PendingSide& ps, const Fp2* raw);
// Both sides of a (sharded) LogUp proof: the words of vzh_logup_local.
struct PendingLogup {
    Fp2 alpha;
    SideSchedule sch[2];
    PendingSide side[2];
};
PendingLogup logup_local_enqueue(Backend& b, Owned& own, uint64_t f_col, size_t n_f_local, uint64_t t_col,
                                 size_t n_t_local, uint64_t mult, size_t shard_bits, FpStream& chal);
std::vector<Fp2> logup_local_collect(Backend& b, const PendingLogup& pl);
// The proof words of a whole (unsharded) LogUp proof from both sides' raw
// message slots on the host (raw0: the query side, raw1: the table side):
// alpha, then per side its root and round messages, as logup_prove_resident.
void logup_proof_words(const PendingLogup& pl, const Fp2* raw0, const Fp2* raw1, std::vector<Fp2>& out);
// The same, downloading both sides' messages of an enqueued, unsharded proof.
std::vector<Fp2> logup_local_proof_words(Backend& b, const PendingLogup& pl);
// The whole LogUp proof (both sides' batches sharing launches, one download
// per side after everything is enqueued); words as logup_prove_resident.
std::vector<Fp2> logup_prove_scheduled(Backend& b, uint64_t f_col, size_t n_f, uint64_t t_col, size_t n_t,
                                       uint64_t mult, FpStream& chal);

}  // namespace vzh
