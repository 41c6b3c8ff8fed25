// Blind LogUp corrections (extension, include/volta_b200_ext.h).
//
// The VOLE-MAC blind sink of the reference (rust/volta-proto/src/logup.rs:
// 1903-2000, BlindSink::root / round / splits) publishes, instead of each
// clear LogUp message, its correction v - x against a fresh full-field mask
// x (draw_fulls, rust/volta-mac/src/corr.rs:1930-1978):
//   root      (p, q) - masks                                    (2)
//   round j   h0 = cpref (lambda pq0 + qq0), h2 = cpref (lambda pq2 + qq2),
//             then cpref <- cpref (2 pt_j r_j + 1 - pt_j - r_j)  (2 per round)
//   splits    (p0, p1, q0, q1) - masks                          (4)
//   products  (p0 q1, p1 q0, q0 q1) - masks                     (3)
// The same arithmetic as blind_begin / blind_round / blind_finish of the
// reference's blind-rounds benchmark (cuda/p7_logup_blind_rounds.cu:180-214).
//
// Here the raw round accumulators are already resident (the round drivers
// write 4 per round and then the 4 split values), the masks are expanded on
// the device in proof order, and the claim points and challenges are known
// in advance, so every correction of every layer of every instance comes
// out of one launch: one thread per layer job, a few hundred field
// operations each, and nothing waits on the host between rounds.
#include <algorithm>
#include <cstddef>
#include <vector>

#include "runtime.cuh"

namespace vzb {
namespace {

constexpr int kBlindJobsPerLaunch = 64;
static_assert(sizeof(vzb_blind_job) == 112 && offsetof(vzb_blind_job, lambda) == 80,
              "vzb_blind_job layout is ABI (Python mirrors it)");

struct BlindJob {
    const Fp2* raw;   // 4 accumulators per round (pq0, pq2, qq0, qq2), then p0, p1, q0, q1
    const Fp2* root;  // (p, q) of the tree, or null
    const Fp2* pt;    // `rounds` claim-point coordinates
    const Fp2* r;     // `rounds` challenges
    const Fp2* mask;  // mask values in output order
    Fp2* out;
    Fp2 lambda;
    int rounds;
};

struct BlindJobs {
    BlindJob j[kBlindJobsPerLaunch];
};

__global__ void blind_corrections_kernel(const BlindJobs jobs, int count) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= count) return;
    const BlindJob& jb = jobs.j[t];
    const Fp2* m = jb.mask;
    Fp2* o = jb.out;
    if (jb.root) {
        o[0] = d2sub(jb.root[0], m[0]);
        o[1] = d2sub(jb.root[1], m[1]);
        o += 2;
        m += 2;
    }
    Fp2 cpref{1, 0};
    const Fp2 one{1, 0};
    for (int j = 0; j < jb.rounds; ++j) {
        const Fp2* acc = jb.raw + 4 * j;
        const Fp2 h0 = d2mul(cpref, d2add(d2mul(jb.lambda, acc[0]), acc[2]));
        const Fp2 h2 = d2mul(cpref, d2add(d2mul(jb.lambda, acc[1]), acc[3]));
        o[2 * j] = d2sub(h0, m[2 * j]);
        o[2 * j + 1] = d2sub(h2, m[2 * j + 1]);
        const Fp2 pt = jb.pt[j], r = jb.r[j], pr = d2mul(pt, r);
        cpref = d2mul(cpref, d2sub(d2add(d2add(pr, pr), one), d2add(pt, r)));
    }
    const Fp2* s = jb.raw + 4 * jb.rounds;
    o += 2 * jb.rounds;
    m += 2 * jb.rounds;
    for (int k = 0; k < 4; ++k) o[k] = d2sub(s[k], m[k]);
    o[4] = d2sub(d2mul(s[0], s[3]), m[4]);
    o[5] = d2sub(d2mul(s[1], s[2]), m[5]);
    o[6] = d2sub(d2mul(s[2], s[3]), m[6]);
}

template <class P>
int typed_region(Context* c, uint64_t id, size_t off, size_t count, P*& out) {
    void* p = nullptr;
    if (region_elems(c, id, off, count, sizeof(P), &p)) return -1;
    out = static_cast<P*>(p);
    return 0;
}

}  // namespace
}  // namespace vzb

using namespace vzb;

extern "C" int volta_b200_logup_blind_corrections_device(void* raw, const vzb_blind_job* jobs, size_t count) {
    Context* c = static_cast<Context*>(raw);
    if (!c || (count && !jobs)) return fail_message(c, "invalid blind correction jobs");
    std::vector<BlindJob> resolved(count);  // every job checked before anything is launched
    for (size_t i = 0; i < count; ++i) {
        const vzb_blind_job& in = jobs[i];
        BlindJob& jb = resolved[i];
        const size_t rounds = in.rounds, lead = in.root_id ? 2 : 0;
        if (rounds > 64 || in.lambda.c0 >= kP || in.lambda.c1 >= kP)
            return fail_message(c, "invalid blind correction job");
        const size_t outs = lead + 2 * rounds + 7;
        if (typed_region(c, in.raw_id, in.raw_offset, 4 * rounds + 4, jb.raw) ||
            (rounds && typed_region(c, in.sched_id, in.sched_offset, 2 * rounds, jb.pt)) ||
            typed_region(c, in.mask_id, in.mask_offset, outs, jb.mask) ||
            typed_region(c, in.out_id, in.out_offset, outs, jb.out))
            return -1;
        jb.root = nullptr;
        if (in.root_id && typed_region(c, in.root_id, in.root_offset, 2, jb.root)) return -1;
        jb.r = rounds ? jb.pt + rounds : nullptr;
        jb.lambda = Fp2{in.lambda.c0, in.lambda.c1};
        jb.rounds = static_cast<int>(rounds);
    }
    if (op_begin(c) || op_mark(c, 1)) return -1;
    for (size_t base = 0; base < count; base += kBlindJobsPerLaunch) {
        const size_t n = std::min(count - base, size_t(kBlindJobsPerLaunch));
        BlindJobs batch{};
        for (size_t i = 0; i < n; ++i) batch.j[i] = resolved[base + i];
        blind_corrections_kernel<<<1, kBlindJobsPerLaunch, 0, c->stream>>>(batch, static_cast<int>(n));
        VZB_LAUNCHED(c);
    }
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpLogup, 0, 0);
}
