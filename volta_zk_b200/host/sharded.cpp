// Completion of a sharded proof on the host (the shards' local parts come
// from vzh_triple_sumcheck on a slice and vzh_logup_local).  See
// volta_zk_b200/sharded.py for the decomposition: shard g owns the slice
// whose top log2 G index bits equal g; the first k - s rounds of a k-variable
// sumcheck (variables fold LSB-first, rust/volta-proto/src/mle.rs:1-30) stay
// inside a slice, so the global round accumulators are sums of the shards'
// (LogUp: weighted by eq(top coordinates of the claim point, g)), and the last
// s rounds run here on the 2^s values the shards have left.
#include <array>
#include <cstring>

#include "protocol.hpp"

namespace vzh {
namespace {

using vzb::fadd;
using vzb::fmul;
using vzb::fmul7;
using vzb::freduce128;
using vzb::kP;

// prod_b (bit b of g ? point[b] : 1 - point[b])
Fp2 eq_bits(const Fp2* point, size_t bits, size_t g) {
    Fp2 acc{1, 0};
    for (size_t b = 0; b < bits; ++b) acc = f2mul(acc, (g >> b) & 1 ? point[b] : f2sub(Fp2{1, 0}, point[b]));
    return acc;
}

// Suffix-eq table k of `point` (logup.rs:284-305): bit b is point[L - k + b].
std::vector<Fp2> suffix_table(const std::vector<Fp2>& point, size_t k) {
    const size_t L = point.size();
    std::vector<Fp2> t{Fp2{1, 0}};
    for (size_t step = 0; step < k; ++step) {
        const Fp2 p = point[L - 1 - step];
        std::vector<Fp2> nxt;
        nxt.reserve(2 * t.size());
        for (const Fp2& v : t) {
            const Fp2 v1 = f2mul(v, p);
            nxt.push_back(f2sub(v, v1));
            nxt.push_back(v1);
        }
        t.swap(nxt);
    }
    return t;
}

// Unreduced sum of 128-bit products with a carry word: value = carry 2^128 +
// lo, reduced once (2^128 = -2^32 = p - 2^32 mod p).
struct Wide192 {
    unsigned __int128 lo = 0;
    uint64_t carry = 0;
    void mac(uint64_t a, uint64_t b) {
        const unsigned __int128 m = static_cast<unsigned __int128>(a) * b;
        lo += m;
        carry += lo < m;
    }
    uint64_t reduce() const {
        const uint64_t r = freduce128(static_cast<uint64_t>(lo), static_cast<uint64_t>(lo >> 64));
        return fadd(r, fmul(carry, kP - (uint64_t{1} << 32)));
    }
};

// sum_g s[g] * a[g * stride] in Fp2 with one reduction per coordinate
// (s7[g] = 7 s[g].c1): the shard combination of the round accumulators.
Fp2 dot_lazy(const std::vector<Fp2>& sc, const std::vector<uint64_t>& s7, const Fp2* const* a, size_t at) {
    Wide192 c0, c1;
    for (size_t g = 0; g < sc.size(); ++g) {
        const Fp2 v = a[g][at];
        c0.mac(sc[g].c0, v.c0);
        c0.mac(s7[g], v.c1);
        c1.mac(sc[g].c0, v.c1);
        c1.mac(sc[g].c1, v.c0);
    }
    return Fp2{c0.reduce(), c1.reduce()};
}

std::vector<Fp2> fold(const std::vector<Fp2>& v, Fp2 r) {
    std::vector<Fp2> o(v.size() / 2);
    for (size_t i = 0; i < o.size(); ++i) o[i] = f2add(v[2 * i], f2mul(f2sub(v[2 * i + 1], v[2 * i]), r));
    return o;
}

Fp2 at2(Fp2 v0, Fp2 v1) { return f2sub(f2add(v1, v1), v0); }

void triple_round(const std::vector<Fp2>* t, Fp2 g[3]) {
    g[0] = g[1] = g[2] = Fp2{0, 0};
    for (size_t i = 0; i < t[0].size() / 2; ++i) {
        Fp2 x[3][3];
        for (int v = 0; v < 3; ++v) {
            const Fp2 v0 = t[v][2 * i], v1 = t[v][2 * i + 1], d = f2sub(v1, v0), v2 = f2add(v1, d);
            x[v][0] = v0;
            x[v][1] = v2;
            x[v][2] = f2add(v2, d);
        }
        for (int e = 0; e < 3; ++e) g[e] = f2add(g[e], f2mul(f2mul(x[0][e], x[1][e]), x[2][e]));
    }
}

void logup_round(const std::vector<Fp2>* v, const std::vector<Fp2>& s, Fp2 acc[4]) {
    for (int e = 0; e < 4; ++e) acc[e] = Fp2{0, 0};
    for (size_t i = 0; i < v[0].size() / 2; ++i) {
        const Fp2 a0 = v[0][2 * i], a2 = at2(v[0][2 * i], v[0][2 * i + 1]);
        const Fp2 b0 = v[1][2 * i], b2 = at2(v[1][2 * i], v[1][2 * i + 1]);
        const Fp2 c0 = v[2][2 * i], c2 = at2(v[2][2 * i], v[2][2 * i + 1]);
        const Fp2 d0 = v[3][2 * i], d2 = at2(v[3][2 * i], v[3][2 * i + 1]);
        const Fp2 terms[4] = {f2add(f2mul(a0, d0), f2mul(b0, c0)), f2add(f2mul(a2, d2), f2mul(b2, c2)), f2mul(c0, d0),
                              f2mul(c2, d2)};
        for (int e = 0; e < 4; ++e) acc[e] = f2add(acc[e], f2mul(s[i], terms[e]));
    }
}

size_t log2_exact(size_t n) {
    size_t k = 0;
    while ((size_t{1} << k) < n) ++k;
    if ((size_t{1} << k) != n) throw AccelError("sharded sizes must be powers of two");
    return k;
}

size_t local_side_words(size_t depth, size_t s) {
    size_t w = 2;
    for (size_t l = s; l < depth; ++l) w += 4 * (l - s) + 4;
    return w;
}

// One side: parts[g] points at shard g's words for this side.  The top s
// levels of the fraction tree come from the shard roots; every layer's words
// then depend only on the parts, the schedule and those levels, so the layers
// are independent tasks (SideFinish::layer), concatenated in order.
struct SideFinish {
    std::vector<const Fp2*> parts;
    size_t depth = 0, s = 0;
    const SideSchedule* sch = nullptr;
    std::vector<std::vector<Fp2>> lp, lq;  // levels 0 .. s of the tree
    std::vector<size_t> off;               // each shard's word offset of layer l >= s
    std::vector<std::vector<Fp2>> words;   // per layer: 2 per round, then the 4 final values

    SideFinish(const std::vector<const Fp2*>& p, size_t d, size_t s_, const SideSchedule& sc)
        : parts(p), depth(d), s(s_), sch(&sc), lp(s_ + 1), lq(s_ + 1), off(d, 0), words(d) {
        const size_t G = parts.size();
        for (size_t g = 0; g < G; ++g) {
            lp[s].push_back(parts[g][0]);
            lq[s].push_back(parts[g][1]);
        }
        for (size_t lv = s; lv-- > 0;) {
            const auto &cp = lp[lv + 1], &cq = lq[lv + 1];
            for (size_t i = 0; i < cp.size() / 2; ++i) {
                lp[lv].push_back(f2add(f2mul(cp[2 * i], cq[2 * i + 1]), f2mul(cp[2 * i + 1], cq[2 * i])));
                lq[lv].push_back(f2mul(cq[2 * i], cq[2 * i + 1]));
            }
        }
        size_t o = 2;
        for (size_t l = s; l < depth; ++l) {
            off[l] = o;
            o += 4 * (l - s) + 4;
        }
    }

    void layer(size_t l) {
        const SideSchedule& sc = *sch;
        const size_t G = parts.size(), L = l;
        std::vector<std::array<Fp2, 4>> accs;
        std::vector<Fp2> vec[4];
        size_t first_host_round = 0;
        if (l < s) {
            const auto &cp = lp[l + 1], &cq = lq[l + 1];
            for (size_t i = 0; i < cp.size() / 2; ++i) {
                vec[0].push_back(cp[2 * i]);
                vec[1].push_back(cp[2 * i + 1]);
                vec[2].push_back(cq[2 * i]);
                vec[3].push_back(cq[2 * i + 1]);
            }
        } else {
            const size_t Lp = l - s;
            std::vector<Fp2> scale(G);
            std::vector<uint64_t> scale7(G);
            std::vector<const Fp2*> base(G);
            for (size_t g = 0; g < G; ++g) {
                scale[g] = eq_bits(sc.point[l].data() + Lp, s, g);
                scale7[g] = fmul7(scale[g].c1);
                base[g] = parts[g] + off[l];
            }
            for (size_t j = 0; j < Lp; ++j) {
                std::array<Fp2, 4> acc;
                for (int e = 0; e < 4; ++e) acc[e] = dot_lazy(scale, scale7, base.data(), 4 * j + e);
                accs.push_back(acc);
            }
            for (int e = 0; e < 4; ++e)
                for (size_t g = 0; g < G; ++g) vec[e].push_back(base[g][4 * Lp + e]);
            first_host_round = Lp;
        }
        for (size_t j = first_host_round; j < L; ++j) {
            std::array<Fp2, 4> acc;
            logup_round(vec, suffix_table(sc.point[l], L - 1 - j), acc.data());
            accs.push_back(acc);
            for (auto& v : vec) v = fold(v, sc.r[l][j]);
        }
        std::vector<Fp2>& out = words[l];
        out.reserve(2 * L + 4);
        Fp2 cpref{1, 0};
        for (size_t j = 0; j < L; ++j) {
            const auto& a = accs[j];
            out.push_back(f2mul(cpref, f2add(f2mul(sc.lambda[l], a[0]), a[2])));
            out.push_back(f2mul(cpref, f2add(f2mul(sc.lambda[l], a[1]), a[3])));
            cpref = eq_step(cpref, sc.point[l][j], sc.r[l][j]);
        }
        for (auto& v : vec) out.push_back(v[0]);
    }

    void append(std::vector<Fp2>& proof) const {
        proof.push_back(lp[0][0]);
        proof.push_back(lq[0][0]);
        for (const auto& w : words) proof.insert(proof.end(), w.begin(), w.end());
    }
};

}  // namespace

TripleResult triple_finish(const Fp2* parts, size_t G, size_t n, FpStream& tx) {
    const size_t k = log2_exact(n), s = log2_exact(G);
    if (k < s) throw AccelError("more shards than table entries");
    const size_t kl = k - s, per = 3 * kl + 3;
    std::vector<Fp2> r(k);
    for (auto& x : r) x = tx.next_fp2();
    TripleResult out;
    for (size_t j = 0; j < kl; ++j)
        for (int e = 0; e < 3; ++e) {
            Fp2 acc{0, 0};
            for (size_t g = 0; g < G; ++g) acc = f2add(acc, parts[g * per + 3 * j + e]);
            out.messages.push_back(acc);
        }
    std::vector<Fp2> t[3];
    for (int e = 0; e < 3; ++e)
        for (size_t g = 0; g < G; ++g) t[e].push_back(parts[g * per + 3 * kl + e]);
    for (size_t j = kl; j < k; ++j) {
        Fp2 g[3];
        triple_round(t, g);
        out.messages.insert(out.messages.end(), g, g + 3);
        for (auto& v : t) v = fold(v, r[j]);
    }
    for (int e = 0; e < 3; ++e) out.finals[e] = t[e][0];
    return out;
}

std::vector<Fp2> logup_finish(const Fp2* parts, size_t G, size_t words_per_shard, size_t n_f, size_t n_t,
                              FpStream& chal) {
    const size_t s = log2_exact(G), df = log2_exact(n_f), dt = log2_exact(n_t);
    const size_t wf = local_side_words(df, s), wt = local_side_words(dt, s);
    if (words_per_shard != 1 + wf + wt) throw AccelError("shard LogUp parts have the wrong length");
    std::vector<Fp2> proof;
    proof.push_back(chal.next_fp2());  // alpha
    std::vector<const Fp2*> pf(G), pt(G);
    for (size_t g = 0; g < G; ++g) {
        pf[g] = parts + g * words_per_shard + 1;
        pt[g] = pf[g] + wf;
    }
    // both schedules first, in stream order; then every layer of both sides
    // (independent tasks; on one thread: with the branch-free host field
    // arithmetic a 2^24-query finish over 8 shards takes about 0.35 ms,
    // which worker threads no longer shorten)
    const SideSchedule sf = draw_side_schedule(chal, df);
    const SideSchedule st = draw_side_schedule(chal, dt);
    SideFinish fin[2] = {SideFinish(pf, df, s, sf), SideFinish(pt, dt, s, st)};
    for (auto& f : fin)
        for (size_t l = 0; l < f.depth; ++l) f.layer(l);
    fin[0].append(proof);
    fin[1].append(proof);
    return proof;
}

}  // namespace vzh
