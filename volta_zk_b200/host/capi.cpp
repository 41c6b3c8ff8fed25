// C entry points of libvolta_accel.so (the host mirror) for Python/ctypes.
// Every function returns 0 on success, -1 on failure with the message copied
// into `err` (no exception crosses the C boundary).
#include <cstring>
#include <exception>
#include <string>

#include "accel.hpp"
#include "api.hpp"
#include "gpt2.hpp"
#include "protocol.hpp"
#include "transcript.hpp"

using namespace vzh;

namespace {
int fail(char* err, size_t len, const char* msg) {
    if (err && len) {
        std::strncpy(err, msg, len - 1);
        err[len - 1] = 0;
    }
    return -1;
}
template <class F>
int guarded(char* err, size_t len, F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        return fail(err, len, e.what());
    } catch (...) {
        return fail(err, len, "unknown C++ exception");
    }
}
}  // namespace

extern "C" {

// policy: 0 deferred CUDA events, 1 wall-only counters (lib.rs:1009-1044)
void* vzh_open(const char* library, int policy, char* err, size_t len) {
    try {
        return new Backend(library ? library : "", policy ? TimingPolicy::WallOnlyCounters
                                                          : TimingPolicy::DeferredEvents);
    } catch (const std::exception& e) {
        fail(err, len, e.what());
    } catch (...) {
        fail(err, len, "unknown C++ exception");
    }
    return nullptr;
}

void vzh_close(void* h) { delete static_cast<Backend*>(h); }

// on != 0: use the fused fold + round extensions when the library has them
// (the default); 0: the reference's call sequence only.
void vzh_set_fused(void* h, int on) { static_cast<Backend*>(h)->set_fused(on != 0); }

// on != 0: scheduled drivers (challenges first, one message download per
// protocol); 0: one synchronised message per round, as the reference calls.
void vzh_set_scheduled(void* h, int on) { static_cast<Backend*>(h)->set_scheduled(on != 0); }

// on != 0 (default): scheduled LogUp sides run the round steps of their large
// layers as cross-layer batches; 0: layer after layer.
void vzh_set_batched(void* h, int on) { static_cast<Backend*>(h)->set_batched(on != 0); }

void* vzh_context(void* h) { return static_cast<Backend*>(h)->ctx(); }

int vzh_stats(void* h, vz_raw_stats* out, char* err, size_t len) {
    return guarded(err, len, [&] { *out = static_cast<Backend*>(h)->stats(); });
}

int vzh_reset_stats(void* h, char* err, size_t len) {
    return guarded(err, len, [&] { static_cast<Backend*>(h)->reset_stats(); });
}

// Triple-product sumcheck on three resident tables of n Fp2 entries;
// challenges from FpStream(seed, u64::MAX) (a private Transcript).
int vzh_triple_sumcheck(void* h, uint64_t a, uint64_t b, uint64_t c, size_t n, const uint8_t* seed,
                        vz_fp2* messages, vz_fp2* finals, char* err, size_t len) {
    return guarded(err, len, [&] {
        FpStream tx(seed, UINT64_MAX);
        TripleResult r = triple_sumcheck_resident(*static_cast<Backend*>(h), a, b, c, n, tx);
        std::memcpy(messages, r.messages.data(), r.messages.size() * sizeof(vz_fp2));
        std::memcpy(finals, r.finals, sizeof(r.finals));
    });
}

// The same on three resident columns of n canonical Fp values (tables whose
// c1 is 0); the messages equal those of the lifted tables.
int vzh_triple_sumcheck_fp(void* h, uint64_t a, uint64_t b, uint64_t c, size_t n, const uint8_t* seed,
                           vz_fp2* messages, vz_fp2* finals, char* err, size_t len) {
    return guarded(err, len, [&] {
        FpStream tx(seed, UINT64_MAX);
        TripleResult r = triple_sumcheck_resident_fp(*static_cast<Backend*>(h), a, b, c, n, tx);
        std::memcpy(messages, r.messages.data(), r.messages.size() * sizeof(vz_fp2));
        std::memcpy(finals, r.finals, sizeof(r.finals));
    });
}

// The same proof with the columns still in host memory (HostColumns): the
// device columns a, b, c are filled chunk by chunk while the first rounds run.
int vzh_triple_sumcheck_fp_host(void* h, uint64_t a, uint64_t b, uint64_t c, const uint64_t* host_a,
                                const uint64_t* host_b, const uint64_t* host_c, size_t n, size_t chunk,
                                const uint8_t* seed, vz_fp2* messages, vz_fp2* finals, char* err, size_t len) {
    return guarded(err, len, [&] {
        if (!host_a || !host_b || !host_c) throw AccelError("null host column");
        FpStream tx(seed, UINT64_MAX);
        HostColumns hc;
        hc.col[0] = host_a;
        hc.col[1] = host_b;
        hc.col[2] = host_c;
        hc.chunk = chunk;
        TripleResult r = triple_sumcheck_resident_fp(*static_cast<Backend*>(h), a, b, c, n, tx, &hc);
        std::memcpy(messages, r.messages.data(), r.messages.size() * sizeof(vz_fp2));
        std::memcpy(finals, r.finals, sizeof(r.finals));
    });
}

// LogUp proof over resident Fp columns; challenges from FpStream(seed, domain).
int vzh_logup_prove(void* h, uint64_t f_col, size_t n_f, uint64_t t_col, size_t n_t, uint64_t mult,
                    const uint8_t* seed, uint64_t domain, vz_fp2* out, size_t cap, size_t* written,
                    char* err, size_t len) {
    return guarded(err, len, [&] {
        FpStream chal(seed, domain);
        std::vector<Fp2> proof = logup_prove_resident(*static_cast<Backend*>(h), f_col, n_f, t_col, n_t, mult, chal);
        if (proof.size() > cap) throw AccelError("logup proof buffer too small");
        std::memcpy(out, proof.data(), proof.size() * sizeof(vz_fp2));
        *written = proof.size();
    });
}

// Ligero commitment + openings (see accel.hpp); challenges from
// FpStream(chal_seed, u64::MAX).  columns: queries x rows u64, paths:
// queries x log2(code_len) x 32 bytes.
int vzh_ligero_commit_open(void* h, const uint8_t* row_seed, size_t rows, size_t msg_len, size_t code_len,
                           size_t queries, const uint8_t* chal_seed, uint8_t* root, uint32_t* indices,
                           uint64_t* columns, uint8_t* paths, char* err, size_t len) {
    return guarded(err, len, [&] {
        FpStream tx(chal_seed, UINT64_MAX);
        LigeroOpening o = ligero_commit_open_resident(*static_cast<Backend*>(h), row_seed, rows, msg_len, code_len,
                                                      queries, tx);
        std::memcpy(root, o.root, 32);
        std::memcpy(indices, o.indices.data(), o.indices.size() * sizeof(uint32_t));
        std::memcpy(columns, o.columns.data(), o.columns.size() * sizeof(uint64_t));
        std::memcpy(paths, o.paths.data(), o.paths.size());
    });
}

// One shard's share of a LogUp proof (both sides, see frac_side_local):
// leaves are this shard's slices of the query / table columns (n_f_local,
// n_t_local entries), shard_bits = log2(shards).  Output (Fp2 words): alpha,
// then per side root_p, root_q and per global layer l >= shard_bits the
// 4 (l - shard_bits) local round accumulators followed by 4 left-over values.
int vzh_logup_local(void* h, uint64_t f_col, size_t n_f_local, uint64_t t_col, size_t n_t_local, uint64_t mult,
                    size_t shard_bits, const uint8_t* seed, uint64_t domain, vz_fp2* out, size_t cap,
                    size_t* written, char* err, size_t len) {
    return guarded(err, len, [&] {
        Backend& b = *static_cast<Backend*>(h);
        FpStream chal(seed, domain);
        Owned own(b);
        const PendingLogup pl = logup_local_enqueue(b, own, f_col, n_f_local, t_col, n_t_local, mult, shard_bits, chal);
        const std::vector<Fp2> words = logup_local_collect(b, pl);
        if (words.size() > cap) throw AccelError("local LogUp buffer too small");
        std::memcpy(out, words.data(), words.size() * sizeof(vz_fp2));
        *written = words.size();
    });
}

// One shard's whole config-1 part in one call: both LogUp sides and then the
// triple-product sumcheck of its table slices (Fp columns when base != 0) are
// enqueued back to back and downloaded once; the triple part first waits for
// the context's asynchronous uploads (volta_b200_wait_uploads), so its tables
// may still be arriving while the LogUp part computes.  out = the triple's
// 3 k messages and 3 finals (k = log2 n_local), then the words of
// vzh_logup_local.  Needs the scheduled drivers.
static void proof_local(Backend& b, uint64_t a, uint64_t bb, uint64_t c, size_t n_local, int base,
                        const HostColumns* host, const uint8_t* triple_seed, uint64_t f_col, size_t n_f_local,
                        uint64_t t_col, size_t n_t_local, uint64_t mult, size_t shard_bits, const uint8_t* logup_seed,
                        uint64_t domain, vz_fp2* out, size_t cap, size_t* written) {
    if (!b.scheduled()) throw AccelError("vzh_proof_local needs the scheduled drivers");
    if (base && !(b.ext().triple_round_fp && b.ext().triple_fold_round_fp && n_local >= 4))
        throw AccelError("vzh_proof_local: base-field rounds unavailable for this table length");
    FpStream tx(triple_seed, UINT64_MAX);
    FpStream chal(logup_seed, domain);
    Owned own(b);
    const PendingLogup pl = logup_local_enqueue(b, own, f_col, n_f_local, t_col, n_t_local, mult, shard_bits, chal);
    if (b.ext().wait_uploads) b.check(b.ext().wait_uploads(b.ctx()), "volta_b200_wait_uploads");
    size_t k = 0;
    const uint64_t tm = triple_enqueue(b, own, a, bb, c, n_local, tx, base != 0, k, host);
    const std::vector<Fp2> words = logup_local_collect(b, pl);
    const TripleResult tr = triple_collect(b, tm, k);
    const size_t total = tr.messages.size() + 3 + words.size();
    if (total > cap) throw AccelError("local proof buffer too small");
    std::memcpy(out, tr.messages.data(), tr.messages.size() * sizeof(vz_fp2));
    std::memcpy(out + tr.messages.size(), tr.finals, sizeof(tr.finals));
    std::memcpy(out + tr.messages.size() + 3, words.data(), words.size() * sizeof(vz_fp2));
    *written = total;
}

int vzh_proof_local(void* h, uint64_t a, uint64_t bb, uint64_t c, size_t n_local, int base,
                    const uint8_t* triple_seed, uint64_t f_col, size_t n_f_local, uint64_t t_col, size_t n_t_local,
                    uint64_t mult, size_t shard_bits, const uint8_t* logup_seed, uint64_t domain, vz_fp2* out,
                    size_t cap, size_t* written, char* err, size_t len) {
    return guarded(err, len, [&] {
        proof_local(*static_cast<Backend*>(h), a, bb, c, n_local, base, nullptr, triple_seed, f_col, n_f_local, t_col,
                    n_t_local, mult, shard_bits, logup_seed, domain, out, cap, written);
    });
}

// The same with the triple columns still in host memory (base-field columns):
// they upload chunk by chunk on the copy stream while the LogUp part and the
// first triple rounds compute.
int vzh_proof_local_host(void* h, uint64_t a, uint64_t bb, uint64_t c, const uint64_t* host_a,
                         const uint64_t* host_b, const uint64_t* host_c, size_t chunk, size_t n_local,
                         const uint8_t* triple_seed, uint64_t f_col, size_t n_f_local, uint64_t t_col,
                         size_t n_t_local, uint64_t mult, size_t shard_bits, const uint8_t* logup_seed,
                         uint64_t domain, vz_fp2* out, size_t cap, size_t* written, char* err, size_t len) {
    return guarded(err, len, [&] {
        if (!host_a || !host_b || !host_c) throw AccelError("null host column");
        HostColumns hc;
        hc.col[0] = host_a;
        hc.col[1] = host_b;
        hc.col[2] = host_c;
        hc.chunk = chunk;
        proof_local(*static_cast<Backend*>(h), a, bb, c, n_local, 1, &hc, triple_seed, f_col, n_f_local, t_col,
                    n_t_local, mult, shard_bits, logup_seed, domain, out, cap, written);
    });
}

// Weight-matrix commitment + zero-knowledge multi-claim opening, device part
// (see accel.hpp).  Claim g has point_lens[g] coordinates, concatenated in
// `points`, and offsets[g]; outputs as in LigeroZkOpening (flat arrays).
int vzh_ligero_commit_open_zk(void* h, const int16_t* weights, size_t rows, size_t col_bits, size_t pad,
                              size_t code_bits, const uint8_t* pad_seed, size_t claims, const uint64_t* offsets,
                              const size_t* point_lens, const vz_fp2* points, const uint8_t* mask_seed, uint64_t c0,
                              uint64_t c1, const uint32_t* indices, size_t queries, uint8_t* root, uint8_t* mask_root,
                              vz_fp2* u_c, vz_fp2* u_g, vz_fp2* s, uint64_t* columns, vz_fp2* mask_columns,
                              uint8_t* paths, uint8_t* mask_paths, double* phase_ms, char* err, size_t len) {
    return guarded(err, len, [&] {
        LigeroShape sh;
        sh.rows = rows;
        sh.col_bits = col_bits;
        sh.pad = pad;
        sh.code_bits = code_bits;
        std::vector<ZkClaim> cl(claims);
        size_t at = 0;
        for (size_t g = 0; g < claims; ++g) {
            cl[g].offset = offsets[g];
            cl[g].point.assign(points + at, points + at + point_lens[g]);
            at += point_lens[g];
        }
        const std::vector<uint32_t> idx(indices, indices + queries);
        const LigeroZkOpening o =
            ligero_commit_open_zk(*static_cast<Backend*>(h), weights, sh, pad_seed, cl, mask_seed, Fp2{c0, c1}, idx,
                                  phase_ms);
        std::memcpy(root, o.root, 32);
        std::memcpy(mask_root, o.mask_root, 32);
        std::memcpy(u_c, o.u_c.data(), o.u_c.size() * sizeof(vz_fp2));
        std::memcpy(u_g, o.u_g.data(), o.u_g.size() * sizeof(vz_fp2));
        std::memcpy(s, o.s.data(), o.s.size() * sizeof(vz_fp2));
        std::memcpy(columns, o.columns.data(), o.columns.size() * sizeof(uint64_t));
        std::memcpy(mask_columns, o.mask_columns.data(), o.mask_columns.size() * sizeof(vz_fp2));
        std::memcpy(paths, o.paths.data(), o.paths.size());
        std::memcpy(mask_paths, o.mask_paths.data(), o.mask_paths.size());
    });
}

// Sharded-proof completion (see accel.hpp); no device involved.
int vzh_triple_finish(const vz_fp2* parts, size_t shards, size_t n, const uint8_t* seed, vz_fp2* messages,
                      vz_fp2* finals, char* err, size_t len) {
    return guarded(err, len, [&] {
        FpStream tx(seed, UINT64_MAX);
        TripleResult r = triple_finish(parts, shards, n, tx);
        std::memcpy(messages, r.messages.data(), r.messages.size() * sizeof(vz_fp2));
        std::memcpy(finals, r.finals, sizeof(r.finals));
    });
}

int vzh_logup_finish(const vz_fp2* parts, size_t shards, size_t words_per_shard, size_t n_f, size_t n_t,
                     const uint8_t* seed, uint64_t domain, vz_fp2* out, size_t cap, size_t* written, char* err,
                     size_t len) {
    return guarded(err, len, [&] {
        FpStream chal(seed, domain);
        std::vector<Fp2> proof = logup_finish(parts, shards, words_per_shard, n_f, n_t, chal);
        if (proof.size() > cap) throw AccelError("logup proof buffer too small");
        std::memcpy(out, proof.data(), proof.size() * sizeof(vz_fp2));
        *written = proof.size();
    });
}

// The first n Fp2 draws of FpStream(seed, domain) (challenge schedules).
void vzh_fpstream_fp2(const uint8_t* seed, uint64_t domain, size_t n, vz_fp2* out) {
    FpStream s(seed, domain);
    for (size_t i = 0; i < n; ++i) out[i] = s.next_fp2();
}

// ---- whole-model GPT-2 session (gpt2.hpp) ----------------------------------
// dims: layers, d, heads, head_dim, dff, vocab, positions, t.
// shifts: ln_var, ln_norm, recip_den, recip_log2, qkv, scores, softmax_norm,
// av, attn_proj, ffn_up, ffn_down, embed (two's complement), row_shift flag.
// layer_weights: layers x 8 pointers (c_attn, attn_proj, ffn_up, ffn_down,
// ln1_gain, ln1_bias, ln2_gain, ln2_bias); luts: ln_rsqrt, exp,
// softmax_recip, gelu with their lengths.
void* vzh_gpt2_open(void* h, const size_t* dims, const uint32_t* shifts, const int16_t* const* layer_weights,
                    const int16_t* wte, const int16_t* wpe, const int16_t* lnf_gain, const int16_t* lnf_bias,
                    const int16_t* const* luts, const size_t* lut_lens, char* err, size_t len) {
    try {
        Gpt2Shape s;
        s.layers = dims[0];
        s.d = dims[1];
        s.heads = dims[2];
        s.head_dim = dims[3];
        s.dff = dims[4];
        s.vocab = dims[5];
        s.positions = dims[6];
        s.t = dims[7];
        Gpt2Shifts& f = s.shifts;
        f.ln_var = shifts[0];
        f.ln_norm = shifts[1];
        f.recip_den = shifts[2];
        f.recip_log2 = shifts[3];
        f.qkv = shifts[4];
        f.scores = shifts[5];
        f.softmax_norm = shifts[6];
        f.av = shifts[7];
        f.attn_proj = shifts[8];
        f.ffn_up = shifts[9];
        f.ffn_down = shifts[10];
        f.embed = static_cast<int32_t>(shifts[11]);
        f.row_shift = shifts[12] != 0;
        std::vector<Gpt2LayerHost> lw(s.layers);
        for (size_t l = 0; l < s.layers; ++l) {
            const int16_t* const* p = layer_weights + 8 * l;
            lw[l] = Gpt2LayerHost{p[0], p[1], p[2], p[3], p[4], p[5], p[6], p[7]};
        }
        return new Gpt2Session(*static_cast<Backend*>(h), s, lw, wte, wpe, lnf_gain, lnf_bias,
                               {luts[0], luts[1], luts[2], luts[3]},
                               {lut_lens[0], lut_lens[1], lut_lens[2], lut_lens[3]});
    } catch (const std::exception& e) {
        fail(err, len, e.what());
    } catch (...) {
        fail(err, len, "unknown C++ exception");
    }
    return nullptr;
}

void vzh_gpt2_close(void* s) { delete static_cast<Gpt2Session*>(s); }

// Enqueue the whole forward; tokens (t u32 ids) are uploaded first when given,
// else the session's resident token buffer is used.
int vzh_gpt2_forward(void* s, const uint32_t* tokens, char* err, size_t len) {
    return guarded(err, len, [&] {
        Gpt2Session& g = *static_cast<Gpt2Session*>(s);
        if (tokens) g.upload_tokens(tokens);
        g.forward(g.tokens_id());
    });
}

// Arena id of one resident buffer: wire w of layer l (w < kWireCount), or for
// l == SIZE_MAX: 0 tokens, 1 embed acc, 2 logits, 3 error word, 4..9 final
// LN (mean, var, rin, rout, acc, out), 10..13 luts, 14 wte.
uint64_t vzh_gpt2_buffer(void* s, size_t layer, int which) {
    const Gpt2Session& g = *static_cast<Gpt2Session*>(s);
    if (layer != SIZE_MAX) {
        if (layer >= g.shape().layers || which < 0 || which >= kWireCount) return 0;
        return g.wire(layer, which);
    }
    switch (which) {
        case 0: return g.tokens_id();
        case 1: return g.embed_acc();
        case 2: return g.logits();
        case 3: return g.error_word();
        case 14: return g.wte();
        default:
            if (which >= 4 && which <= 9) return g.final_ln(which - 4);
            if (which >= 10 && which <= 13) return g.lut(which - 10);
            return 0;
    }
}

// The prefill proof schedule over a session's witness (gpt2_proof.cpp).
void* vzh_gpt2_prover_open(void* session, char* err, size_t len) {
    try {
        return new Gpt2Prover(*static_cast<Gpt2Session*>(session));
    } catch (const std::exception& e) {
        fail(err, len, e.what());
    } catch (...) {
        fail(err, len, "unknown C++ exception");
    }
    return nullptr;
}

void vzh_gpt2_prover_close(void* p) { delete static_cast<Gpt2Prover*>(p); }

int vzh_gpt2_prove_layers(void* p, const uint8_t* seed, const uint8_t* mac_seed, const uint8_t* pad_seed,
                          size_t first, size_t stride, int with_pcs, vz_fp2* words, size_t cap, size_t* written,
                          size_t* per_layer, uint8_t* root, char* err, size_t len);

// Prove the session's last forward.  words: every layer's words in order
// (cap Fp2 at most; *written gets the total and *per_layer the count of
// one layer); root: the 32-byte PCS commitment.
int vzh_gpt2_prove(void* p, const uint8_t* seed, const uint8_t* mac_seed, const uint8_t* pad_seed, vz_fp2* words,
                   size_t cap, size_t* written, size_t* per_layer, uint8_t* root, char* err, size_t len) {
    return vzh_gpt2_prove_layers(p, seed, mac_seed, pad_seed, 0, 1, 1, words, cap, written, per_layer, root, err,
                                 len);
}

// Layers first, first + stride, ... only (with_pcs: also the weight
// commitment); words of the proved layers in layer order.
int vzh_gpt2_prove_layers(void* p, const uint8_t* seed, const uint8_t* mac_seed, const uint8_t* pad_seed,
                          size_t first, size_t stride, int with_pcs, vz_fp2* words, size_t cap, size_t* written,
                          size_t* per_layer, uint8_t* root, char* err, size_t len) {
    return guarded(err, len, [&] {
        const Gpt2Proof pr =
            static_cast<Gpt2Prover*>(p)->prove_layers(seed, mac_seed, pad_seed, first, stride, with_pcs != 0);
        size_t total = 0;
        for (const auto& w : pr.layer_words) total += w.size();
        if (total > cap) throw AccelError("GPT-2 proof buffer too small");
        size_t at = 0;
        for (const auto& w : pr.layer_words) {
            std::memcpy(words + at, w.data(), w.size() * sizeof(vz_fp2));
            at += w.size();
        }
        *written = total;
        *per_layer = pr.layer_words.empty() ? 0 : pr.layer_words[0].size();
        std::memcpy(root, pr.pcs_root, 32);
    });
}

// The units (layers[u], sites[u]) of a proof only, in that order (one GPU's
// share of a proof split by sites; site k = bit k, 0 the boundary
// corrections): words of every unit in order; per proved site, in order, its
// id and word count (site_ids / site_words, site_cap entries at most,
// *n_sites written) and per unit its site count (unit_sites, n_units).
int vzh_gpt2_prove_units(void* p, const uint8_t* seed, const uint8_t* mac_seed, const uint8_t* pad_seed,
                         const size_t* layers, const uint32_t* sites, size_t n_units, int with_pcs, vz_fp2* words,
                         size_t cap, size_t* written, uint32_t* site_ids, size_t* site_words, size_t site_cap,
                         size_t* n_sites, size_t* unit_sites, uint8_t* root, char* err, size_t len) {
    return guarded(err, len, [&] {
        std::vector<Gpt2Unit> units(n_units);
        for (size_t u = 0; u < n_units; ++u) units[u] = Gpt2Unit{layers[u], sites[u]};
        const Gpt2Proof pr = static_cast<Gpt2Prover*>(p)->prove_units(seed, mac_seed, pad_seed, units, with_pcs != 0);
        size_t total = 0, ns = 0;
        for (size_t u = 0; u < pr.layer_words.size(); ++u) {
            total += pr.layer_words[u].size();
            ns += pr.unit_sites[u].size();
        }
        if (total > cap) throw AccelError("GPT-2 proof buffer too small");
        if (ns > site_cap) throw AccelError("GPT-2 proof site buffer too small");
        size_t at = 0, k = 0;
        for (size_t u = 0; u < pr.layer_words.size(); ++u) {
            std::memcpy(words + at, pr.layer_words[u].data(), pr.layer_words[u].size() * sizeof(vz_fp2));
            at += pr.layer_words[u].size();
            unit_sites[u] = pr.unit_sites[u].size();
            for (const auto& st : pr.unit_sites[u]) {
                site_ids[k] = static_cast<uint32_t>(st.first);
                site_words[k++] = st.second;
            }
        }
        *written = total;
        *n_sites = ns;
        std::memcpy(root, pr.pcs_root, 32);
    });
}

// A decode band's proof (chunk >= 1) over the prover's session: layers first,
// first + stride, ... in layer order; no weight commitment.
int vzh_gpt2_prove_band(void* p, void* band, size_t chunk, const uint8_t* seed, const uint8_t* mac_seed,
                        size_t first, size_t stride, vz_fp2* words, size_t cap, size_t* written, size_t* per_layer,
                        char* err, size_t len) {
    return guarded(err, len, [&] {
        if (!band) throw AccelError("no band");
        const Gpt2Proof pr = static_cast<Gpt2Prover*>(p)->prove_band(*static_cast<Gpt2Band*>(band), chunk, seed,
                                                                     mac_seed, first, stride);
        size_t total = 0;
        for (const auto& w : pr.layer_words) total += w.size();
        if (total > cap) throw AccelError("GPT-2 proof buffer too small");
        size_t at = 0;
        for (const auto& w : pr.layer_words) {
            std::memcpy(words + at, w.data(), w.size() * sizeof(vz_fp2));
            at += w.size();
        }
        *written = total;
        *per_layer = pr.layer_words.empty() ? 0 : pr.layer_words[0].size();
    });
}

// Band witness of rows t0 .. t-1 of a session's last forward (band.rs).
void* vzh_gpt2_band_open(void* session, size_t t0, char* err, size_t len) {
    try {
        return new Gpt2Band(*static_cast<Gpt2Session*>(session), t0);
    } catch (const std::exception& e) {
        fail(err, len, e.what());
    } catch (...) {
        fail(err, len, "unknown C++ exception");
    }
    return nullptr;
}

void vzh_gpt2_band_close(void* b) { delete static_cast<Gpt2Band*>(b); }

int vzh_gpt2_band_build(void* b, char* err, size_t len) {
    return guarded(err, len, [&] { static_cast<Gpt2Band*>(b)->build(); });
}

// Buffer id and element offset of band wire w of layer l; for l == SIZE_MAX:
// 0..5 final LN (mean, var, rin, rout, acc, out), 6 logits (q x vocab), 7 the
// band's error word (offset 0).
int vzh_gpt2_band_buffer(void* b, size_t layer, int which, uint64_t* id, size_t* offset, char* err, size_t len) {
    return guarded(err, len, [&] {
        const Gpt2Band& g = *static_cast<Gpt2Band*>(b);
        *offset = 0;
        if (layer != SIZE_MAX) {
            const auto w = g.wire(layer, which);
            *id = w.first;
            *offset = w.second;
        } else if (which >= 0 && which <= 5) {
            *id = g.final_ln(which);
        } else if (which == 6) {
            *id = g.logits();
        } else if (which == 7) {
            *id = g.error_word();
        } else {
            throw AccelError("unknown band buffer");
        }
    });
}

// KV-cached greedy decoding after a session's forward (decode.rs).
void* vzh_gpt2_decoder_open(void* session, size_t max_steps, char* err, size_t len) {
    try {
        return new Gpt2Decoder(*static_cast<Gpt2Session*>(session), max_steps);
    } catch (const std::exception& e) {
        fail(err, len, e.what());
    } catch (...) {
        fail(err, len, "unknown C++ exception");
    }
    return nullptr;
}

void vzh_gpt2_decoder_close(void* d) { delete static_cast<Gpt2Decoder*>(d); }

int vzh_gpt2_decode(void* d, size_t n, char* err, size_t len) {
    return guarded(err, len, [&] { static_cast<Gpt2Decoder*>(d)->generate(n); });
}

// 0 tokens (u32), 1 logits rows (i64), 2 error word, 3 K cache of `layer`,
// 4 V cache of `layer`; 5 the next position (not an id).
uint64_t vzh_gpt2_decoder_buffer(void* d, size_t layer, int which) {
    const Gpt2Decoder& g = *static_cast<Gpt2Decoder*>(d);
    switch (which) {
        case 0: return g.tokens();
        case 1: return g.logits();
        case 2: return g.error_word();
        case 3: return g.cache(layer, 0);
        case 4: return g.cache(layer, 1);
        case 5: return g.position();
        default: return 0;
    }
}

// Host wall time of the prover's last proof: enqueueing its launches, and in all.
void vzh_gpt2_prover_timing(void* p, double* enqueue_ms, double* total_ms) {
    const Gpt2Prover& g = *static_cast<Gpt2Prover*>(p);
    *enqueue_ms = g.host_enqueue_ms();
    *total_ms = g.host_total_ms();
}

// One GPU's row block of the weight commitment: the column chaining values
// of rows row0 .. row0 + rows - 1 (code_len x 32 bytes into cvs).
int vzh_gpt2_commit_rows(void* p, const uint8_t* pad_seed, size_t row0, size_t rows, uint8_t* cvs, char* err,
                         size_t len) {
    return guarded(err, len, [&] { static_cast<Gpt2Prover*>(p)->commit_rows(pad_seed, row0, rows, cvs); });
}

// Host destination of every later proof's boundary corrections (nullptr: none).
void vzh_gpt2_set_correction_sink(void* p, uint64_t* host) { static_cast<Gpt2Prover*>(p)->set_correction_sink(host); }

// Rows of the prover's weight commitment (8192 for GPT-2 small).
size_t vzh_gpt2_prover_pcs_rows(void* p) { return static_cast<Gpt2Prover*>(p)->pcs_rows(); }

// Arena id of the boundary corrections of wire w (0..4) of layer l.
uint64_t vzh_gpt2_correction(void* p, size_t layer, int w) {
    try {
        return static_cast<Gpt2Prover*>(p)->correction(layer, w);
    } catch (...) {
        return 0;
    }
}

// The first n Fp draws (rejection-sampled next_fp) of FpStream(seed, domain):
// row `domain` of the ChaCha8 prover-secret rows (input synthesis).
void vzh_fpstream_fp(const uint8_t* seed, uint64_t domain, size_t n, uint64_t* out) {
    FpStream s(seed, domain);
    for (size_t i = 0; i < n; ++i) out[i] = s.next_fp();
}

// Raw u64 draws of FpStream(seed, domain) (input synthesis for benches).
void vzh_fpstream_u64(const uint8_t* seed, uint64_t domain, size_t n, uint64_t* out) {
    FpStream s(seed, domain);
    for (size_t i = 0; i < n; ++i) out[i] = s.next_u64();
}

// BLAKE3 of `len` bytes: plain hash (context null) or derive-key mode with
// the given context string (the transcript's binding hash).
void vzh_blake3(const char* context, const uint8_t* data, size_t len, uint8_t* out) {
    if (context)
        blake3_derive_key(context, data, len, out);
    else
        blake3_hash(data, len, out);
}

// Blind LogUp proof (logup.rs:3184-3225 blind_logup_prove) of the resident
// query column f_col (n_f canonical Fp values), table column t_col (n_t) and
// u32 multiplicities mult, with a fresh transcript Transcript::new(tx_seed)
// and the mock correlation stream seeded with corr_seed, domains from
// dom_base.  Writes the BlindLogupProof wire bytes (model_proof_codec.rs
// rules) to out (cap bytes; *written), the transcript's canonical binding
// digest (32 bytes), its charged bytes and the domain cursor after the proof.
int vzh_blind_logup_prove(void* h, uint64_t f_col, size_t n_f, uint64_t t_col, size_t n_t, uint64_t mult,
                          const uint8_t* tx_seed, const uint8_t* corr_seed, uint64_t dom_base, uint8_t* out,
                          size_t cap, size_t* written, uint8_t* digest, uint64_t* tx_bytes, uint64_t* next_dom,
                          char* err, size_t len) {
    return guarded(err, len, [&] {
        Transcript tx(tx_seed);
        const BlindLogupResult r =
            blind_logup_prove(*static_cast<Backend*>(h), f_col, n_f, t_col, n_t, mult, corr_seed, dom_base, tx);
        const std::vector<uint8_t> bytes = encode_blind_logup(r.proof);
        if (bytes.size() > cap) throw AccelError("blind LogUp proof buffer too small");
        std::memcpy(out, bytes.data(), bytes.size());
        *written = bytes.size();
        tx.binding_digest(digest);
        *tx_bytes = tx.total_bytes();
        *next_dom = r.next_domain;
    });
}

// Decode and re-encode BlindLogupProof wire bytes (strict: canonical field
// elements, collection caps, option tags, no trailing bytes); writes the
// per-layer round counts of both sides (lookup side first) to rounds.
int vzh_blind_logup_check(const uint8_t* data, size_t n, uint32_t* rounds, size_t rounds_cap, size_t* layers,
                          char* err, size_t len) {
    return guarded(err, len, [&] {
        const BlindLogupProof p = decode_blind_logup(data, n);
        size_t k = 0;
        for (const BlindFracProof* side : {&p.lookup, &p.table})
            for (const BlindLayerProof& l : side->layers) {
                if (k == rounds_cap) throw AccelError("rounds buffer too small");
                rounds[k++] = static_cast<uint32_t>(l.round_corrs.size());
            }
        *layers = k;
        if (encode_blind_logup(p) != std::vector<uint8_t>(data, data + n))
            throw AccelError("blind LogUp proof does not re-encode to its bytes");
    });
}

}  // extern "C"
