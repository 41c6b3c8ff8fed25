// Transcript, wire format and the blind LogUp prover (see transcript.hpp for
// the reference sources each part follows).
#include "transcript.hpp"

#include <cstring>

#include "protocol.hpp"

namespace vzh {

// ---- BLAKE3 (hash and derive-key modes) ----------------------------------------

namespace {

constexpr uint32_t kIv[8] = {0x6A09E667u, 0xBB67AE85u, 0x3C6EF372u, 0xA54FF53Au,
                             0x510E527Fu, 0x9B05688Cu, 0x1F83D9ABu, 0x5BE0CD19u};
constexpr int kMsgPerm[16] = {2, 6, 3, 10, 7, 0, 4, 13, 1, 11, 12, 5, 9, 14, 15, 8};
constexpr uint32_t kChunkStart = 1, kChunkEnd = 2, kParent = 4, kRoot = 8, kDeriveContext = 32, kDeriveMaterial = 64;
constexpr size_t kChunk = 1024, kBlock = 64;

inline uint32_t rotr32(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

inline void quarter(uint32_t* v, int a, int b, int c, int d, uint32_t x, uint32_t y) {
    v[a] += v[b] + x;
    v[d] = rotr32(v[d] ^ v[a], 16);
    v[c] += v[d];
    v[b] = rotr32(v[b] ^ v[c], 12);
    v[a] += v[b] + y;
    v[d] = rotr32(v[d] ^ v[a], 8);
    v[c] += v[d];
    v[b] = rotr32(v[b] ^ v[c], 7);
}

// First eight output words of the compression function.
void compress(const uint32_t cv[8], const uint8_t block[kBlock], uint64_t counter, uint32_t len, uint32_t flags,
              uint32_t out[8]) {
    uint32_t m[16], v[16];
    for (int i = 0; i < 16; ++i) {
        const uint8_t* p = block + 4 * i;
        m[i] = uint32_t(p[0]) | uint32_t(p[1]) << 8 | uint32_t(p[2]) << 16 | uint32_t(p[3]) << 24;
    }
    std::memcpy(v, cv, 32);
    std::memcpy(v + 8, kIv, 16);
    v[12] = static_cast<uint32_t>(counter);
    v[13] = static_cast<uint32_t>(counter >> 32);
    v[14] = len;
    v[15] = flags;
    for (int round = 0; round < 7; ++round) {
        quarter(v, 0, 4, 8, 12, m[0], m[1]);
        quarter(v, 1, 5, 9, 13, m[2], m[3]);
        quarter(v, 2, 6, 10, 14, m[4], m[5]);
        quarter(v, 3, 7, 11, 15, m[6], m[7]);
        quarter(v, 0, 5, 10, 15, m[8], m[9]);
        quarter(v, 1, 6, 11, 12, m[10], m[11]);
        quarter(v, 2, 7, 8, 13, m[12], m[13]);
        quarter(v, 3, 4, 9, 14, m[14], m[15]);
        uint32_t t[16];
        for (int i = 0; i < 16; ++i) t[i] = m[kMsgPerm[i]];
        std::memcpy(m, t, sizeof m);
    }
    for (int i = 0; i < 8; ++i) out[i] = v[i] ^ v[i + 8];
}

// Chaining value of chunk `index` (len <= 1024 bytes; a zero-length input is
// one empty block).
void chunk_cv(const uint32_t key[8], uint32_t mode, const uint8_t* data, size_t len, uint64_t index, bool root,
              uint32_t out[8]) {
    uint32_t cv[8];
    std::memcpy(cv, key, 32);
    const size_t blocks = len ? (len + kBlock - 1) / kBlock : 1;
    for (size_t b = 0; b < blocks; ++b) {
        uint8_t block[kBlock] = {0};
        const size_t take = len ? std::min(kBlock, len - b * kBlock) : 0;
        if (take) std::memcpy(block, data + b * kBlock, take);
        uint32_t flags = mode | (b == 0 ? kChunkStart : 0u);
        if (b + 1 == blocks) flags |= kChunkEnd | (root ? kRoot : 0u);
        compress(cv, block, index, static_cast<uint32_t>(take), flags, cv);
    }
    std::memcpy(out, cv, 32);
}

// The tree over chunks [first, first + count): left subtree the largest
// power of two of chunks below count (the spec's left-balanced tree).
void subtree(const uint32_t key[8], uint32_t mode, const uint8_t* data, size_t len, size_t first, size_t count,
             bool root, uint32_t out[8]) {
    if (count == 1) {
        const size_t off = first * kChunk;
        chunk_cv(key, mode, data + off, std::min(kChunk, len - off), first, root, out);
        return;
    }
    size_t left = 1;
    while (2 * left < count) left *= 2;
    uint32_t children[16];
    subtree(key, mode, data, len, first, left, false, children);
    subtree(key, mode, data, len, first + left, count - left, false, children + 8);
    uint8_t block[kBlock];
    for (int i = 0; i < 16; ++i)
        for (int k = 0; k < 4; ++k) block[4 * i + k] = static_cast<uint8_t>(children[i] >> (8 * k));
    compress(key, block, 0, kBlock, mode | kParent | (root ? kRoot : 0u), out);
}

void root_hash(const uint32_t key[8], uint32_t mode, const uint8_t* data, size_t len, uint8_t out[32]) {
    uint32_t cv[8];
    subtree(key, mode, data, len, 0, len ? (len + kChunk - 1) / kChunk : 1, true, cv);
    for (int i = 0; i < 8; ++i)
        for (int k = 0; k < 4; ++k) out[4 * i + k] = static_cast<uint8_t>(cv[i] >> (8 * k));
}

constexpr const char* kMovesContext = "volta-zk/transcript/canonical-moves/v1";
constexpr uint64_t kTxDomain = ~uint64_t{0};
constexpr size_t kMaxCollection = 1000000;

}  // namespace

void blake3_hash(const uint8_t* data, size_t len, uint8_t out[32]) { root_hash(kIv, 0, data, len, out); }

void blake3_derive_key(const char* context, const uint8_t* data, size_t len, uint8_t out[32]) {
    uint8_t k[32];
    root_hash(kIv, kDeriveContext, reinterpret_cast<const uint8_t*>(context), std::strlen(context), k);
    uint32_t key[8];
    for (int i = 0; i < 8; ++i)
        key[i] = uint32_t(k[4 * i]) | uint32_t(k[4 * i + 1]) << 8 | uint32_t(k[4 * i + 2]) << 16 |
                 uint32_t(k[4 * i + 3]) << 24;
    root_hash(key, kDeriveMaterial, data, len, out);
}

// ---- Transcript --------------------------------------------------------------------

Transcript::Transcript(const uint8_t seed[32]) : chal_(seed, kTxDomain) {}

void Transcript::account(const std::string& label, uint64_t n) {
    ledger_[label] += n;
    ++n_messages_;
}

// kind || u16 label length || label || u64 length || body
void Transcript::event(uint8_t kind, const std::string& label, uint64_t len, const uint8_t* body, size_t body_len) {
    if (label.size() > 0xFFFF) throw AccelError("transcript label exceeds u16");
    moves_.push_back(kind);
    moves_.push_back(static_cast<uint8_t>(label.size()));
    moves_.push_back(static_cast<uint8_t>(label.size() >> 8));
    moves_.insert(moves_.end(), label.begin(), label.end());
    for (int i = 0; i < 8; ++i) moves_.push_back(static_cast<uint8_t>(len >> (8 * i)));
    if (body_len) moves_.insert(moves_.end(), body, body + body_len);
}

void Transcript::append_message(const std::string& label, const uint8_t* msg, size_t len) {
    account(label, len);
    event(1, label, len, msg, len);
}

void Transcript::append_fp2s(const std::string& label, const Fp2* values, size_t n) {
    WireWriter w;
    for (size_t i = 0; i < n; ++i) w.fp2(values[i]);
    append_message(label, w.bytes().data(), w.bytes().size());
}

void Transcript::append_fps(const std::string& label, const uint64_t* values, size_t n) {
    WireWriter w;
    for (size_t i = 0; i < n; ++i) w.u64(values[i]);
    append_message(label, w.bytes().data(), w.bytes().size());
}

void Transcript::append_message_digest(const std::string& label, uint64_t logical_bytes, const uint8_t digest[32]) {
    account(label, logical_bytes);
    event(2, label, logical_bytes, digest, 32);
}

void Transcript::absorb_public_message(const std::string& label, const uint8_t* msg, size_t len) {
    account(label, 0);
    event(5, label, len, msg, len);
}

Fp2 Transcript::challenge_fp2() {
    moves_.push_back(3);
    moves_.push_back(2);
    return chal_.next_fp2();
}

uint64_t Transcript::challenge_fp() {
    moves_.push_back(3);
    moves_.push_back(1);
    return chal_.next_fp();
}

uint64_t Transcript::challenge_bits(unsigned width) {
    if (width < 1 || width > 64) throw AccelError("transcript bit width must be in 1..=64");
    moves_.push_back(3);
    moves_.push_back(3);
    moves_.push_back(static_cast<uint8_t>(width));
    return chal_.next_bits(width);
}

void Transcript::binding_digest(uint8_t out[32]) const {
    blake3_derive_key(kMovesContext, moves_.data(), moves_.size(), out);
}

uint64_t Transcript::bytes_for(const std::string& label) const {
    const auto it = ledger_.find(label);
    return it == ledger_.end() ? 0 : it->second;
}

uint64_t Transcript::total_bytes() const {
    uint64_t t = 0;
    for (const auto& kv : ledger_) t += kv.second;
    return t;
}

// ---- wire format -------------------------------------------------------------------

void WireWriter::len(size_t n) {
    if (n > 0xFFFFFFFFull) throw AccelError("model-proof collection exceeds u32");
    u32(static_cast<uint32_t>(n));
}

uint64_t WireReader::le(int n) {
    if (n_ - off_ < static_cast<size_t>(n)) throw AccelError("truncated model-proof encoding");
    uint64_t v = 0;
    for (int i = 0; i < n; ++i) v |= uint64_t(p_[off_ + i]) << (8 * i);
    off_ += n;
    return v;
}

uint8_t WireReader::u8() { return static_cast<uint8_t>(le(1)); }

Fp2 WireReader::fp2() {
    const uint64_t c0 = u64(), c1 = u64();
    if (c0 >= vzb::kP || c1 >= vzb::kP) throw AccelError("noncanonical Goldilocks element");
    return Fp2{c0, c1};
}

size_t WireReader::len() {
    const size_t n = u32();
    if (n > kMaxCollection) throw AccelError("model-proof collection exceeds strict cap");
    return n;
}

void WireReader::finish() const {
    if (off_ != n_) throw AccelError("trailing model-proof bytes");
}

namespace {

void put_frac(WireWriter& w, const BlindFracProof& p) {
    for (const Fp2& x : p.root_corrs) w.fp2(x);
    w.len(p.layers.size());
    for (const BlindLayerProof& l : p.layers) {
        w.len(l.round_corrs.size());
        for (const auto& r : l.round_corrs) {
            w.fp2(r[0]);
            w.fp2(r[1]);
        }
        for (const Fp2& x : l.split_corrs) w.fp2(x);
        for (const Fp2& x : l.z_corrs) w.fp2(x);
    }
    w.u8(0);  // aux: None
}

BlindFracProof get_frac(WireReader& r) {
    BlindFracProof p;
    for (Fp2& x : p.root_corrs) x = r.fp2();
    p.layers.resize(r.len());
    for (BlindLayerProof& l : p.layers) {
        l.round_corrs.resize(r.len());
        for (auto& rc : l.round_corrs) {
            rc[0] = r.fp2();
            rc[1] = r.fp2();
        }
        for (Fp2& x : l.split_corrs) x = r.fp2();
        for (Fp2& x : l.z_corrs) x = r.fp2();
    }
    const uint8_t tag = r.u8();
    if (tag == 1) throw AccelError("blind LogUp proof with an auxiliary part is not handled by this build");
    if (tag != 0) throw AccelError("noncanonical model-proof option tag");
    return p;
}

}  // namespace

std::vector<uint8_t> encode_blind_logup(const BlindLogupProof& p) {
    WireWriter w;
    put_frac(w, p.lookup);
    put_frac(w, p.table);
    for (const Fp2& x : p.cross_corrs) w.fp2(x);
    return w.bytes();
}

BlindLogupProof decode_blind_logup(const uint8_t* data, size_t len) {
    WireReader r(data, len);
    BlindLogupProof p;
    p.lookup = get_frac(r);
    p.table = get_frac(r);
    for (Fp2& x : p.cross_corrs) x = r.fp2();
    r.finish();
    return p;
}

// ---- the blind LogUp prover ------------------------------------------------------------

namespace {

// Full-field mask values x of one correlation domain (draw_fulls).
std::vector<Fp2> full_masks(const uint8_t seed[32], uint64_t dom, size_t n) {
    if (dom >> 61) throw AccelError("correlation domain cursor entered reserved top bits");
    FpStream xs(seed, dom | (uint64_t{1} << 62));
    std::vector<Fp2> m(n);
    for (auto& x : m) x = xs.next_fp2();
    return m;
}

inline bool same(Fp2 a, Fp2 b) { return a.c0 == b.c0 && a.c1 == b.c1; }

// One side: replays BlindSink::root / lambda / round / splits on the side's
// clear messages (root, then per layer the round pairs and the 4 splits).
BlindFracProof blind_side(const SideSchedule& sch, const uint8_t seed[32], uint64_t& dom, Transcript& tx,
                          const std::vector<Fp2>& words, size_t& pos) {
    BlindFracProof out;
    const Fp2 root[2] = {words[pos], words[pos + 1]};
    pos += 2;
    auto m = full_masks(seed, dom++, 2);
    out.root_corrs = {f2sub(root[0], m[0]), f2sub(root[1], m[1])};
    tx.append_fp2s("logup_root_corrections", out.root_corrs.data(), 2);
    const size_t depth = sch.lambda.size();
    out.layers.resize(depth);
    for (size_t l = 0; l < depth; ++l) {
        BlindLayerProof& lp = out.layers[l];
        if (!same(tx.challenge_fp2(), sch.lambda[l])) throw AccelError("blind LogUp: transcript lambda diverged");
        for (size_t j = 0; j < l; ++j) {
            m = full_masks(seed, dom++, 2);
            lp.round_corrs.push_back({f2sub(words[pos], m[0]), f2sub(words[pos + 1], m[1])});
            pos += 2;
            tx.append_fp2s("logup_round_corrections", lp.round_corrs.back().data(), 2);
            if (!same(tx.challenge_fp2(), sch.r[l][j])) throw AccelError("blind LogUp: transcript challenge diverged");
        }
        const Fp2* s = &words[pos];
        pos += 4;
        m = full_masks(seed, dom++, 4);
        for (int k = 0; k < 4; ++k) lp.split_corrs[k] = f2sub(s[k], m[k]);
        tx.append_fp2s("logup_split_corrections", lp.split_corrs.data(), 4);
        const Fp2 z[3] = {f2mul(s[0], s[3]), f2mul(s[1], s[2]), f2mul(s[2], s[3])};
        m = full_masks(seed, dom++, 3);
        for (int k = 0; k < 3; ++k) lp.z_corrs[k] = f2sub(z[k], m[k]);
        tx.append_fp2s("logup_prod_corrections", lp.z_corrs.data(), 3);
        if (!same(tx.challenge_fp2(), sch.t[l])) throw AccelError("blind LogUp: transcript split challenge diverged");
    }
    return out;
}

}  // namespace

BlindLogupResult blind_logup_prove(Backend& b, uint64_t f_col, size_t n_f, uint64_t t_col, size_t n_t, uint64_t mult,
                                   const uint8_t corr_seed[32], uint64_t dom_base, Transcript& tx) {
    if (n_f < 2 || n_t < 2 || (n_f & (n_f - 1)) || (n_t & (n_t - 1)))
        throw AccelError("blind LogUp sides must have a power-of-two length of at least 2");
    // The clear rounds with the transcript's private stream: the scheduled
    // driver draws alpha and both sides' schedules in the order BlindSink
    // requests them, so replaying the moves below draws the same values.
    BlindLogupResult res;
    std::vector<Fp2> words;
    PendingLogup pl;
    {
        Owned own(b);
        FpStream chal = tx.challenge_stream();
        pl = logup_local_enqueue(b, own, f_col, n_f, t_col, n_t, mult, 0, chal);
        words = logup_local_proof_words(b, pl);
    }
    res.alpha = tx.challenge_fp2();
    if (!same(res.alpha, pl.alpha)) throw AccelError("blind LogUp: transcript alpha diverged");
    uint64_t dom = dom_base;
    size_t pos = 1;
    res.proof.lookup = blind_side(pl.sch[0], corr_seed, dom, tx, words, pos);
    const Fp2 pf = words[1], qf = words[2];
    const size_t table_root = pos;
    res.proof.table = blind_side(pl.sch[1], corr_seed, dom, tx, words, pos);
    if (pos != words.size()) throw AccelError("blind LogUp: proof word count mismatch");
    const Fp2 pt = words[table_root], qt = words[table_root + 1];
    // cross_prover: z_a = p_f q_t, z_b = p_t q_f, 1 / q_f, 1 / q_t
    const Fp2 zx[4] = {f2mul(pf, qt), f2mul(pt, qf), vzb::f2inv(qf), vzb::f2inv(qt)};
    const auto m = full_masks(corr_seed, dom++, 4);
    for (int k = 0; k < 4; ++k) res.proof.cross_corrs[k] = f2sub(zx[k], m[k]);
    tx.append_fp2s("logup_cross_corrections", res.proof.cross_corrs.data(), 4);
    res.next_domain = dom;
    return res;
}

}  // namespace vzh
