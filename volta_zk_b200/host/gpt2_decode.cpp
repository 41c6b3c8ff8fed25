// Decode bands and KV-cached greedy decoding over the resident GPT-2 session
// (see gpt2.hpp for the reference sources each part follows).
#include <algorithm>

#include "api.hpp"
#include "gpt2.hpp"

namespace vzh {

namespace {

size_t tri(size_t x) { return x * (x + 1) / 2; }

}  // namespace

// ---- band witness ------------------------------------------------------------------

Gpt2Band::Gpt2Band(Gpt2Session& s, size_t t0) : s_(s), t0_(t0) {
    const Gpt2Shape& sh = s_.shape();
    if (t0 == 0 || t0 >= sh.t) throw AccelError("band must be a proper suffix of the forward (0 < t0 < t)");
    q_ = sh.t - t0;
    Backend& b = s_.backend();
    const size_t h = sh.heads, d = sh.d, bc = q_ * t0_ + tri(q_);
    auto alloc = [&](size_t bytes) {
        const uint64_t id = b.alloc(std::max<size_t>(bytes, 16));
        owned_.push_back(id);
        return id;
    };
    try {
        derived_.resize(sh.layers);
        for (auto& dv : derived_) {
            dv[0] = alloc(8 * h * bc);  // scores_acc
            dv[1] = alloc(2 * h * bc);  // scores_q
            dv[2] = alloc(2 * h * q_);  // row_shift
            dv[3] = alloc(2 * h * bc);  // exp_out
            dv[4] = alloc(8 * h * q_);  // denoms
            dv[5] = alloc(2 * h * q_);  // recips
            dv[6] = alloc(2 * h * bc);  // weights
        }
        const size_t fin_elem[6] = {8, 8, 8, 2, 8, 2}, fin_count[6] = {q_, q_, q_, q_, q_ * d, q_ * d};
        for (int k = 0; k < 6; ++k) fin_[k] = alloc(fin_elem[k] * fin_count[k]);
        logits_ = alloc(8 * q_ * sh.vocab);
        err_ = alloc(4);
    } catch (...) {
        for (uint64_t id : owned_) b.api().volta_cuda_resident_free(b.ctx(), id);
        throw;
    }
}

Gpt2Band::~Gpt2Band() {
    Backend& b = s_.backend();
    for (uint64_t id : owned_) b.api().volta_cuda_resident_free(b.ctx(), id);
}

void Gpt2Band::build() {
    Backend& b = s_.backend();
    const Api& A = b.api();
    void* c = b.ctx();
    const Gpt2Shape& sh = s_.shape();
    const size_t t = sh.t, h = sh.heads, d = sh.d, bc = q_ * t0_ + tri(q_), full = tri(t), start = tri(t0_);
    // packed per-head fields: head h's rows t0 .. t-1 are the tail of its segment
    const int packed[4] = {kScoresAcc, kScoresQ, kExpOut, kWeights};
    const int packed_slot[4] = {0, 1, 3, 6};
    const size_t packed_elem[4] = {8, 2, 2, 2};
    const int table[3] = {kRowShift, kDenoms, kRecips};
    const int table_slot[3] = {2, 4, 5};
    const size_t table_elem[3] = {2, 8, 2};
    for (size_t l = 0; l < sh.layers; ++l) {
        for (int k = 0; k < 4; ++k) {
            const size_t e = packed_elem[k];
            b.check(A.volta_cuda_resident_copy_rows(c, s_.wire(l, packed[k]), start * e, full * e,
                                                    derived_[l][packed_slot[k]], 0, bc * e, h, bc * e),
                    "resident_copy_rows");
        }
        for (int k = 0; k < 3; ++k) {
            const size_t e = table_elem[k];
            b.check(A.volta_cuda_resident_copy_rows(c, s_.wire(l, table[k]), t0_ * e, t * e,
                                                    derived_[l][table_slot[k]], 0, q_ * e, h, q_ * e),
                    "resident_copy_rows");
        }
    }
    const Gpt2Shifts& f = sh.shifts;
    b.check(A.volta_cuda_resident_zero(c, err_, 0, sizeof(uint32_t)), "resident_zero");
    b.check(A.volta_cuda_fixed_layer_norm_device(c, s_.wire(sh.layers - 1, kFfnOut), t0_ * d, s_.lnf(0), 0, s_.lnf(1),
                                                  0, s_.lut(0), 0, fin_[0], 0, fin_[1], 0, fin_[2], 0, fin_[3], 0,
                                                  fin_[4], 0, fin_[5], 0, err_, 0, q_, d, f.ln_var, f.ln_norm),
             "fixed_layer_norm_device");
    b.check(A.volta_cuda_fixed_logits_device(c, fin_[5], 0, s_.wte(), 0, logits_, 0, q_, d, sh.vocab),
            "fixed_logits_device");
}

std::pair<uint64_t, size_t> Gpt2Band::wire(size_t layer, int w) const {
    const Gpt2Shape& sh = s_.shape();
    if (layer >= sh.layers) throw AccelError("band layer out of range");
    switch (w) {
        case kScoresAcc: return {derived_[layer][0], 0};
        case kScoresQ: return {derived_[layer][1], 0};
        case kRowShift: return {derived_[layer][2], 0};
        case kExpOut: return {derived_[layer][3], 0};
        case kDenoms: return {derived_[layer][4], 0};
        case kRecips: return {derived_[layer][5], 0};
        case kWeights: return {derived_[layer][6], 0};
        case kLayerError: return {s_.wire(layer, w), 0};
        default: break;
    }
    if (w < 0 || w >= kWireCount) throw AccelError("unknown GPT-2 wire");
    const size_t width = gpt2_wire_spec(sh, w).count / sh.t;  // row-local: the session's rows from t0 on
    return {s_.wire(layer, w), t0_ * width};
}

// ---- KV-cached decoding --------------------------------------------------------------

Gpt2Decoder::Gpt2Decoder(Gpt2Session& s, size_t max_steps) : s_(s), b_(s.backend()) {
    const Gpt2Shape& sh = s_.shape();
    pos_ = sh.t;
    cap_ = sh.positions;
    gen_max_ = cap_ > pos_ ? cap_ - pos_ : 0;
    if (max_steps && max_steps < gen_max_) gen_max_ = max_steps;
    if (!gen_max_) throw AccelError("no position left to decode after the prefill");
    const size_t d = sh.d, h = sh.heads;
    auto alloc = [&](size_t bytes) {
        const uint64_t id = b_.alloc(std::max<size_t>(bytes, 16));
        owned_.push_back(id);
        return id;
    };
    try {
        Gpt2Shape one = sh;
        one.t = 1;
        for (int w = 0; w < kWireCount; ++w) {
            const WireSpec ws = gpt2_wire_spec(one, w);
            w_[w] = alloc(ws.elem * ws.count);
        }
        // the causal-packed row of one step holds pos + 1 <= cap entries per head
        w_[kScoresAcc] = alloc(8 * h * cap_);
        w_[kScoresQ] = alloc(2 * h * cap_);
        w_[kExpOut] = alloc(2 * h * cap_);
        w_[kWeights] = alloc(2 * h * cap_);
        xalt_ = alloc(2 * d);  // the layer input alternates between kXin and this row
        for (size_t l = 0; l < sh.layers; ++l) {
            kcache_.push_back(alloc(2 * cap_ * d));
            vcache_.push_back(alloc(2 * cap_ * d));
        }
        const size_t fin_elem[6] = {8, 8, 8, 2, 8, 2}, fin_count[6] = {1, 1, 1, 1, d, d};
        for (int k = 0; k < 6; ++k) fin_[k] = alloc(fin_elem[k] * fin_count[k]);
        embed_acc_ = alloc(8 * d);
        tokens_ = alloc(4 * (gen_max_ + 1));
        logits_ = alloc(8 * gen_max_ * sh.vocab);
        err_ = alloc(4);
        // KvCache::from_prefill: the prefill's K/V rows
        const Api& A = b_.api();
        for (size_t l = 0; l < sh.layers; ++l) {
            b_.check(A.volta_cuda_resident_copy_rows(b_.ctx(), s_.wire(l, kK), 0, 2 * sh.t * d, kcache_[l], 0,
                                                      2 * sh.t * d, 1, 2 * sh.t * d),
                     "resident_copy_rows");
            b_.check(A.volta_cuda_resident_copy_rows(b_.ctx(), s_.wire(l, kV), 0, 2 * sh.t * d, vcache_[l], 0,
                                                      2 * sh.t * d, 1, 2 * sh.t * d),
                     "resident_copy_rows");
        }
        b_.check(A.volta_cuda_resident_zero(b_.ctx(), err_, 0, sizeof(uint32_t)), "resident_zero");
    } catch (...) {
        for (uint64_t id : owned_) b_.api().volta_cuda_resident_free(b_.ctx(), id);
        throw;
    }
}

Gpt2Decoder::~Gpt2Decoder() {
    for (uint64_t id : owned_) b_.api().volta_cuda_resident_free(b_.ctx(), id);
}

void Gpt2Decoder::generate(size_t n) {
    if (!b_.ext().argmax_i64) throw AccelError("the CUDA library lacks volta_b200_argmax_i64_device");
    if (done_ + n > gen_max_) throw AccelError("decode would run past the model's positions or the decoder's steps");
    if (done_ == 0)  // token 0: the argmax of the prefill's last-position logits
        b_.check(b_.ext().argmax_i64(b_.ctx(), s_.logits(), 0, s_.shape().vocab, tokens_, 0), "argmax_i64_device");
    for (size_t i = 0; i < n; ++i) step(done_ + i);
    done_ += n;
}

void Gpt2Decoder::step(size_t i) {
    const Api& A = b_.api();
    void* c = b_.ctx();
    const Gpt2Shape& sh = s_.shape();
    const Gpt2Shifts& f = sh.shifts;
    const size_t d = sh.d, h = sh.heads, dff = sh.dff, p = pos_, seq = p + 1;
    const auto& W = w_;
    // decode.rs:137-160: embedding row at position p
    b_.check(A.volta_cuda_fixed_embed_device(c, tokens_, i, s_.wte(), 0, s_.wpe(), 0, embed_acc_, 0, W[kXin], 0, err_,
                                             0, 1, d, sh.vocab, sh.positions, p, f.embed),
             "fixed_embed_device");
    uint64_t x = W[kXin], y = xalt_;  // layer input, then the layer output
    for (size_t l = 0; l < sh.layers; ++l) {
        const uint64_t e = err_;
        auto w = [&](int which) { return s_.weight(l, which); };
        b_.check(A.volta_cuda_fixed_layer_norm_device(c, x, 0, w(4), 0, w(5), 0, s_.lut(0), 0, W[kLn1Mean], 0,
                                                      W[kLn1Var], 0, W[kLn1Rin], 0, W[kLn1Rout], 0, W[kLn1Acc], 0,
                                                      W[kLn1Out], 0, e, 0, 1, d, f.ln_var, f.ln_norm),
                 "fixed_layer_norm_device");
        b_.check(A.volta_cuda_fixed_gemm_device(c, W[kLn1Out], 0, w(0), 0, 0, 0, 0, 0, W[kQkvAcc], 0, W[kQkvQ], 0, 0,
                                                0, e, 0, 1, d, 3 * d, f.qkv),
                 "fixed_gemm_device");
        // the new K/V row goes straight to cache row p (decode.rs:172-176)
        b_.check(A.volta_cuda_fixed_qkv_split_device(c, W[kQkvQ], 0, W[kQ], 0, kcache_[l], p * d, vcache_[l], p * d,
                                                     1, d),
                 "fixed_qkv_split_device");
        b_.check(A.volta_cuda_fixed_attention_scores_device(c, W[kQ], 0, kcache_[l], 0, W[kScoresAcc], 0,
                                                            W[kScoresQ], 0, e, 0, 1, seq, p, h, sh.head_dim,
                                                            f.scores),
                 "fixed_attention_scores_device");
        b_.check(A.volta_cuda_fixed_softmax_device(c, W[kScoresQ], 0, s_.lut(1), 0, s_.lut(2), 0, W[kRowShift], 0,
                                                   W[kExpOut], 0, W[kDenoms], 0, W[kRecips], 0, W[kWeights], 0, e, 0,
                                                   1, seq, p, h, f.recip_den, f.recip_log2, f.softmax_norm,
                                                   f.row_shift ? 1 : 0),
                 "fixed_softmax_device");
        b_.check(A.volta_cuda_fixed_av_device(c, W[kWeights], 0, vcache_[l], 0, W[kAvAcc], 0, W[kAvQ], 0, e, 0, 1,
                                              seq, p, d, h, f.av),
                 "fixed_av_device");
        b_.check(A.volta_cuda_fixed_gemm_device(c, W[kAvQ], 0, w(1), 0, 0, 0, x, 0, W[kProjAcc], 0, W[kProjQ], 0,
                                                W[kAttnOut], 0, e, 0, 1, d, d, f.attn_proj),
                 "fixed_gemm_device");
        b_.check(A.volta_cuda_fixed_layer_norm_device(c, W[kAttnOut], 0, w(6), 0, w(7), 0, s_.lut(0), 0, W[kLn2Mean],
                                                      0, W[kLn2Var], 0, W[kLn2Rin], 0, W[kLn2Rout], 0, W[kLn2Acc], 0,
                                                      W[kLn2Out], 0, e, 0, 1, d, f.ln_var, f.ln_norm),
                 "fixed_layer_norm_device");
        b_.check(A.volta_cuda_fixed_gemm_device(c, W[kLn2Out], 0, w(2), 0, 0, 0, 0, 0, W[kUpAcc], 0, W[kUpQ], 0, 0, 0,
                                                e, 0, 1, d, dff, f.ffn_up),
                 "fixed_gemm_device");
        b_.check(A.volta_cuda_fixed_lookup_device(c, W[kUpQ], 0, s_.lut(3), 0, W[kGelu], 0, dff),
                 "fixed_lookup_device");
        b_.check(A.volta_cuda_fixed_gemm_device(c, W[kGelu], 0, w(3), 0, 0, 0, W[kAttnOut], 0, W[kDownAcc], 0,
                                                W[kDownQ], 0, y, 0, e, 0, 1, dff, d, f.ffn_down),
                 "fixed_gemm_device");
        std::swap(x, y);
    }
    // final LN + logits row (decode.rs:257-268), next token (argmax)
    b_.check(A.volta_cuda_fixed_layer_norm_device(c, x, 0, s_.lnf(0), 0, s_.lnf(1), 0, s_.lut(0), 0, fin_[0], 0,
                                                  fin_[1], 0, fin_[2], 0, fin_[3], 0, fin_[4], 0, fin_[5], 0, err_, 0,
                                                  1, d, f.ln_var, f.ln_norm),
             "fixed_layer_norm_device");
    b_.check(A.volta_cuda_fixed_logits_device(c, fin_[5], 0, s_.wte(), 0, logits_, i * sh.vocab, 1, d, sh.vocab),
             "fixed_logits_device");
    b_.check(b_.ext().argmax_i64(c, logits_, i * sh.vocab, sh.vocab, tokens_, i + 1), "argmax_i64_device");
    ++pos_;
}

}  // namespace vzh
