// Whole-model int16 GPT-2 forward over the resident fixed-point entry points
// (see gpt2.hpp for the reference sources it follows).
#include "gpt2.hpp"

#include "api.hpp"

namespace vzh {

WireSpec gpt2_wire_spec(const Gpt2Shape& s, int wire) {
    const size_t t = s.t, d = s.d, td = t * d, n = s.packed(), ht = s.heads * t;
    switch (wire) {
        case kXin: case kLn1Out: case kQ: case kK: case kV: case kAvQ: case kProjQ: case kAttnOut: case kLn2Out:
        case kDownQ: case kFfnOut:
            return {2, td};
        case kLn1Mean: case kLn1Var: case kLn1Rin: case kLn2Mean: case kLn2Var: case kLn2Rin:
            return {8, t};
        case kLn1Rout: case kLn2Rout:
            return {2, t};
        case kLn1Acc: case kLn2Acc: case kAvAcc: case kProjAcc: case kDownAcc:
            return {8, td};
        case kQkvAcc:
            return {8, 3 * td};
        case kQkvQ:
            return {2, 3 * td};
        case kScoresAcc:
            return {8, n};
        case kScoresQ: case kExpOut: case kWeights:
            return {2, n};
        case kRowShift: case kRecips:
            return {2, ht};
        case kDenoms:
            return {8, ht};
        case kUpAcc:
            return {8, t * s.dff};
        case kUpQ: case kGelu:
            return {2, t * s.dff};
        case kLayerError:
            return {4, 1};
        default:
            throw AccelError("unknown GPT-2 wire");
    }
}

Gpt2Session::Gpt2Session(Backend& b, const Gpt2Shape& shape, const std::vector<Gpt2LayerHost>& layers,
                         const int16_t* wte, const int16_t* wpe, const int16_t* lnf_gain, const int16_t* lnf_bias,
                         const std::array<const int16_t*, 4>& luts, const std::array<size_t, 4>& lut_lens)
    : b_(b), s_(shape), lut_lens_(lut_lens) {
    if (!s_.t || s_.t > s_.positions || layers.size() != s_.layers || s_.heads * s_.head_dim != s_.d)
        throw AccelError("invalid GPT-2 session shape");
    try {
        const size_t d = s_.d, dff = s_.dff;
        auto up = [&](const int16_t* src, size_t count) {
            const uint64_t id = own(b_.alloc(count * sizeof(int16_t)));
            b_.upload(id, 0, src, count * sizeof(int16_t));
            return id;
        };
        const size_t sizes[8] = {d * 3 * d, d * d, d * dff, dff * d, d, d, d, d};
        lw_.resize(s_.layers);
        for (size_t l = 0; l < s_.layers; ++l) {
            const int16_t* src[8] = {layers[l].c_attn, layers[l].attn_proj, layers[l].ffn_up, layers[l].ffn_down,
                                     layers[l].ln1_gain, layers[l].ln1_bias, layers[l].ln2_gain, layers[l].ln2_bias};
            for (int k = 0; k < 8; ++k) lw_[l][k] = up(src[k], sizes[k]);
        }
        wte_ = up(wte, s_.vocab * d);
        wpe_ = up(wpe, s_.positions * d);
        lnf_gain_ = up(lnf_gain, d);
        lnf_bias_ = up(lnf_bias, d);
        for (int k = 0; k < 4; ++k) {
            luts_[k] = up(luts[k], lut_lens[k]);
            luts_host_[k].assign(luts[k], luts[k] + lut_lens[k]);
        }
        tokens_ = own(b_.alloc(s_.t * sizeof(uint32_t)));
        embed_acc_ = own(b_.alloc(s_.t * d * sizeof(int64_t)));
        wires_.resize(s_.layers);
        for (size_t l = 0; l < s_.layers; ++l)
            for (int w = 0; w < kWireCount; ++w) {
                if (w == kXin && l > 0) {  // layer l's input is layer l-1's output
                    wires_[l][w] = wires_[l - 1][kFfnOut];
                    continue;
                }
                const WireSpec ws = gpt2_wire_spec(s_, w);
                wires_[l][w] = own(b_.alloc(ws.elem * ws.count));
            }
        const size_t fin_elem[6] = {8, 8, 8, 2, 8, 2}, fin_count[6] = {1, 1, 1, 1, d, d};
        for (int k = 0; k < 6; ++k) fin_[k] = own(b_.alloc(fin_elem[k] * fin_count[k]));
        logits_ = own(b_.alloc(s_.vocab * sizeof(int64_t)));
        err_ = own(b_.alloc(sizeof(uint32_t)));
    } catch (...) {
        for (uint64_t id : owned_) b_.api().volta_cuda_resident_free(b_.ctx(), id);
        throw;
    }
}

Gpt2Session::~Gpt2Session() {
    for (uint64_t id : owned_) b_.api().volta_cuda_resident_free(b_.ctx(), id);
}

void Gpt2Session::upload_tokens(const uint32_t* tokens) { b_.upload(tokens_, 0, tokens, s_.t * sizeof(uint32_t)); }

void Gpt2Session::forward(uint64_t tokens_id) {
    const Api& A = b_.api();
    void* c = b_.ctx();
    const size_t t = s_.t, d = s_.d, dff = s_.dff, h = s_.heads;
    const Gpt2Shifts& sh = s_.shifts;
    b_.check(A.volta_cuda_resident_zero(c, err_, 0, sizeof(uint32_t)), "resident_zero");
    // x_0 = requant(wte[tok] + wpe[pos], shift_embed) (gpt2_fixed.py:646-670)
    b_.check(A.volta_cuda_fixed_embed_device(c, tokens_id, 0, wte_, 0, wpe_, 0, embed_acc_, 0, wires_[0][kXin], 0,
                                             err_, 0, t, d, s_.vocab, s_.positions, 0, sh.embed),
             "fixed_embed_device");
    for (size_t l = 0; l < s_.layers; ++l) {
        const auto& W = wires_[l];
        const auto& w = lw_[l];
        const uint64_t e = W[kLayerError];
        b_.check(A.volta_cuda_resident_zero(c, e, 0, sizeof(uint32_t)), "resident_zero");
        // LN1 (gpt2_fixed.py:385-425)
        b_.check(A.volta_cuda_fixed_layer_norm_device(c, W[kXin], 0, w[4], 0, w[5], 0, luts_[0], 0, W[kLn1Mean], 0,
                                                      W[kLn1Var], 0, W[kLn1Rin], 0, W[kLn1Rout], 0, W[kLn1Acc], 0,
                                                      W[kLn1Out], 0, e, 0, t, d, sh.ln_var, sh.ln_norm),
                 "fixed_layer_norm_device");
        // fused QKV projection, split into q, k, v
        b_.check(A.volta_cuda_fixed_gemm_device(c, W[kLn1Out], 0, w[0], 0, 0, 0, 0, 0, W[kQkvAcc], 0, W[kQkvQ], 0, 0,
                                                0, e, 0, t, d, 3 * d, sh.qkv),
                 "fixed_gemm_device");
        b_.check(A.volta_cuda_fixed_qkv_split_device(c, W[kQkvQ], 0, W[kQ], 0, W[kK], 0, W[kV], 0, t, d),
                 "fixed_qkv_split_device");
        // causal scores, softmax (exp / recip tables), A.V
        b_.check(A.volta_cuda_fixed_attention_scores_device(c, W[kQ], 0, W[kK], 0, W[kScoresAcc], 0, W[kScoresQ], 0,
                                                            e, 0, t, t, 0, h, s_.head_dim, sh.scores),
                 "fixed_attention_scores_device");
        b_.check(A.volta_cuda_fixed_softmax_device(c, W[kScoresQ], 0, luts_[1], 0, luts_[2], 0, W[kRowShift], 0,
                                                   W[kExpOut], 0, W[kDenoms], 0, W[kRecips], 0, W[kWeights], 0, e, 0,
                                                   t, t, 0, h, sh.recip_den, sh.recip_log2, sh.softmax_norm,
                                                   sh.row_shift ? 1 : 0),
                 "fixed_softmax_device");
        b_.check(A.volta_cuda_fixed_av_device(c, W[kWeights], 0, W[kV], 0, W[kAvAcc], 0, W[kAvQ], 0, e, 0, t, t, 0, d,
                                              h, sh.av),
                 "fixed_av_device");
        // attention projection + residual
        b_.check(A.volta_cuda_fixed_gemm_device(c, W[kAvQ], 0, w[1], 0, 0, 0, W[kXin], 0, W[kProjAcc], 0, W[kProjQ],
                                                0, W[kAttnOut], 0, e, 0, t, d, d, sh.attn_proj),
                 "fixed_gemm_device");
        // LN2, FFN up, GELU, FFN down + residual
        b_.check(A.volta_cuda_fixed_layer_norm_device(c, W[kAttnOut], 0, w[6], 0, w[7], 0, luts_[0], 0, W[kLn2Mean],
                                                      0, W[kLn2Var], 0, W[kLn2Rin], 0, W[kLn2Rout], 0, W[kLn2Acc], 0,
                                                      W[kLn2Out], 0, e, 0, t, d, sh.ln_var, sh.ln_norm),
                 "fixed_layer_norm_device");
        b_.check(A.volta_cuda_fixed_gemm_device(c, W[kLn2Out], 0, w[2], 0, 0, 0, 0, 0, W[kUpAcc], 0, W[kUpQ], 0, 0, 0,
                                                e, 0, t, d, dff, sh.ffn_up),
                 "fixed_gemm_device");
        b_.check(A.volta_cuda_fixed_lookup_device(c, W[kUpQ], 0, luts_[3], 0, W[kGelu], 0, t * dff),
                 "fixed_lookup_device");
        b_.check(A.volta_cuda_fixed_gemm_device(c, W[kGelu], 0, w[3], 0, 0, 0, W[kAttnOut], 0, W[kDownAcc], 0,
                                                W[kDownQ], 0, W[kFfnOut], 0, e, 0, t, dff, d, sh.ffn_down),
                 "fixed_gemm_device");
    }
    // final LN of the last position and its logits against the tied wte
    // (gpt2_fixed.py:673-686)
    const uint64_t last = wires_[s_.layers - 1][kFfnOut];
    b_.check(A.volta_cuda_fixed_layer_norm_device(c, last, (t - 1) * d, lnf_gain_, 0, lnf_bias_, 0, luts_[0], 0,
                                                  fin_[0], 0, fin_[1], 0, fin_[2], 0, fin_[3], 0, fin_[4], 0, fin_[5],
                                                  0, err_, 0, 1, d, sh.ln_var, sh.ln_norm),
             "fixed_layer_norm_device");
    b_.check(A.volta_cuda_fixed_logits_device(c, fin_[5], 0, wte_, 0, logits_, 0, 1, d, s_.vocab),
             "fixed_logits_device");
}

}  // namespace vzh
