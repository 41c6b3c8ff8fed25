// Whole-model int16 fixed-point GPT-2 forward (the witness of a prefill
// proof) over the seam's resident fixed-point entry points, and the per-layer
// proof schedule that consumes it.
//
//   forward   rust/volta-gpt2/src/resident.rs:1106-1300
//             (forward_model_tokens_resident / build_resident_forward),
//             value-for-value the reference NumPy mirror
//             scripts/gpt2_fixed.py:427-645 forward_layer and 688-760
//             forward_model: embed -> L x (LN1, QKV, scores, softmax, A.V,
//             projection + residual, LN2, FFN up, GELU, FFN down + residual)
//             -> final LN of the last position -> logits of that position.
//   model     rust/volta-gpt2/src/model.rs:504-600 synthetic_model is built by
//             the caller; this session only uploads the weights it is given.
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>
#include <map>
#include <memory>
#include <utility>
#include <vector>

#include "accel.hpp"

namespace vzh {

// LutParams defaults (rust/volta-gpt2/src/luts.rs; gpt2_fixed.py:94-110).
struct Gpt2Shifts {
    uint32_t ln_var = 7, ln_norm = 16, recip_den = 6, recip_log2 = 26;
    uint32_t qkv = 10, scores = 10, softmax_norm = 14, av = 12, attn_proj = 10, ffn_up = 10, ffn_down = 10;
    int32_t embed = 0;
    bool row_shift = true;  // P5 stable softmax (luts.rs:57-59); needed past T ~ 300 (u16 recip domain)
};

struct Gpt2Shape {
    size_t layers = 12, d = 768, heads = 12, head_dim = 64, dff = 3072, vocab = 50257, positions = 1024;
    size_t t = 0;  // tokens of the prefill this session proves
    Gpt2Shifts shifts;
    size_t packed() const { return heads * (t * (t + 1) / 2); }  // causal-packed attention entries
};

// Per-layer wires of the forward, kept resident for the proof (arena ids).
enum Gpt2Wire : int {
    kXin = 0, kLn1Mean, kLn1Var, kLn1Rin, kLn1Rout, kLn1Acc, kLn1Out, kQkvAcc, kQkvQ, kQ, kK, kV, kScoresAcc,
    kScoresQ, kRowShift, kExpOut, kDenoms, kRecips, kWeights, kAvAcc, kAvQ, kProjAcc, kProjQ, kAttnOut, kLn2Mean,
    kLn2Var, kLn2Rin, kLn2Rout, kLn2Acc, kLn2Out, kUpAcc, kUpQ, kGelu, kDownAcc, kDownQ, kFfnOut, kLayerError,
    kWireCount
};

// Element size and count of one wire at this shape.
struct WireSpec {
    size_t elem, count;
};
WireSpec gpt2_wire_spec(const Gpt2Shape& s, int wire);

// The weights of one layer, host side, row-major (k x n for GEMM weights).
struct Gpt2LayerHost {
    const int16_t *c_attn, *attn_proj, *ffn_up, *ffn_down, *ln1_gain, *ln1_bias, *ln2_gain, *ln2_bias;
};

class Gpt2Session {
   public:
    // Uploads every weight and the four int16 lookup tables (ln_rsqrt, exp,
    // softmax_recip, gelu; lengths in lut_lens) once, and allocates every
    // wire for `shape.t` tokens.
    Gpt2Session(Backend& b, const Gpt2Shape& shape, const std::vector<Gpt2LayerHost>& layers, const int16_t* wte,
                const int16_t* wpe, const int16_t* lnf_gain, const int16_t* lnf_bias,
                const std::array<const int16_t*, 4>& luts, const std::array<size_t, 4>& lut_lens);
    ~Gpt2Session();
    Gpt2Session(const Gpt2Session&) = delete;
    Gpt2Session& operator=(const Gpt2Session&) = delete;

    // Enqueue the whole forward for the resident token ids (u32, t entries):
    // every wire of every layer, the final LN of the last row and its logits.
    // Nothing is downloaded and nothing waits on the device.
    void forward(uint64_t tokens_id);
    // Upload t token ids from host memory into the session's token buffer.
    void upload_tokens(const uint32_t* tokens);
    uint64_t tokens_id() const { return tokens_; }

    const Gpt2Shape& shape() const { return s_; }
    Backend& backend() { return b_; }
    uint64_t wire(size_t layer, int w) const { return wires_[layer][w]; }
    uint64_t weight(size_t layer, int which) const { return lw_[layer][which]; }  // 0..7 as in Gpt2LayerHost
    uint64_t embed_acc() const { return embed_acc_; }
    uint64_t final_ln(int which) const { return fin_[which]; }  // 0 mean 1 var 2 rin 3 rout 4 acc 5 out
    uint64_t logits() const { return logits_; }
    uint64_t error_word() const { return err_; }  // sticky u32 of the embed, final LN and every layer
    uint64_t lut(int which) const { return luts_[which]; }
    size_t lut_len(int which) const { return lut_lens_[which]; }
    const std::vector<int16_t>& lut_host(int which) const { return luts_host_[which]; }
    uint64_t wte() const { return wte_; }
    uint64_t wpe() const { return wpe_; }
    uint64_t lnf(int which) const { return which ? lnf_bias_ : lnf_gain_; }

   private:
    Backend& b_;
    Gpt2Shape s_;
    std::vector<std::array<uint64_t, 8>> lw_;
    std::vector<std::array<uint64_t, kWireCount>> wires_;
    uint64_t wte_ = 0, wpe_ = 0, lnf_gain_ = 0, lnf_bias_ = 0, tokens_ = 0, embed_acc_ = 0, logits_ = 0, err_ = 0;
    std::array<uint64_t, 6> fin_{};
    std::array<uint64_t, 4> luts_{};
    std::array<size_t, 4> lut_lens_{};
    std::array<std::vector<int16_t>, 4> luts_host_;
    std::vector<uint64_t> owned_;
    uint64_t own(uint64_t id) {
        owned_.push_back(id);
        return id;
    }
};

// ---- decode bands and KV-cached decoding (gpt2_decode.cpp) ------------------

// The band witness of rows t0 .. t-1 of the session's last forward
// (rust/volta-gpt2/src/band.rs:77-196, resident.rs:335-455 and 941-1030):
// row-local wires are the session's rows from t0 on; the causal-packed
// per-head wires (scores, exp, weights) are compacted to the band packing
// (head h: rows t0 .. t-1, windows t0 + i + 1) and the per-head row tables
// (row shift, denominators, reciprocals) cut to h x q; the final LayerNorm
// runs over every band row of the last layer's output and the logits over
// every band row (each decode position's sampled token is checkable).
class Gpt2Band {
   public:
    Gpt2Band(Gpt2Session& s, size_t t0);
    ~Gpt2Band();
    Gpt2Band(const Gpt2Band&) = delete;
    Gpt2Band& operator=(const Gpt2Band&) = delete;
    // Enqueue the compaction, the final LN and the logits (no wait).
    void build();
    size_t t0() const { return t0_; }
    size_t q() const { return q_; }
    const Gpt2Session& session() const { return s_; }
    // Buffer and element offset of a band wire of `layer` (Gpt2Wire).
    std::pair<uint64_t, size_t> wire(size_t layer, int w) const;
    uint64_t final_ln(int which) const { return fin_[which]; }  // 0 mean 1 var 2 rin 3 rout 4 acc 5 out
    uint64_t logits() const { return logits_; }                  // q x vocab i64
    uint64_t error_word() const { return err_; }

   private:
    Gpt2Session& s_;
    size_t t0_, q_;
    std::vector<std::array<uint64_t, 7>> derived_;  // scores_acc, scores_q, row_shift, exp, denoms, recips, weights
    std::array<uint64_t, 6> fin_{};
    uint64_t logits_ = 0, err_ = 0;
    std::vector<uint64_t> owned_;
};

// KV-cached greedy decoding (rust/volta-gpt2/src/decode.rs:80-300): caches
// seeded with the session's K/V rows of its t tokens (KvCache::from_prefill),
// then one row per step at position pos: embed, every layer on the new row
// with attention over cache rows 0 .. pos (the new K/V row appended first),
// final LN, the logits row, and the next token as the argmax of that row (the
// last of equal maxima), kept on the device for the next step's embed.
class Gpt2Decoder {
   public:
    // max_steps: the most steps this decoder will run (0: every position left)
    Gpt2Decoder(Gpt2Session& s, size_t max_steps);
    ~Gpt2Decoder();
    Gpt2Decoder(const Gpt2Decoder&) = delete;
    Gpt2Decoder& operator=(const Gpt2Decoder&) = delete;
    // Enqueue n greedy steps; the first token is the argmax of the session's
    // last-position logits.  Step i writes its token to tokens()[i] and its
    // logits row to logits() row i.  Throws when the positions run out.
    void generate(size_t n);
    size_t position() const { return pos_; }
    uint64_t tokens() const { return tokens_; }  // u32, one per generated token
    uint64_t logits() const { return logits_; }  // i64, n_max x vocab
    uint64_t cache(size_t layer, int kv) const {
        return layer >= kcache_.size() ? 0 : (kv ? vcache_[layer] : kcache_[layer]);
    }
    uint64_t error_word() const { return err_; }
    size_t capacity() const { return cap_; }

   private:
    void step(size_t i);
    Gpt2Session& s_;
    Backend& b_;
    size_t pos_ = 0, cap_ = 0, gen_max_ = 0, done_ = 0;
    std::vector<uint64_t> kcache_, vcache_;
    uint64_t xalt_ = 0;  // second layer-input row (inputs and outputs alternate)
    std::array<uint64_t, kWireCount> w_{};  // one-row wires of the current step
    std::array<uint64_t, 6> fin_{};
    uint64_t tokens_ = 0, logits_ = 0, embed_acc_ = 0, err_ = 0;
    std::vector<uint64_t> owned_;
};

// ---- the prefill proof schedule (gpt2_proof.cpp) -----------------------------

// Sub-proof sites of one layer, in proof order; each draws from its own
// private transcript FpStream(seed, gpt2_site_domain(layer, site, chunk)),
// chunk 0 for the prefill and c >= 1 for the c-th decode band of a response.
enum Gpt2Site : int {
    kSiteDownRange = 1, kSiteGelu, kSiteUpRange, kSiteLn2Norm, kSiteLn2Rsqrt, kSiteProjRange, kSiteAvRange,
    kSiteNormRange, kSiteExp, kSiteRecip, kSiteScoresRange, kSiteQkvRange, kSiteLn1Norm, kSiteLn1Rsqrt,
    kSiteGemmDown = 16, kSiteGemmUp, kSiteLn2Had, kSiteGemmProj, kSiteAv, kSiteNormHad, kSiteQk, kSiteGemmQkv,
    kSiteLn1Had
};
uint64_t gpt2_site_domain(size_t layer, int site, size_t chunk = 0);
// Site 0 of a unit's mask: the layer's VOLE-MAC boundary corrections.
constexpr int kSiteCorrections = 0;
constexpr uint32_t kGpt2AllSites = 0x1FF7FFFu;  // bits 0 .. 14 and 16 .. 24

// A unit of proof work: the sites (bit k = site k) of one layer.  The sites of
// a layer are independent sub-proofs over the same witness, so a proof can be
// split over GPUs by units as well as by layers.
struct Gpt2Unit {
    size_t layer;
    uint32_t sites;
};

struct Gpt2Proof {
    std::vector<std::vector<Fp2>> layer_words;  // per proved unit (layer), its sites' words in site order
    std::vector<std::vector<std::pair<int, size_t>>> unit_sites;  // per unit: (site, words) in order
    uint8_t pcs_root[32] = {0};
};

struct Owned;
struct PendingLogup;

class Gpt2Prover {
   public:
    // Ligero shape of the weight commitment (GPT2_FULL, ligero.rs:59-60).
    // kPcsRows is the row count while the weights fit (GPT-2 small); larger
    // models take the power of two their weights fill (the MLE row
    // variables are ceil(log2 rows) either way, ligero.rs:47-50, 66-68).
    static constexpr size_t kPcsRows = 8192, kPcsColBits = 14, kPcsPad = 512, kPcsCodeBits = 15;
    static size_t pcs_rows_for(size_t weights) {
        const size_t need = (weights + (size_t{1} << kPcsColBits) - 1) >> kPcsColBits;
        size_t rows = kPcsRows;
        while (rows < need) rows <<= 1;
        return rows;
    }
    size_t pcs_rows() const { return pcs_rows_; }

    // Builds the lookup tables and the committed weight matrix once.
    explicit Gpt2Prover(Gpt2Session& s);
    ~Gpt2Prover();
    Gpt2Prover(const Gpt2Prover&) = delete;
    Gpt2Prover& operator=(const Gpt2Prover&) = delete;

    // Prove the witness of the session's last forward.  seed: the
    // sub-proofs' transcripts; mac_seed: the VOLE-MAC mask stream; pad_seed:
    // the PCS row pads.  The boundary corrections stay resident
    // (correction()).
    Gpt2Proof prove(const uint8_t seed[32], const uint8_t mac_seed[32], const uint8_t pad_seed[32]);
    // The same for layers first, first + stride, ... only (one GPU's share
    // of a proof split by layers; the sub-proofs of different layers are
    // independent), with the weight commitment when with_pcs.
    Gpt2Proof prove_layers(const uint8_t seed[32], const uint8_t mac_seed[32], const uint8_t pad_seed[32],
                           size_t first, size_t stride, bool with_pcs);
    // Prove a decode band of the same session (rust/volta-proto/src/
    // block_proof.rs:10112-10125 prove_layer_phase1_band; model_proof.rs:2710
    // prove_response's deferred chunks): the layer schedule over the band's q
    // rows, with the attention sites over q_pad x s_pad rectangles (s = t0 + q
    // keys, the session's K/V rows 0 .. s - 1: the earlier rows are the cache
    // segments, the band's own rows its new ones).  `band` must be built from
    // this prover's session; chunk >= 1 separates the band's transcripts and
    // mask domains from the prefill's and from other chunks'.  No weight
    // commitment (one per response, with the prefill).
    Gpt2Proof prove_band(const Gpt2Band& band, size_t chunk, const uint8_t seed[32], const uint8_t mac_seed[32],
                         size_t first, size_t stride);
    // The given units only, in the given order (one GPU's share of a proof
    // split by sites), with the weight commitment when with_pcs.
    Gpt2Proof prove_units(const uint8_t seed[32], const uint8_t mac_seed[32], const uint8_t pad_seed[32],
                          const std::vector<Gpt2Unit>& units, bool with_pcs);
    // One GPU's row block of the weight commitment, for a commitment split
    // by rows over GPUs (ligero.rs commit_impl rows are independent until
    // the column hash): the pads, messages and RS code of rows row0 ..
    // row0 + rows - 1, then each code column's BLAKE3 chaining value over
    // those rows (chunk counters from row0 / 128).  rows = 128 * 2^k and
    // row0 a multiple of rows.  Writes code_len x 32 bytes to cvs (host).
    void commit_rows(const uint8_t pad_seed[32], size_t row0, size_t rows, uint8_t* cvs);
    // Host destination of the boundary corrections (nullptr: none): wire w
    // of layer l goes to host + (l * 5 + w) * rows * d (rows: the proof's t
    // or the band's q), copied asynchronously while the later layers
    // compute; every copy has landed when the proof call returns.  Pinned
    // memory makes the copies overlap; host must hold layers * 5 * rows * d.
    void set_correction_sink(uint64_t* host) { sink_ = host; }
    // Corrections x - mask of boundary wire w (0 x_in, 1 k, 2 v, 3
    // attn_block_out, 4 ffn_block_out) of layer l: rows x d u64 (the last
    // proof's rows: t, or the band's q).
    uint64_t correction(size_t layer, int w) const { return corrections_.at(layer).at(w); }
    // Host wall time of the last proof: enqueueing every launch, and in all
    // (the enqueue, then the downloads that wait for the device).
    double host_enqueue_ms() const { return host_enqueue_ms_; }
    double host_total_ms() const { return host_total_ms_; }

   private:
    struct Slot {
        PendingLogup* logup = nullptr;  // a LogUp instance, else `words` message slots at msgs
        int site = 0;
        uint64_t msgs = 0;
        size_t words = 0;
        size_t at = 0;  // offset of its raw messages in the layer's buffer
    };
    std::vector<Slot> enqueue_layer(size_t l, Owned& own, const uint8_t seed[32], const uint8_t mac_seed[32],
                                    const Gpt2Band* band, size_t chunk, uint32_t mask);
    Gpt2Proof run(const uint8_t seed[32], const uint8_t mac_seed[32], const uint8_t pad_seed[32],
                  const std::vector<Gpt2Unit>& units, bool with_pcs, const Gpt2Band* band, size_t chunk);

    Gpt2Session& s_;
    Backend& b_;
    std::map<uint32_t, uint64_t> range_;
    double host_enqueue_ms_ = 0, host_total_ms_ = 0;
    uint64_t gelu_pairs_ = 0, rsqrt_pairs_ = 0, expgap_pairs_ = 0, recip_pairs_ = 0, shifts_ = 0;
    uint64_t exp_pad_out_ = 0, recip_pad_out_ = 0;
    uint64_t wmat_ = 0, pads_ = 0, code_ = 0, tree_ = 0, err_ = 0, cvs_ = 0;
    size_t pcs_rows_ = kPcsRows;
    uint64_t* sink_ = nullptr;
    std::vector<uint64_t> owned_;
    std::map<size_t, std::vector<uint64_t>> corrections_;  // per proved layer
    std::vector<std::vector<std::unique_ptr<PendingLogup>>> pending_logups_;
    uint64_t own(uint64_t id) {
        owned_.push_back(id);
        return id;
    }
};

}  // namespace vzh
