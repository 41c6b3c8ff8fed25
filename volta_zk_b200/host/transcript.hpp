// Transcript and proof wire format of the blind LogUp argument.
//
//   BLAKE3        third-party crate blake3 1.8.5 (hash and derive-key modes),
//                 restated from the published BLAKE3 specification
//   Transcript    rust/volta-mac/src/transcript.rs: private seeded mode
//                 (challenges from FpStream(seed, u64::MAX), 84-110), the byte
//                 ledger (account, 358-361), canonical moves bound into a
//                 derive-key BLAKE3 hash (append_message 215-233,
//                 append_message_digest 337-360, absorb_public_message 237-250,
//                 challenge requests 362-380, canonical_binding_digest 654-667)
//   wire format   rust/volta-proto/src/model_proof_codec.rs: little-endian
//                 integers, Fp2 as (c0, c1) u64 pairs rejected unless
//                 canonical, u32 collection lengths capped at 1,000,000, Option
//                 as a 0/1 tag byte, fixed arrays without a length, no trailing
//                 bytes (Writer/Reader 65-182, Wire impls 202-320); the blind
//                 LogUp proof structs BlindLayerProof / BlindFracProof /
//                 BlindLogupProof (logup.rs:1852-1875, 3164-3169) in field order
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

#include "accel.hpp"

namespace vzh {

void blake3_hash(const uint8_t* data, size_t len, uint8_t out[32]);
void blake3_derive_key(const char* context, const uint8_t* data, size_t len, uint8_t out[32]);

class Transcript {
   public:
    explicit Transcript(const uint8_t seed[32]);
    // Charge and bind one canonical provider message.
    void append_message(const std::string& label, const uint8_t* msg, size_t len);
    void append_fp2s(const std::string& label, const Fp2* values, size_t n);
    void append_fps(const std::string& label, const uint64_t* values, size_t n);
    // Bind a message by its length and BLAKE3 digest.
    void append_message_digest(const std::string& label, uint64_t logical_bytes, const uint8_t digest[32]);
    // Bind public bytes both roles rebuild (not charged as provider wire).
    void absorb_public_message(const std::string& label, const uint8_t* msg, size_t len);
    Fp2 challenge_fp2();
    uint64_t challenge_fp();
    uint64_t challenge_bits(unsigned width);
    void binding_digest(uint8_t out[32]) const;
    uint64_t bytes_for(const std::string& label) const;
    uint64_t total_bytes() const;
    uint64_t messages() const { return n_messages_; }
    // A copy of the challenge stream at its current position (a schedule
    // drawn from it in advance equals the challenges drawn later).
    FpStream challenge_stream() const { return chal_; }

   private:
    void account(const std::string& label, uint64_t n);
    void event(uint8_t kind, const std::string& label, uint64_t len, const uint8_t* body, size_t body_len);
    FpStream chal_;
    std::vector<uint8_t> moves_;  // the canonical move stream, hashed on demand
    std::map<std::string, uint64_t> ledger_;
    uint64_t n_messages_ = 0;
};

// ---- wire format -------------------------------------------------------------

class WireWriter {
   public:
    void u8(uint8_t v) { b_.push_back(v); }
    void u16(uint16_t v) { le(v, 2); }
    void u32(uint32_t v) { le(v, 4); }
    void u64(uint64_t v) { le(v, 8); }
    void fp2(Fp2 v) {
        u64(v.c0);
        u64(v.c1);
    }
    void len(size_t n);
    const std::vector<uint8_t>& bytes() const { return b_; }

   private:
    void le(uint64_t v, int n) {
        for (int i = 0; i < n; ++i) b_.push_back(static_cast<uint8_t>(v >> (8 * i)));
    }
    std::vector<uint8_t> b_;
};

class WireReader {
   public:
    WireReader(const uint8_t* data, size_t len) : p_(data), n_(len) {}
    uint8_t u8();
    uint16_t u16() { return static_cast<uint16_t>(le(2)); }
    uint32_t u32() { return static_cast<uint32_t>(le(4)); }
    uint64_t u64() { return le(8); }
    Fp2 fp2();
    size_t len();
    void finish() const;

   private:
    uint64_t le(int n);
    const uint8_t* p_;
    size_t n_, off_ = 0;
};

struct BlindLayerProof {
    std::vector<std::array<Fp2, 2>> round_corrs;
    std::array<Fp2, 4> split_corrs;
    std::array<Fp2, 3> z_corrs;
};

struct BlindFracProof {
    std::array<Fp2, 2> root_corrs;
    std::vector<BlindLayerProof> layers;  // no auxiliary part (Option None on the wire)
};

struct BlindLogupProof {
    BlindFracProof lookup, table;
    std::array<Fp2, 4> cross_corrs;
};

std::vector<uint8_t> encode_blind_logup(const BlindLogupProof& p);
BlindLogupProof decode_blind_logup(const uint8_t* data, size_t len);  // throws AccelError

// ---- the blind LogUp prover ----------------------------------------------------

struct BlindLogupResult {
    BlindLogupProof proof;
    Fp2 alpha;
    uint64_t next_domain = 0;  // the correlation-domain cursor after the proof
};

// blind_logup_prove (logup.rs:3184-3225) over resident query / table columns
// of canonical Fp values (f_col: n_f entries, t_col: n_t entries, both powers
// of two) and u32 multiplicities: the clear rounds run as the scheduled
// device driver with the transcript's private challenge stream (alpha, then
// per layer lambda, the round challenges and the split challenge, lookup
// side then table side: the order BlindSink draws them); every message is
// then published as its correction against the mock correlation stream's
// full-field masks x = FpStream(corr_seed, dom | FULL_BIT) (corr.rs:
// 1930-1978), one domain per root / round / split / product group and one
// for the cross corrections (cross_prover, logup.rs:2526-2556), taken from
// the cursor starting at dom_base.  The transcript receives the same moves
// in the same order as the reference's BlindSink.
BlindLogupResult blind_logup_prove(Backend& b, uint64_t f_col, size_t n_f, uint64_t t_col, size_t n_t, uint64_t mult,
                                   const uint8_t corr_seed[32], uint64_t dom_base, Transcript& tx);

}  // namespace vzh
