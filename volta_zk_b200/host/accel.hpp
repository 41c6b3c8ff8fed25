// Host side above the C ABI: a C++ restatement of the reference's Rust seam
// `volta_accel::Backend` for the resident CUDA backend and of the protocol
// callers on the hot path.
//
//   loader         rust/volta-accel/src/cuda.rs:1119-1420 (dlopen of
//                  $VOLTA_CUDA_LIBRARY or the in-package library, ABI version
//                  check, eager resolution of all 124 symbols)
//   Backend        rust/volta-accel/src/lib.rs:986-1640 (cuda_resident with a
//                  timing policy, typed device buffers, segment downloads)
//   FpStream       rust/volta-field/src/lib.rs:222-268
//   Transcript     rust/volta-mac/src/transcript.rs:84-103, 563-590 (private
//                  challenge mode: FpStream(seed, u64::MAX))
//
// Errors are reported as AccelError exceptions carrying the backend's
// last_error text; nothing falls back to the CPU.
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#ifndef __CUDACC__
#define __host__
#define __device__
#define __forceinline__ inline
#endif
#include "../csrc/field.cuh"

namespace vzh {

using vzb::Fp2;

struct AccelError : std::runtime_error {
    explicit AccelError(const std::string& m) : std::runtime_error(m) {}
};

// ---- host FpStream (ChaCha8Rng, rand_chacha 0.3.1 layout) ----------------
class FpStream {
   public:
    FpStream(const uint8_t seed[32], uint64_t domain);
    uint64_t next_u64();
    uint64_t next_fp();
    Fp2 next_fp2() {
        const uint64_t a = next_fp();
        const uint64_t b = next_fp();
        return Fp2{a, b};
    }
    uint64_t next_bits(unsigned width) {
        const uint64_t raw = next_u64();
        return width >= 64 ? raw : raw & ((uint64_t{1} << width) - 1);
    }

   private:
    uint32_t key_[8];
    uint64_t stream_, counter_ = 0;
    uint32_t words_[16];
    unsigned idx_ = 8;
};

// ---- the loaded C ABI ------------------------------------------------------
struct Api;     // function table, defined in api.hpp
struct ExtApi;  // optional extensions, defined in api.hpp

enum class TimingPolicy { DeferredEvents = 0, WallOnlyCounters = 1 };

enum Operation : int { kGemm = 0, kLogup = 1, kPcsRows = 2, kPcsNtt = 3, kPcsMerkle = 4,
                       kAuthMasks = 5, kMailbox = 6 };

class Backend {
   public:
    // Load the library (path, else $VOLTA_CUDA_LIBRARY, else the in-package
    // libvolta_cuda_backend.so) and create a resident context.
    explicit Backend(const std::string& library, TimingPolicy policy);
    ~Backend();
    Backend(const Backend&) = delete;
    Backend& operator=(const Backend&) = delete;

    const Api& api() const { return *api_; }
    const ExtApi& ext() const { return *ext_; }
    // Use the fused fold + round extensions when the library has them.
    void set_fused(bool on);
    // Scheduled drivers: draw every challenge first, enqueue all rounds with
    // device-side message slots and download the messages once (valid for
    // the clear / private-transcript sinks, whose challenges do not depend on
    // the messages).  Off: the reference's round-by-round call sequence.
    void set_scheduled(bool on) { scheduled_ = on; }
    bool scheduled() const { return scheduled_; }
    // Scheduled LogUp sides: run the round steps of all large layers as
    // cross-layer batches (volta_b200_logup_round_batch_device) when the
    // library has it.  Off: layer after layer.
    void set_batched(bool on) { batched_ = on; }
    bool batched() const { return batched_; }
    void* ctx() const { return ctx_; }
    [[noreturn]] void raise(const char* what) const;
    void check(int rc, const char* what) const {
        if (rc != 0) raise(what);
    }

    // typed device buffers: id + element count
    uint64_t alloc(size_t bytes);
    void free(uint64_t id);
    void upload(uint64_t id, size_t offset_bytes, const void* src, size_t bytes);
    void download(uint64_t id, size_t offset_bytes, void* dst, size_t bytes);
    // one mailbox download of several Fp2 slices (lib.rs:1523-1577)
    std::vector<Fp2> download_fp2_segments(const std::vector<std::pair<uint64_t, size_t>>& elems);

    vz_raw_stats stats();
    void reset_stats();

   private:
    void* handle_ = nullptr;
    Api* api_ = nullptr;
    ExtApi* ext_ = nullptr;
    ExtApi* ext_loaded_ = nullptr;
    bool scheduled_ = false;
    bool batched_ = true;
    void* ctx_ = nullptr;
};

// ---- protocol drivers (resident) -------------------------------------------

// Triple-product sumcheck over three device tables of n = 2^k Fp2 entries
// (hadamard.rs:186-260 device calls, clear messages).  The input buffers are
// not modified.  Returns 3*k round messages and the three final openings.
struct TripleResult {
    std::vector<Fp2> messages;
    Fp2 finals[3];
};
TripleResult triple_sumcheck_resident(Backend& b, uint64_t a, uint64_t bb, uint64_t c, size_t n,
                                      FpStream& tx);
// The same sumcheck on three device columns of n canonical Fp values (Fp2
// tables with c1 = 0).  The scheduled driver runs rounds 0 and 1 on the base
// columns (volta_b200_triple_*_fp extensions); otherwise the columns are
// lifted to Fp2 (base_broadcast_fp2_device) and proved as above.  Same result.
//
// With `host` set, the three device columns are still to be filled from host
// memory (pinned for the transfer to overlap): the scheduled driver uploads
// them chunk by chunk on the context's copy stream (volta_b200_upload_async)
// and, where the on-chip rounds apply (n >= 8192), proves each chunk's tiles
// as soon as that chunk has landed, so the first 13 rounds run under the
// transfer; otherwise everything lands before the first round.
struct HostColumns {
    const uint64_t* col[3] = {nullptr, nullptr, nullptr};
    size_t chunk = 0;  // entries per column and upload chunk (0: 2^21)
};
TripleResult triple_sumcheck_resident_fp(Backend& b, uint64_t a, uint64_t bb, uint64_t c, size_t n,
                                         FpStream& tx, const HostColumns* host = nullptr);

// LogUp (logup.rs:1760-1771, resident engine 995-1470): queries and table are
// device columns of canonical Fp values (n_f and n_t entries, powers of two),
// mult a device u32 column of n_t multiplicities.  Appends the flat proof
// (alpha, per side root_p, root_q, per layer rounds (h0, h2) and splits).
std::vector<Fp2> logup_prove_resident(Backend& b, uint64_t f_col, size_t n_f, uint64_t t_col,
                                      size_t n_t, uint64_t mult, FpStream& chal);

// Completion of a proof sharded over G = 2^s shards (sharded.cpp): `parts`
// holds every shard's local output in shard order (triple: the messages of
// its own rounds then its 3 final values; LogUp: vzh_logup_local's words).
// The challenges are redrawn from the stream; the result equals the
// one-device proof.
TripleResult triple_finish(const Fp2* parts, size_t shards, size_t n, FpStream& tx);
std::vector<Fp2> logup_finish(const Fp2* parts, size_t shards, size_t words_per_shard, size_t n_f, size_t n_t,
                              FpStream& chal);

// Ligero commitment of `rows` seeded Fp message rows (FpStream(row_seed, r),
// msg_len words each) zero-padded to code_len, and `queries` column openings
// at challenge_fp2().c0 mod code_len drawn from `tx` (ligero.rs:465-505,
// 1440-1480).  Columns are query-major (queries x rows); paths hold
// log2(code_len) sibling hashes per query, leaf level first.
struct LigeroOpening {
    uint8_t root[32];
    std::vector<uint32_t> indices;
    std::vector<uint64_t> columns;
    std::vector<uint8_t> paths;
};
LigeroOpening ligero_commit_open_resident(Backend& b, const uint8_t row_seed[32], size_t rows, size_t msg_len,
                                          size_t code_len, size_t queries, FpStream& tx);

// Weight-matrix commitment and its zero-knowledge multi-claim opening, device
// part (rust/volta-pcs/src/ligero.rs:465-505 finish_resident_commit,
// 1187-1480 open_multi_zk_resident).  The matrix is rows x 2^col_bits int16
// weights; each row is (weights mod p || pad ChaCha8 words from
// FpStream(pad_seed, r)) zero-padded to 2^code_bits, RS-encoded by the batched
// NTT and committed by the BLAKE3 column tree.  The opening draws claims + 1
// prover-secret Fp2 mask rows (FpStream(mask_seed, g), msg_len words, padded),
// encodes and commits them, forms u_c = sum_r c^r row_r + mask_0 (proximity)
// and, per claim g, u_g = sum_r eq(point[col_bits..], r - row0) row_r +
// mask_{g+1} and s_g = <mask_{g+1}[0 .. cols), eq(point[.. col_bits])>, then
// gathers the queried data and mask columns with their Merkle paths.  The
// transcript values (c, the query indices) come from the caller, and the
// VOLE-MAC bookkeeping on s_g (corrections, zero batch) stays with the
// caller's correlation stream: it is O(claims) host work.
struct LigeroShape {
    size_t rows = 0, col_bits = 0, pad = 0, code_bits = 0;
    size_t cols() const { return size_t{1} << col_bits; }
    size_t msg_len() const { return cols() + pad; }
    size_t code_len() const { return size_t{1} << code_bits; }
};
struct ZkClaim {
    size_t offset = 0;        // first coefficient of the claimed block (aligned to its size)
    std::vector<Fp2> point;   // LSB-first: col_bits column coordinates, then row coordinates
};
struct LigeroZkOpening {
    uint8_t root[32];
    uint8_t mask_root[32];
    std::vector<Fp2> u_c;               // msg_len
    std::vector<Fp2> u_g;               // claims x msg_len
    std::vector<Fp2> s;                 // claims
    std::vector<uint64_t> columns;      // queries x rows
    std::vector<Fp2> mask_columns;      // queries x (claims + 1)
    std::vector<uint8_t> paths, mask_paths;  // queries x code_bits x 32
};
LigeroZkOpening ligero_commit_open_zk(Backend& b, const int16_t* weights, const LigeroShape& shape,
                                      const uint8_t pad_seed[32], const std::vector<ZkClaim>& claims,
                                      const uint8_t mask_seed[32], Fp2 c, const std::vector<uint32_t>& indices,
                                      double phase_ms[2] = nullptr);

}  // namespace vzh
