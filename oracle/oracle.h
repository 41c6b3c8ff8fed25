/*
 * CPU oracle for the VOLTA-ZK prover hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library links or calls
 * this code; it is the checker that the CUDA backend is compared against in
 * tests/, in __graft_entry__.smoke() and in the cpu_baseline leg of bench.py.
 *
 * Every function restates the reference's CPU semantics (okrame/volta-zk,
 * Rust crates) and cites the file:line it follows.  Parity is pinned by the
 * reference's own published golden vectors (tests/test_oracle_golden.py).
 */
#ifndef VOLTA_ORACLE_H
#define VOLTA_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    uint64_t c0, c1;
} ofp2;

/* ---- Goldilocks / Fp2 (rust/volta-field/src/lib.rs:10-210) ---- */
uint64_t or_fp_add(uint64_t a, uint64_t b);
uint64_t or_fp_sub(uint64_t a, uint64_t b);
uint64_t or_fp_mul(uint64_t a, uint64_t b);
uint64_t or_fp_pow(uint64_t a, uint64_t e);
uint64_t or_fp_inv(uint64_t a);
ofp2 or_fp2_add(ofp2 a, ofp2 b);
ofp2 or_fp2_sub(ofp2 a, ofp2 b);
ofp2 or_fp2_mul(ofp2 a, ofp2 b);
ofp2 or_fp2_inv(ofp2 a);
void or_fp_mul_batch(const uint64_t* a, const uint64_t* b, uint64_t* out, size_t n);

/* ---- FpStream = rand_chacha 0.3.1 ChaCha8Rng (rust/volta-field/src/lib.rs:222-268) ---- */
typedef struct {
    uint32_t key[8];
    uint64_t stream;
    uint64_t block;
    uint32_t words[16];
    uint32_t idx; /* next u64 index in words (0..8) */
} or_stream;

void or_stream_init(or_stream* s, const uint8_t seed[32], uint64_t domain);
uint64_t or_stream_next_u64(or_stream* s);
uint64_t or_stream_next_fp(or_stream* s);
ofp2 or_stream_next_fp2(or_stream* s);
uint64_t or_stream_next_bits(or_stream* s, unsigned width);
void or_stream_fill_u64(const uint8_t seed[32], uint64_t domain, size_t n, uint64_t* out);
/* rows x count Fp, row r from FpStream(seed, base+r) */
void or_chacha_fp_rows(const uint8_t seed[32], uint64_t base, size_t rows, size_t count,
                       uint64_t* out);
/* rows x padded Fp2, first count from next_fp2, rest zero */
void or_chacha_fp2_rows_padded(const uint8_t seed[32], uint64_t base, size_t rows,
                               size_t count, size_t padded, ofp2* out);

/* ---- sumcheck primitives ---- */
void or_product_round(const ofp2* a, const ofp2* b, size_t pairs, ofp2 out[2]);
void or_triple_product_round(const ofp2* a, const ofp2* b, const ofp2* c, size_t pairs,
                             ofp2 out[3]);
void or_logup_general_round(const ofp2* p0, const ofp2* p1, const ofp2* q0, const ofp2* q1,
                            const ofp2* suffix, size_t pairs, ofp2 out[4]);
void or_fold_rows(const ofp2* in, size_t rows, size_t len, ofp2 r, ofp2* out);
void or_logup_tree(const uint64_t* leaf, const uint32_t* mult, size_t n, uint64_t alpha1,
                   int neg_mult, ofp2* p, ofp2* q);
void or_materialize_leaves(const uint64_t* leaf, const uint32_t* mult, size_t n,
                           uint64_t alpha1, int neg_mult, ofp2* p, ofp2* q);
void or_suffix_eq(const ofp2* point, size_t len, ofp2* out);
void or_eq_rows(const ofp2* points, size_t rows, size_t dims, ofp2* out);
void or_eq_vec(const ofp2* point, size_t len, ofp2* out);
void or_aux_round(const ofp2* q0, const ofp2* q1, const ofp2* suffix, const ofp2* columns,
                  const ofp2* eq_rows, const uint32_t* claim_cols, const ofp2* weights,
                  size_t column_count, size_t claim_count, size_t vector_len, ofp2 lambda,
                  ofp2 cpref, ofp2 point, ofp2 out[3]);
void or_matrix_fold(const void* input, const ofp2* weights, size_t rows, size_t stride,
                    size_t column_offset, size_t cols, size_t out_pad, int kind, int axis,
                    ofp2* out);

/* Full protocol drivers (clear sinks).  Messages are written flat. */
/* Triple-product sumcheck (hadamard.rs:186-260, clear variant):
 * rounds*3 messages, challenges from FpStream(chal_seed, u64::MAX).next_fp2()
 * after each message; returns the three final openings in finals[3]. */
void or_triple_sumcheck(ofp2* a, ofp2* b, ofp2* c, size_t n, const uint8_t chal_seed[32],
                        ofp2* messages, ofp2* finals);
/* logup_prove (logup.rs:1760-1771) over i16 queries/table; writes the
 * proof in a flat layout: alpha, then per side root_p, root_q, then per layer
 * [rounds x (h0,h2)], p0,p1,q0,q1.  Returns number of Fp2 written. */
size_t or_logup_prove_fp(const uint64_t* f, size_t n_f, const uint64_t* table, size_t n_t,
                         const uint32_t* mult, const uint8_t chal_seed[32], uint64_t chal_domain,
                         ofp2* out, size_t out_cap);
size_t or_logup_prove(const int16_t* f, size_t n_f, const int16_t* table, size_t n_t,
                      const uint32_t* mult, const uint8_t chal_seed[32], uint64_t chal_domain,
                      ofp2* out, size_t out_cap);

/* ---- NTT (rust/volta-pcs/src/ntt.rs:9-70) ---- */
void or_ntt_batch(const uint64_t* in, size_t rows, size_t msg_len, size_t n, uint64_t* out);
void or_ntt_fp2_batch(const ofp2* in, size_t rows, size_t msg_len, size_t n, ofp2* out);

/* ---- BLAKE3 (third-party blake3 1.8.5, restated from the published spec) ---- */
void or_blake3(const uint8_t* data, size_t len, uint8_t out[32]);
void or_blake3_derive_key(const uint8_t* context, size_t context_len, const uint8_t* data, size_t len,
                          uint8_t out[32]);
/* Column leaves (ligero.rs:351-359, 595-616) and merkle levels (merkle.rs:27-36) */
void or_hash_fp_columns(const uint64_t* m, size_t rows, size_t cols, uint8_t* leaves);
void or_hash_fp2_columns(const ofp2* m, size_t rows, size_t cols, uint8_t* leaves);
void or_merkle_tree(const uint8_t* leaves, size_t n, uint8_t* tree); /* (2n-1)*32 bytes */
void or_merkle_paths(const uint8_t* tree, size_t leaves, const uint32_t* idx, size_t q,
                     uint8_t* paths);

/* ---- PCS rows ---- */
void or_pcs_messages(const int16_t* w, const uint64_t* pads, size_t rows, size_t cols,
                     size_t pad, size_t code_len, uint64_t* out);
void or_pcs_combine_rows(const int16_t* w, const uint64_t* pads, const ofp2* coeffs,
                         size_t rows, size_t cols, size_t pad, size_t combos, ofp2* out);

/* ---- GEMM + requant + MAC corrections (rust/volta-gpt2/src/gemm.rs:19-154) ---- */
void or_gemm_i64(const int16_t* a, const int16_t* b, int64_t* out, size_t m, size_t k,
                 size_t n);
void or_gemm_requant_auth(const int16_t* a, const int16_t* b, const uint64_t* masks,
                          int16_t* out, uint64_t* corr, size_t m, size_t k, size_t n,
                          uint32_t shift);

/* ---- FNV-1a style checksums used by the reference p7 recipes ---- */
uint64_t or_fnv_u64(uint64_t h, const uint64_t* v, size_t n);
void or_set_threads(int n);
int or_max_threads(void);

/* ---- int16 fixed-point forward primitives (fixed.c; backend.cu:1442-1740) ---- */
void or_fixed_embed(const uint32_t* tokens, const int16_t* wte, const int16_t* wpe, int64_t* acc_out,
                    int16_t* out, uint32_t* err, size_t rows, size_t d, size_t vocab, size_t positions,
                    size_t pos0, int32_t shift);
void or_fixed_layer_norm(const int16_t* input, const int16_t* gain, const int16_t* bias, const int16_t* lut,
                         int64_t* means, int64_t* vars, int64_t* rin, int16_t* rout, int64_t* accs, int16_t* outs,
                         uint32_t* err, size_t rows, size_t d, uint32_t var_shift, uint32_t norm_shift);
void or_fixed_gemm(const int16_t* input, const int16_t* w, const int16_t* bias, const int16_t* residual,
                   int64_t* accs, int16_t* req, int16_t* res_out, uint32_t* err, size_t m, size_t k, size_t n,
                   uint32_t shift);
void or_fixed_qkv_split(const int16_t* qkv, int16_t* q, int16_t* k, int16_t* v, size_t rows, size_t d);
void or_fixed_attention_scores(const int16_t* q, const int16_t* k, int64_t* accs, int16_t* outs, uint32_t* err,
                               size_t rows, size_t seq, size_t pos0, size_t heads, size_t head_dim,
                               uint32_t shift);
void or_fixed_softmax(const int16_t* scores, const int16_t* exp_lut, const int16_t* recip_lut, int16_t* row_shifts,
                      int16_t* exp_out, int64_t* denoms, int16_t* recips, int16_t* weights, uint32_t* err,
                      size_t rows, size_t pos0, size_t heads, uint32_t recip_den_shift, uint32_t recip_log2,
                      uint32_t norm_shift, int use_row_shift);
void or_fixed_av(const int16_t* weights, const int16_t* values, int64_t* accs, int16_t* outs, uint32_t* err,
                 size_t rows, size_t seq, size_t pos0, size_t d, size_t heads, uint32_t shift);
void or_fixed_lookup(const int16_t* input, const int16_t* lut, int16_t* out, size_t n);
void or_fixed_requant_i16(const int16_t* input, int16_t* out, uint32_t* err, size_t n, uint32_t shift);
void or_fixed_logits(const int16_t* input, const int16_t* w, int64_t* out, size_t rows, size_t d, size_t vocab);
/* attention proof wires (backend.cu:2202-2470) */
typedef struct {
    size_t query_rows, seq, pos0, heads, head_pad, head_dim, query_pad, seq_pad, d_pad;
    uint32_t shift_scores, shift_softmax_norm, shift_qkv, recip_den_shift, recip_log2;
    int32_t exp_pad_input, recip_pad_output, use_row_shift;
} or_wires_geom;
void or_attention_wires(const or_wires_geom* g, const int16_t* q, const int16_t* k_cache, const int16_t* own_k,
                        const int16_t* v, const int64_t* scores_acc, const int16_t* scores_q,
                        const int16_t* row_shifts, const int16_t* exp_outputs, const int64_t* denoms,
                        const int16_t* recips, const int16_t* weights, const int16_t* recip_lut,
                        const int64_t* qkv_acc, uint64_t* rect, uint64_t* rows_out, uint64_t* above,
                        uint64_t* qkv_cols, uint32_t* err);

#ifdef __cplusplus
}
#endif
#endif
