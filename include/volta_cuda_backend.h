/*
 * libvolta_cuda_backend.so -- B200 (sm_100a) build of VOLTA-ZK's accelerator
 * seam.  Drop-in for the reference library loaded by the Rust crate
 * `volta-accel` (okrame/volta-zk rust/volta-accel/src/cuda.rs:1119-1420:
 * dlopen, ABI version check, eager dlsym of every symbol below).
 *
 * Every declaration keeps the reference signature so the unchanged Rust FFI
 * binds it; each cites the reference definition in cuda/volta_cuda_backend.cu
 * (file:line).  Conventions (reference lines 300-403):
 *   - return 0 on success; -1 or a cudaError_t value on failure, with the
 *     message available from volta_cuda_last_error(ctx);
 *   - device buffers are opaque u64 ids ((generation << 32) | (slot + 1))
 *     plus element offsets; every region is bounds-checked on the host;
 *   - Fp2 values are canonical Goldilocks pairs {c0, c1} (phi^2 = 7);
 *   - one in-order stream per context; a context is used by one host thread
 *     at a time.
 * Entry points of the reference's X4b/X4c folding PCS and C3 private argmax
 * are outside this build's scope: they exist (the loader resolves every
 * symbol) and fail with "unsupported in the B200 build".
 */
#ifndef VOLTA_CUDA_BACKEND_H
#define VOLTA_CUDA_BACKEND_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Fp2Repr (rust/volta-accel/src/lib.rs:394-399); 16-byte aligned as the
 * reference's `struct alignas(16) Fp2` (cuda/volta_cuda_backend.cu:48-51). */
typedef struct __attribute__((aligned(16))) vz_fp2 {
    uint64_t c0;
    uint64_t c1;
} vz_fp2;

/* RawStats, 504 bytes (cuda/volta_cuda_backend.cu:55-124;
 * rust/volta-accel/src/cuda.rs:21-76).  Field order is ABI. */
typedef struct vz_raw_stats {
    uint64_t calls[7];
    uint64_t kernel_ns[7];
    uint64_t h2d_bytes, d2h_bytes, d2d_bytes, device_zeroed_bytes, device_generated_bytes;
    uint64_t h2d_ns, d2h_ns;
    uint64_t resident_h2d_host_calls, resident_d2h_host_calls;
    uint64_t resident_h2d_host_call_ns, resident_d2h_host_call_ns;
    uint64_t synchronizations, synchronization_ns;
    uint64_t sync_host_output, sync_upload_lifetime, sync_timing_flush, sync_profiling_legacy,
        sync_allocator_flush;
    uint64_t allocation_calls, resident_alloc_requests, resident_reuse_hits,
        resident_free_requests, physical_free_calls, live_device_bytes, peak_device_bytes;
    uint64_t pinned_allocation_calls, pinned_alloc_requests, pinned_reuse_hits,
        pinned_free_requests, pinned_physical_free_calls, pinned_host_write_calls,
        pinned_host_write_bytes, live_pinned_bytes, peak_pinned_bytes;
    uint64_t x4c_arena_reset_calls, x4c_arena_reset_bytes, x4c_kernel_launches,
        x4c_control_peek_calls, x4c_control_peek_pending;
    uint64_t timing_records, timing_elapsed_query_attempts, timing_elapsed_no_write,
        timing_event_queries, timing_event_api_calls, timing_pending_high_water,
        timing_flush_count, coarse_timing_scopes, coarse_timing_ns;
    uint32_t timing_mode;
    uint32_t reserved;
} vz_raw_stats;

/* RawPinnedMemoryStats, 104 bytes (cuda/volta_cuda_backend.cu:128-142). */
typedef struct vz_raw_pinned_stats {
    uint64_t active_bytes, cached_bytes, active_allocations, cached_allocations,
        in_flight_allocations, physical_allocation_calls, allocation_requests, reuse_hits,
        free_requests, physical_free_calls, host_write_calls, host_write_bytes, peak_bytes;
} vz_raw_pinned_stats;

/* RawX4cControlState, 104 bytes (cuda/volta_cuda_backend.cu:148-163). */
typedef struct vz_raw_control_state {
    uint32_t stream_state, flags;
    uint64_t outstanding_cuda_operations, pending_timing_records, active_device_allocations,
        cached_device_allocations, active_pinned_allocations, cached_pinned_allocations,
        in_flight_pinned_allocations, workspace_device_bytes, active_device_bytes,
        cached_device_bytes, active_pinned_bytes, cached_pinned_bytes;
} vz_raw_control_state;

/* AttentionProofWiresArgs (cuda/volta_cuda_backend.cu:2216-2252). */
typedef struct vz_attention_wires_args {
    uint64_t q_id; size_t q_offset;
    uint64_t k_cache_id; size_t k_cache_offset;
    uint64_t own_k_id; size_t own_k_offset;
    uint64_t v_id; size_t v_offset;
    uint64_t scores_acc_id; size_t scores_acc_offset;
    uint64_t scores_q_id; size_t scores_q_offset;
    uint64_t row_shifts_id; size_t row_shifts_offset;
    uint64_t exp_outputs_id; size_t exp_outputs_offset;
    uint64_t denoms_id; size_t denoms_offset;
    uint64_t recips_id; size_t recips_offset;
    uint64_t softmax_weights_id; size_t softmax_weights_offset;
    uint64_t recip_lut_id; size_t recip_lut_offset;
    uint64_t qkv_acc_id; size_t qkv_acc_offset;
    uint64_t error_id; size_t error_offset;
    uint64_t rect_id; size_t rect_offset;
    uint64_t rows_id; size_t rows_offset;
    uint64_t above_id; size_t above_offset;
    uint64_t qkv_id; size_t qkv_offset;
    size_t query_rows, seq, pos0, heads, head_pad, head_dim, query_pad, seq_pad, d_pad;
    uint32_t shift_scores, shift_softmax_norm, shift_qkv, recip_den_shift, recip_log2;
    int exp_pad_input, recip_pad_output, use_row_shift;
} vz_attention_wires_args;

/* ---- context, errors, measurement (reference 3148-3568) ------------------ */
uint32_t volta_cuda_abi_version(void);                            /* 3148; returns 37 */
int volta_cuda_create(void** out);                                /* 3150 */
void volta_cuda_destroy(void* ctx);                               /* 3177 */
const char* volta_cuda_last_error(void* ctx);                     /* 3203 */
int volta_cuda_set_resident_timing_policy(void* ctx, int policy); /* 3213: 0 deferred, 1 counters */
int volta_cuda_test_inject_elapsed_no_write_once(void* ctx);      /* 3241 */
int volta_cuda_begin_coarse_timing(void* ctx, int operation);     /* 3253 */
int volta_cuda_end_coarse_timing(void* ctx);                      /* 3277 */
int volta_cuda_abort_coarse_timing(void* ctx);                    /* 3306 */
int volta_cuda_ensure_timing_capacity(void* ctx, size_t bound, size_t* pending_before,
                                      size_t* pending_after, int* flushed); /* 3319 */
int volta_cuda_flush_profiling(void* ctx);                        /* 3347 */
int volta_cuda_reset_stats(void* ctx);                            /* 3359 */
int volta_cuda_get_stats(void* ctx, vz_raw_stats* out);           /* 3391 */
int volta_cuda_memory_breakdown(void* ctx, uint64_t* workspace_bytes, uint64_t* resident_bytes,
                                uint64_t* cached_resident_bytes); /* 3418 */
int volta_cuda_trim_resident_cache(void* ctx);                    /* 3450 */
int volta_cuda_pinned_memory_stats(void* ctx, vz_raw_pinned_stats* out); /* 3464 */
int volta_cuda_x4c_control_state(void* ctx, vz_raw_control_state* out);  /* 3502 */

/* ---- pinned pool and resident arena (reference 3570-3960) ---------------- */
int volta_cuda_pinned_alloc(void* ctx, size_t bytes, uint64_t* out_id);   /* 3570 */
int volta_cuda_pinned_write(void* ctx, uint64_t id, size_t offset_bytes, const void* source,
                            size_t bytes);                                /* 3654 */
int volta_cuda_pinned_wait_ready(void* ctx, uint64_t id);                 /* 3672 */
int volta_cuda_pinned_free(void* ctx, uint64_t id);                       /* 3698 */
int volta_cuda_trim_pinned_cache(void* ctx);                              /* 3719 */
int volta_cuda_resident_alloc(void* ctx, size_t bytes, uint64_t* out_id); /* 3733 */
int volta_cuda_resident_free(void* ctx, uint64_t id);                     /* 3818 */
int volta_cuda_resident_upload(void* ctx, uint64_t id, size_t offset_bytes, const void* src,
                               size_t bytes);                             /* 3843 */
int volta_cuda_resident_download(void* ctx, uint64_t id, size_t offset_bytes, void* dst,
                                 size_t bytes);                           /* 3863 */
int volta_cuda_resident_zero(void* ctx, uint64_t id, size_t offset_bytes, size_t bytes); /* 3883 */
int volta_cuda_resident_copy_rows(void* ctx, uint64_t src_id, size_t src_offset_bytes,
                                  size_t src_stride_bytes, uint64_t dst_id,
                                  size_t dst_offset_bytes, size_t dst_stride_bytes, size_t rows,
                                  size_t row_bytes);                      /* 3936 */
int volta_cuda_resident_mailbox_copy_rows(void* ctx, uint64_t src_id, size_t src_offset_bytes,
                                          size_t src_stride_bytes, uint64_t dst_id,
                                          size_t dst_offset_bytes, size_t dst_stride_bytes,
                                          size_t rows, size_t row_bytes); /* 3947 */

/* ---- ChaCha8 FpStream expansion (reference 3991-4047) -------------------- */
int volta_cuda_chacha8_prover_secret_fp_rows_device(void* ctx, uint64_t output_id,
                                                    size_t output_offset_bytes,
                                                    const uint8_t* prover_secret_seed,
                                                    uint64_t base_domain, size_t rows,
                                                    size_t count);        /* 3991 */
int volta_cuda_mock_correlation_sub_masks_device(void* ctx, uint64_t output_id,
                                                 size_t output_offset_bytes,
                                                 const uint8_t* mock_correlation_seed,
                                                 uint64_t base_domain, size_t rows,
                                                 size_t cols);            /* 4002 */
int volta_cuda_chacha8_prover_secret_fp2_rows_padded_device(void* ctx, uint64_t output_id,
                                                            size_t output_offset_bytes,
                                                            const uint8_t* prover_secret_seed,
                                                            uint64_t base_domain, size_t rows,
                                                            size_t count,
                                                            size_t padded_count); /* 4013 */

/* ---- small Fp2 vector primitives ----------------------------------------- */
int volta_cuda_fp2_row_dots_device(void* ctx, uint64_t a_id, size_t a_offset, size_t a_stride,
                                   uint64_t b_id, size_t b_offset, size_t b_stride,
                                   uint64_t output_id, size_t output_offset, size_t rows,
                                   size_t len);                           /* 4049 */
int volta_cuda_fp2_powers_device(void* ctx, uint64_t base_c0, uint64_t base_c1,
                                 uint64_t output_id, size_t output_offset, size_t count); /* 4107 */

/* ---- GEMM and fused requant + MAC-correction epilogue (reference 4128-4206) */
int volta_cuda_gemm_i64(void* ctx, const int16_t* a, const int16_t* b, int64_t* out, size_t m,
                        size_t k, size_t n);                              /* 4128 */
int volta_cuda_gemm_i64_device(void* ctx, uint64_t a_id, size_t a_offset, uint64_t b_id,
                               size_t b_offset, uint64_t out_id, size_t out_offset, size_t m,
                               size_t k, size_t n);                       /* 4143 */
int volta_cuda_gemm_requant_auth(void* ctx, const int16_t* a, const int16_t* b,
                                 const uint64_t* masks, int16_t* out, uint64_t* corr, size_t m,
                                 size_t k, size_t n, uint32_t shift);     /* 4164 */
int volta_cuda_gemm_requant_auth_device(void* ctx, uint64_t a_id, size_t a_offset, uint64_t b_id,
                                        size_t b_offset, uint64_t masks_id, size_t masks_offset,
                                        uint64_t out_id, size_t out_offset, uint64_t corr_id,
                                        size_t corr_offset, size_t m, size_t k, size_t n,
                                        uint32_t shift);                  /* 4182 */

/* ---- int16 fixed-point GPT-2 witness forward (reference 4208-4499) ------- */
int volta_cuda_fixed_embed_device(void* ctx, uint64_t tokens_id, size_t tokens_offset,
                                  uint64_t wte_id, size_t wte_offset, uint64_t wpe_id,
                                  size_t wpe_offset, uint64_t acc_id, size_t acc_offset,
                                  uint64_t out_id, size_t out_offset, uint64_t error_id,
                                  size_t error_offset, size_t rows, size_t d, size_t vocab,
                                  size_t positions, size_t pos0, int32_t shift); /* 4208 */
int volta_cuda_fixed_layer_norm_device(void* ctx, uint64_t input_id, size_t input_offset,
                                       uint64_t gain_id, size_t gain_offset, uint64_t bias_id,
                                       size_t bias_offset, uint64_t lut_id, size_t lut_offset,
                                       uint64_t mean_id, size_t mean_offset, uint64_t var_id,
                                       size_t var_offset, uint64_t rin_id, size_t rin_offset,
                                       uint64_t rout_id, size_t rout_offset, uint64_t acc_id,
                                       size_t acc_offset, uint64_t out_id, size_t out_offset,
                                       uint64_t error_id, size_t error_offset, size_t rows,
                                       size_t d, uint32_t var_shift, uint32_t norm_shift); /* 4238 */
int volta_cuda_fixed_gemm_device(void* ctx, uint64_t input_id, size_t input_offset,
                                 uint64_t weights_id, size_t weights_offset, uint64_t bias_id,
                                 size_t bias_offset, uint64_t residual_id, size_t residual_offset,
                                 uint64_t acc_id, size_t acc_offset, uint64_t requant_id,
                                 size_t requant_offset, uint64_t residual_out_id,
                                 size_t residual_out_offset, uint64_t error_id,
                                 size_t error_offset, size_t m, size_t k, size_t n,
                                 uint32_t shift);                         /* 4279 */
int volta_cuda_fixed_qkv_split_device(void* ctx, uint64_t input_id, size_t input_offset,
                                      uint64_t q_id, size_t q_offset, uint64_t k_id,
                                      size_t k_offset, uint64_t v_id, size_t v_offset,
                                      size_t rows, size_t d);             /* 4316 */
int volta_cuda_fixed_attention_scores_device(void* ctx, uint64_t q_id, size_t q_offset,
                                             uint64_t k_id, size_t k_offset, uint64_t acc_id,
                                             size_t acc_offset, uint64_t out_id,
                                             size_t out_offset, uint64_t error_id,
                                             size_t error_offset, size_t rows, size_t seq,
                                             size_t pos0, size_t heads, size_t head_dim,
                                             uint32_t shift);             /* 4338 */
int volta_cuda_fixed_softmax_device(void* ctx, uint64_t scores_id, size_t scores_offset,
                                    uint64_t exp_lut_id, size_t exp_lut_offset,
                                    uint64_t recip_lut_id, size_t recip_lut_offset,
                                    uint64_t row_shift_id, size_t row_shift_offset,
                                    uint64_t exp_id, size_t exp_offset, uint64_t denoms_id,
                                    size_t denoms_offset, uint64_t recips_id,
                                    size_t recips_offset, uint64_t weights_id,
                                    size_t weights_offset, uint64_t error_id,
                                    size_t error_offset, size_t rows, size_t seq, size_t pos0,
                                    size_t heads, uint32_t recip_den_shift, uint32_t recip_log2,
                                    uint32_t norm_shift, int use_row_shift); /* 4367 */
int volta_cuda_fixed_av_device(void* ctx, uint64_t weights_id, size_t weights_offset,
                               uint64_t values_id, size_t values_offset, uint64_t acc_id,
                               size_t acc_offset, uint64_t out_id, size_t out_offset,
                               uint64_t error_id, size_t error_offset, size_t rows, size_t seq,
                               size_t pos0, size_t d, size_t heads, uint32_t shift); /* 4409 */
int volta_cuda_fixed_lookup_device(void* ctx, uint64_t input_id, size_t input_offset,
                                   uint64_t lut_id, size_t lut_offset, uint64_t out_id,
                                   size_t out_offset, size_t n);          /* 4438 */
int volta_cuda_fixed_requant_i16_device(void* ctx, uint64_t input_id, size_t input_offset,
                                        uint64_t out_id, size_t out_offset, uint64_t error_id,
                                        size_t error_offset, size_t n, uint32_t shift); /* 4458 */
int volta_cuda_fixed_logits_device(void* ctx, uint64_t input_id, size_t input_offset,
                                   uint64_t weights_id, size_t weights_offset, uint64_t out_id,
                                   size_t out_offset, size_t rows, size_t d, size_t vocab); /* 4479 */

/* ---- C3 private argmax (out of scope: unsupported) (reference 4501-4610) - */
int volta_cuda_private_argmax_witness_device(
    void* ctx, uint64_t input_id, size_t input_offset, uint64_t selected_indices_id,
    size_t selected_indices_offset, uint64_t selected_rows_id, size_t selected_rows_offset,
    uint64_t logits_id, size_t logits_offset, uint64_t strict_id, size_t strict_offset,
    uint64_t is_max_id, size_t is_max_offset, uint64_t packed_strict_id,
    size_t packed_strict_offset, uint64_t limbs_id, size_t limbs_offset, uint64_t error_id,
    size_t error_offset, size_t rows, size_t vocab, size_t rect_entries, size_t lookup_entries,
    size_t first_job_entries, size_t selected_row_entries);            /* 4501 */
int volta_cuda_private_argmax_phase_factors_device(void* ctx, uint64_t logits_id,
                                                   size_t logits_offset, uint64_t mask_id,
                                                   size_t mask_offset, uint64_t masked_id,
                                                   size_t masked_offset, size_t entries,
                                                   size_t row_start, size_t row_count,
                                                   size_t vocab);         /* 4558 */
int volta_cuda_private_argmax_selector_device(void* ctx, uint64_t eq_vocab_id,
                                              size_t eq_vocab_offset, uint64_t eq_rows_id,
                                              size_t eq_rows_offset, uint64_t output_id,
                                              size_t output_offset, size_t entries, size_t job,
                                              size_t vocab, vz_fp2 coefficient); /* 4581 */

/* ---- subfield corrections, padding, matrix folds (reference 4612-4713) --- */
int volta_cuda_subfield_corrections_device(void* ctx, uint64_t input_id, size_t input_offset,
                                           uint64_t masks_id, size_t masks_offset,
                                           uint64_t output_id, size_t output_offset, size_t n,
                                           int kind);                     /* 4612 */
int volta_cuda_pad_base_vector_device(void* ctx, uint64_t input_id, size_t input_offset,
                                      uint64_t output_id, size_t output_offset, size_t real,
                                      size_t padded, uint64_t pad, int kind); /* 4633 */
int volta_cuda_matrix_fold_device(void* ctx, uint64_t input_id, size_t input_offset,
                                  uint64_t weights_id, size_t weights_offset, uint64_t output_id,
                                  size_t output_offset, size_t rows, size_t stride,
                                  size_t column_offset, size_t cols, size_t out_pad, int kind,
                                  int axis);                              /* 4655 */

/* ---- sumcheck round engine (reference 4715-5153) ------------------------- */
int volta_cuda_fp2_dot_device(void* ctx, uint64_t a_id, size_t a_offset, uint64_t b_id,
                              size_t b_offset, size_t n, vz_fp2* output); /* 4715 */
int volta_cuda_reserve_fp2_product_round_workspace(void* ctx, size_t max_pairs); /* 4748 */
int volta_cuda_reserve_logup_round_workspace(void* ctx, size_t max_pairs);       /* 4768 */
int volta_cuda_fp2_product_round_device(void* ctx, uint64_t a_id, size_t a_offset, uint64_t b_id,
                                        size_t b_offset, size_t pairs, vz_fp2* output); /* 4827 */
int volta_cuda_fp2_product_round_into_device(void* ctx, uint64_t a_id, size_t a_offset,
                                             uint64_t b_id, size_t b_offset, size_t pairs,
                                             uint64_t output_id, size_t output_offset); /* 4846 */
int volta_cuda_fp2_product_round_scaled_into_device(void* ctx, uint64_t a_id, size_t a_offset,
                                                    uint64_t b_id, size_t b_offset, size_t pairs,
                                                    vz_fp2 scale, uint64_t output_id,
                                                    size_t output_offset); /* 4870 */
int volta_cuda_claim_reduce_f_two_into_device(void* ctx, uint64_t points_id, size_t points_offset,
                                              size_t n_vars, uint64_t output_id,
                                              size_t output_offset, uint64_t scratch_one_id,
                                              size_t scratch_one_offset, uint64_t scratch_two_id,
                                              size_t scratch_two_offset,
                                              uint64_t scratch_three_id,
                                              size_t scratch_three_offset); /* 4895 */
int volta_cuda_x4d_link_eq_accumulate_device(void* ctx, uint64_t point_id, size_t point_offset,
                                             size_t n_vars, uint64_t target_id,
                                             size_t target_offset, uint64_t scratch_one_id,
                                             size_t scratch_one_offset, uint64_t scratch_two_id,
                                             size_t scratch_two_offset, int initialize); /* 4959 */
int volta_cuda_fp2_dot_scaled_pair_into_device(void* ctx, uint64_t a_id, size_t a_offset,
                                               uint64_t b_id, size_t b_offset, size_t n,
                                               vz_fp2 scale, uint64_t output_id,
                                               size_t output_offset); /* 5001 */
int volta_cuda_fp2_pair_sum_device(void* ctx, uint64_t input_id, size_t input_offset,
                                   size_t pairs, vz_fp2* output);        /* 5034 */
int volta_cuda_fp2_triple_product_round_device(void* ctx, uint64_t a_id, size_t a_offset,
                                               uint64_t b_id, size_t b_offset, uint64_t c_id,
                                               size_t c_offset, size_t pairs,
                                               vz_fp2* output);           /* 5106 */
int volta_cuda_fp2_triple_product_round_into_device(void* ctx, uint64_t a_id, size_t a_offset,
                                                    uint64_t b_id, size_t b_offset,
                                                    uint64_t c_id, size_t c_offset, size_t pairs,
                                                    uint64_t output_id,
                                                    size_t output_offset); /* 5129 */

/* ---- lookup-column preparation and attention wires (reference 5155-5532) - */
int volta_cuda_ln_hadamard_factors_device(void* ctx, uint64_t input_id, size_t input_offset,
                                          uint64_t mean_id, size_t mean_offset, uint64_t rsqrt_id,
                                          size_t rsqrt_offset, uint64_t gain_id,
                                          size_t gain_offset, uint64_t centered_id,
                                          size_t centered_offset, uint64_t scaled_id,
                                          size_t scaled_offset, size_t rows, size_t cols,
                                          size_t row_pad, size_t col_pad); /* 5155 */
int volta_cuda_base_broadcast_fp2_device(void* ctx, uint64_t input_id, size_t input_offset,
                                         uint64_t output_id, size_t output_offset,
                                         size_t input_len, size_t repeat, int kind); /* 5186 */
int volta_cuda_repeat_vector_device(void* ctx, uint64_t input_id, size_t input_offset,
                                    uint64_t output_id, size_t output_offset, size_t input_len,
                                    size_t repeat, int kind);             /* 5208 */
int volta_cuda_compact_strided_rows_device(void* ctx, uint64_t input_id, size_t input_offset,
                                           uint64_t output_id, size_t output_offset, size_t rows,
                                           size_t source_stride, size_t width, int kind); /* 5231 */
int volta_cuda_attention_above_mask_device(void* ctx, uint64_t equality_id,
                                           size_t equality_offset, size_t entries, size_t rows,
                                           size_t seq, size_t pos0, size_t heads,
                                           size_t head_pad, size_t query_pad,
                                           size_t seq_pad);               /* 5254 */
int volta_cuda_attention_proof_wires_device(void* ctx, const vz_attention_wires_args* args); /* 5278 */
int volta_cuda_requant_columns_device(void* ctx, uint64_t acc_id, size_t acc_offset,
                                      uint64_t out_id, size_t out_offset, uint64_t columns_id,
                                      size_t columns_offset, uint64_t error_id,
                                      size_t error_offset, size_t rows, size_t cols,
                                      size_t row_pad, size_t col_pad, int acc_kind,
                                      uint32_t shift);                    /* 5378 */
int volta_cuda_pair_columns_device(void* ctx, uint64_t input_id, size_t input_offset,
                                   uint64_t out_id, size_t out_offset, uint64_t columns_id,
                                   size_t columns_offset, size_t rows, size_t cols,
                                   size_t row_pad, size_t col_pad, uint64_t pad_input,
                                   uint64_t pad_output, int input_kind, int output_kind); /* 5409 */
int volta_cuda_histogram_lut_device(void* ctx, uint64_t input_id, size_t input_offset,
                                    uint64_t output_id, size_t output_offset, size_t n,
                                    int signed_input);                    /* 5438 */
int volta_cuda_histogram_fp_device(void* ctx, uint64_t input_id, size_t input_offset,
                                   uint64_t output_id, size_t output_offset, size_t n,
                                   size_t bins);                          /* 5458 */
int volta_cuda_u32_add_inplace_device(void* ctx, uint64_t target_id, size_t target_offset,
                                      uint64_t add_id, size_t add_offset, size_t n); /* 5476 */
int volta_cuda_pack_lookup_leaf_device(void* ctx, uint64_t columns_id, size_t columns_offset,
                                       uint64_t shifts_id, size_t shifts_offset, uint64_t leaf_id,
                                       size_t leaf_offset, size_t column_count, size_t n,
                                       uint64_t alpha0);                  /* 5493 */
int volta_cuda_deinterleave_base_columns_device(void* ctx, uint64_t columns_id,
                                                size_t columns_offset, uint64_t output_id,
                                                size_t output_offset, size_t column_count,
                                                size_t n);                /* 5515 */

/* ---- NTT (reference 5534-5576, 6545-6579) -------------------------------- */
int volta_cuda_ntt_fp(void* ctx, const uint64_t* msg, size_t msg_len, size_t n, uint64_t* out); /* 5534 */
int volta_cuda_ntt_fp_batch(void* ctx, const uint64_t* messages, size_t rows, size_t msg_len,
                            size_t n, uint64_t* out);                     /* 5546 */
int volta_cuda_ntt_fp2(void* ctx, const vz_fp2* msg, size_t msg_len, size_t n, vz_fp2* out); /* 5561 */
int volta_cuda_ntt_fp_batch_device(void* ctx, uint64_t input_id, size_t input_offset, size_t rows,
                                   size_t n, uint64_t output_id, size_t output_offset); /* 6545 */
int volta_cuda_ntt_fp2_batch_device(void* ctx, uint64_t input_id, size_t input_offset,
                                    size_t rows, size_t n, uint64_t output_id,
                                    size_t output_offset);                /* 6563 */

/* ---- X4b / X4c folding PCS (out of scope: unsupported) (reference 5577-6543) */
int volta_cuda_x4b_ntt_fp2(void* ctx, const vz_fp2* coefficients, size_t coefficient_len, size_t n,
                           vz_fp2* output);                               /* 5577 */
int volta_cuda_x4b_context_probe(void* ctx, const uint8_t* payload, size_t length,
                                 uint8_t* output);                        /* 5637 */
int volta_cuda_x4b_n4_inner_tile(void* ctx, const vz_fp2* symbols, size_t present_slots,
                                 size_t coordinates, const uint16_t* present_rank,
                                 const uint8_t* descriptors, size_t structural_slots,
                                 uint64_t coordinate_start, uint32_t cohort_id,
                                 uint8_t oracle_kind, uint8_t fold_round,
                                 uint8_t* outer_leaves);                  /* 5667 */
int volta_cuda_x4b_n4_outer_nodes(void* ctx, const uint8_t* children, size_t parents,
                                  uint64_t node_start, uint32_t cohort_id, uint8_t oracle_kind,
                                  uint8_t fold_round, uint8_t level, uint8_t* output); /* 5768 */
int volta_cuda_x4c_upload_pinned(void* ctx, uint64_t pinned_id_value, size_t pinned_offset_bytes,
                                 uint64_t arena_id, size_t arena_offset_bytes, size_t bytes); /* 5808 */
int volta_cuda_x4c_direct_fold_pinned_tile(void* ctx, uint64_t pinned_id_value,
                                           size_t pinned_offset_bytes, uint64_t arena_id,
                                           size_t output_offset_bytes,
                                           size_t scratch_offset_bytes, size_t input_len,
                                           size_t output_start, size_t output_count,
                                           uint64_t challenge_c0, uint64_t challenge_c1); /* 5839 */
int volta_cuda_x4c_direct_fold_arena(void* ctx, uint64_t arena_id, size_t input_offset_bytes,
                                     size_t input_len, size_t output_offset_bytes,
                                     uint64_t challenge_c0, uint64_t challenge_c1); /* 5925 */
int volta_cuda_x4c_activation_add_pinned_tile(void* ctx, uint64_t pinned_id_value,
                                              size_t pinned_offset_bytes, uint64_t arena_id,
                                              size_t destination_offset_bytes,
                                              size_t scratch_offset_bytes, size_t count,
                                              uint64_t activation_c0,
                                              uint64_t activation_c1);   /* 5974 */
int volta_cuda_x4c_build_one_slot_n4(void* ctx, uint64_t arena_id, size_t codeword_offset_bytes,
                                     size_t outer_len, size_t cache_offset_bytes,
                                     const uint8_t* descriptor_bytes, uint32_t cohort_id,
                                     uint8_t oracle_kind, uint8_t fold_round,
                                     uint8_t* root_output);               /* 6032 */
int volta_cuda_x4c_gather_fp2_samples(void* ctx, uint64_t arena_id, size_t source_offset_bytes,
                                      size_t symbols, const uint64_t* indices, size_t count,
                                      vz_fp2* output);                    /* 6109 */
int volta_cuda_x4c_batch_gather_bytes(void* ctx, uint64_t arena_id, uint64_t pinned_requests_id,
                                      size_t pinned_requests_offset_bytes, size_t request_count,
                                      size_t request_scratch_offset_bytes,
                                      size_t mailbox_offset_bytes, size_t mailbox_len); /* 6150 */
int volta_cuda_x4c_batch_gather_canonical_operations(void* ctx, uint64_t arena_id,
                                                     uint64_t pinned_operations_id,
                                                     size_t pinned_operations_offset_bytes,
                                                     size_t operation_count,
                                                     size_t operation_scratch_offset_bytes,
                                                     size_t mailbox_offset_bytes,
                                                     size_t mailbox_len); /* 6262 */
int volta_cuda_x4c_arena_reset(void* ctx, uint64_t arena_id, size_t offset_bytes, size_t bytes,
                               int zero);                                 /* 6513 */
int volta_cuda_x4c_session_reusable_boundary(void* ctx);                  /* 6534 */

/* ---- LogUp fraction tree, rounds and folds (reference 6581-7062) --------- */
int volta_cuda_logup_tree(void* ctx, const uint64_t* leaf, const uint32_t* mult, size_t n,
                          uint64_t alpha1, int neg_mult, vz_fp2* hp, vz_fp2* hq); /* 6581 */
int volta_cuda_logup_tree_device(void* ctx, uint64_t leaf_id, size_t leaf_offset,
                                 uint64_t mult_id, size_t mult_offset, size_t n, uint64_t alpha1,
                                 int neg_mult, uint64_t p_id, size_t p_offset, uint64_t q_id,
                                 size_t q_offset);                        /* 6598 */
int volta_cuda_logup_materialize_leaves_device(void* ctx, uint64_t leaf_id, size_t leaf_offset,
                                               uint64_t mult_id, size_t mult_offset, size_t n,
                                               uint64_t alpha1, int neg_mult, uint64_t p_id,
                                               size_t p_offset, uint64_t q_id,
                                               size_t q_offset);          /* 6630 */
int volta_cuda_logup_general_round(void* ctx, const vz_fp2* p0, const vz_fp2* p1,
                                   const vz_fp2* q0, const vz_fp2* q1, const vz_fp2* suffix,
                                   size_t pairs, vz_fp2* output);         /* 6655 */
int volta_cuda_logup_general_round_device(void* ctx, uint64_t p0_id, size_t p0_offset,
                                          uint64_t p1_id, size_t p1_offset, uint64_t q0_id,
                                          size_t q0_offset, uint64_t q1_id, size_t q1_offset,
                                          uint64_t suffix_id, size_t suffix_offset, size_t pairs,
                                          vz_fp2* output);                /* 6728 */
int volta_cuda_logup_general_round_into_device(void* ctx, uint64_t p0_id, size_t p0_offset,
                                               uint64_t p1_id, size_t p1_offset, uint64_t q0_id,
                                               size_t q0_offset, uint64_t q1_id, size_t q1_offset,
                                               uint64_t suffix_id, size_t suffix_offset,
                                               size_t pairs, uint64_t output_id,
                                               size_t output_offset);    /* 6746 */
int volta_cuda_logup_fold4(void* ctx, const vz_fp2* p0, const vz_fp2* p1, const vz_fp2* q0,
                           const vz_fp2* q1, size_t pairs, vz_fp2 r, vz_fp2* o0, vz_fp2* o1,
                           vz_fp2* o2, vz_fp2* o3);                       /* 6771 */
int volta_cuda_logup_fold4_device(void* ctx, uint64_t p0_id, size_t p0_offset, uint64_t p1_id,
                                  size_t p1_offset, uint64_t q0_id, size_t q0_offset,
                                  uint64_t q1_id, size_t q1_offset, size_t pairs, vz_fp2 r,
                                  uint64_t o0_id, size_t o0_offset, uint64_t o1_id,
                                  size_t o1_offset, uint64_t o2_id, size_t o2_offset,
                                  uint64_t o3_id, size_t o3_offset);     /* 6781 */
int volta_cuda_fp2_deinterleave_device(void* ctx, uint64_t input_id, size_t input_offset,
                                       size_t pairs, uint64_t even_id, size_t even_offset,
                                       uint64_t odd_id, size_t odd_offset); /* 6810 */
int volta_cuda_logup_suffix_eq_device(void* ctx, uint64_t points_id, size_t points_offset,
                                      size_t point_len, uint64_t output_id,
                                      size_t output_offset);              /* 6833 */
int volta_cuda_fp2_fold_rows_device(void* ctx, uint64_t input_id, size_t input_offset,
                                    size_t rows, size_t len, vz_fp2 r, uint64_t output_id,
                                    size_t output_offset);                /* 6862 */
int volta_cuda_logup_eq_rows_device(void* ctx, uint64_t points_id, size_t points_offset,
                                    size_t rows, size_t dims, uint64_t output_id,
                                    size_t output_offset);                /* 6884 */
int volta_cuda_logup_aux_round_device(void* ctx, uint64_t q0_id, size_t q0_offset, uint64_t q1_id,
                                      size_t q1_offset, uint64_t suffix_id, size_t suffix_offset,
                                      uint64_t columns_id, size_t columns_offset, uint64_t eq_id,
                                      size_t eq_offset, uint64_t claim_cols_id,
                                      size_t claim_cols_offset, uint64_t weights_id,
                                      size_t weights_offset, size_t column_count,
                                      size_t claim_count, size_t vector_len, vz_fp2 lambda,
                                      vz_fp2 cpref, vz_fp2 point, vz_fp2* output); /* 7008 */
int volta_cuda_logup_aux_round_into_device(void* ctx, uint64_t q0_id, size_t q0_offset,
                                           uint64_t q1_id, size_t q1_offset, uint64_t suffix_id,
                                           size_t suffix_offset, uint64_t columns_id,
                                           size_t columns_offset, uint64_t eq_id,
                                           size_t eq_offset, uint64_t claim_cols_id,
                                           size_t claim_cols_offset, uint64_t weights_id,
                                           size_t weights_offset, size_t column_count,
                                           size_t claim_count, size_t vector_len, vz_fp2 lambda,
                                           vz_fp2 cpref, vz_fp2 point, uint64_t output_id,
                                           size_t output_offset);        /* 7033 */

/* ---- Ligero PCS rows, Merkle (reference 7064-7264) ----------------------- */
int volta_cuda_pcs_messages_device(void* ctx, uint64_t weights_id, size_t weights_offset,
                                   uint64_t pads_id, size_t pads_offset, size_t rows, size_t cols,
                                   size_t pad, size_t code_len, uint64_t output_id,
                                   size_t output_offset);                 /* 7064 */
int volta_cuda_pcs_combine_rows_device(void* ctx, uint64_t weights_id, size_t weights_offset,
                                       uint64_t pads_id, size_t pads_offset, uint64_t coeffs_id,
                                       size_t coeffs_offset, size_t rows, size_t cols, size_t pad,
                                       size_t combinations, uint64_t output_id,
                                       size_t output_offset);             /* 7081 */
int volta_cuda_fp2_add_inplace_device(void* ctx, uint64_t target_id, size_t target_offset,
                                      uint64_t add_id, size_t add_offset, size_t n); /* 7101 */
int volta_cuda_fp2_mobius_inverse_inplace_device(void* ctx, uint64_t values_id,
                                                 size_t values_offset, size_t n); /* 7114 */
int volta_cuda_fp2_affine_eq_weights_inplace_device(void* ctx, uint64_t values_id, size_t n,
                                                    size_t source_count, uint64_t point_id,
                                                    size_t point_offset, size_t point_len,
                                                    uint64_t rho_c0, uint64_t rho_c1,
                                                    uint64_t gamma_c0, uint64_t gamma_c1); /* 7132 */
int volta_cuda_hash_fp_tree_device(void* ctx, uint64_t matrix_id, size_t matrix_offset,
                                   size_t rows, size_t cols, uint64_t tree_id,
                                   size_t tree_offset_bytes);             /* 7166 */
int volta_cuda_hash_fp2_tree_device(void* ctx, uint64_t matrix_id, size_t matrix_offset,
                                    size_t rows, size_t cols, uint64_t tree_id,
                                    size_t tree_offset_bytes);            /* 7177 */
int volta_cuda_merkle_paths_device(void* ctx, uint64_t tree_id, size_t tree_offset_bytes,
                                   size_t leaves, uint64_t indices_id, size_t indices_offset,
                                   size_t queries, uint64_t paths_id,
                                   size_t paths_offset_bytes);            /* 7188 */
int volta_cuda_pcs_gather_columns_device(void* ctx, uint64_t matrix_id, size_t matrix_offset,
                                         size_t rows, size_t cols, uint64_t indices_id,
                                         size_t indices_offset, size_t queries,
                                         uint64_t output_id, size_t output_offset, int fp2); /* 7206 */
int volta_cuda_pcs_combine_rows(void* ctx, const int16_t* weights, const uint64_t* pads,
                                const vz_fp2* coeffs, size_t rows, size_t cols, size_t pad,
                                size_t combinations, vz_fp2* out);        /* 7228 */
int volta_cuda_pcs_gather_columns(void* ctx, const uint64_t* matrix, size_t rows, size_t cols,
                                  const uint32_t* indices, size_t queries, uint64_t* out); /* 7243 */
int volta_cuda_hash_fp_columns(void* ctx, const uint64_t* matrix, size_t rows, size_t cols,
                               uint8_t* leaves);                          /* 7256 */

#ifdef __cplusplus
}
#endif
#endif /* VOLTA_CUDA_BACKEND_H */
