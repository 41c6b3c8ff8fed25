/*
 * Extensions of libvolta_cuda_backend.so that have no counterpart in the
 * reference seam: timing markers, fused and batched forms of the seam's
 * round kernels used by the scheduled drivers, the column builders of the
 * GPT-2 proof schedule, and the allocation-free round.  A caller of the
 * reference ABI can ignore them.
 */
#ifndef VOLTA_B200_EXT_H
#define VOLTA_B200_EXT_H

#include <stddef.h>
#include <stdint.h>

#include "volta_cuda_backend.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Record timing marker `slot` (0..15) on the context's stream. */
int volta_b200_timing_mark(void* ctx, int slot);
/* Wait for marker `end` and return the device time between two markers. */
int volta_b200_timing_elapsed(void* ctx, int start, int end, float* ms);
/* Kernels this context has launched since it was created. */
int volta_b200_launch_count(void* ctx, uint64_t* launches);

/*
 * Fused fold + next round message.  With r the challenge of round j, fold the
 * current resident vectors (len entries each, len a multiple of 4, offset 0)
 * into the output vectors (len/2 entries) exactly as
 * volta_cuda_fp2_fold_rows_device / volta_cuda_logup_fold4_device would, and
 * return the round j+1 message over the folded vectors exactly as
 * volta_cuda_fp2_triple_product_round_device / volta_cuda_logup_general_round_device
 * would (the LogUp variant reads its suffix table at (suffix_id, suffix_offset)).
 * One pass over the data and one launch instead of two (four for three folds).
 */
int volta_b200_triple_fold_round_device(void* ctx, uint64_t a_id, uint64_t b_id, uint64_t c_id, size_t len,
                                        vz_fp2 r, uint64_t a_out_id, uint64_t b_out_id, uint64_t c_out_id,
                                        vz_fp2* output);
int volta_b200_logup_fold_round_device(void* ctx, uint64_t p0_id, uint64_t p1_id, uint64_t q0_id,
                                       uint64_t q1_id, size_t len, vz_fp2 r, uint64_t o0_id, uint64_t o1_id,
                                       uint64_t o2_id, uint64_t o3_id, uint64_t suffix_id, size_t suffix_offset,
                                       vz_fp2* output);
/* The same, writing the message to the resident buffer (out_id, out_offset
 * in Fp2 elements) instead of the host, with no synchronisation, like the
 * reference's *_into_device rounds. */
int volta_b200_triple_fold_round_into_device(void* ctx, uint64_t a_id, uint64_t b_id, uint64_t c_id, size_t len,
                                             vz_fp2 r, uint64_t a_out_id, uint64_t b_out_id, uint64_t c_out_id,
                                             uint64_t out_id, size_t out_offset);
int volta_b200_logup_fold_round_into_device(void* ctx, uint64_t p0_id, uint64_t p1_id, uint64_t q0_id,
                                            uint64_t q1_id, size_t len, vz_fp2 r, uint64_t o0_id, uint64_t o1_id,
                                            uint64_t o2_id, uint64_t o3_id, uint64_t suffix_id,
                                            size_t suffix_offset, uint64_t out_id, size_t out_offset);

/*
 * Every round of a general LogUp sumcheck on four resident vectors p0, p1,
 * q0, q1 of len = 2^L entries (L >= 1), challenges r[0..L) known in advance
 * (replaces the reference's per-round volta_cuda_logup_general_round_device
 * + volta_cuda_logup_fold4_device loop, rust/volta-proto/src/logup.rs:427-471,
 * and its blind-rounds benchmark loop cuda/p7_logup_blind_rounds.cu:403-431).
 * Round j's message reads the suffix table's first len >> (j+1) entries at
 * (suffix_id, suffix_offset).  The folded levels 1 .. L-1 of vector k go to
 * ladder k (len - 2 entries; level j at offset len - 2 (len >> j); unused
 * when len == 2).  Output at (out_id, out_offset): 4 L accumulators (pq0,
 * pq2, qq0, qq2 of each round, as volta_cuda_logup_general_round_device
 * returns them), then the four final values p0, p1, q0, q1.  L + 1 launches,
 * no host wait.
 */
int volta_b200_logup_rounds_device(void* ctx, uint64_t p0_id, uint64_t p1_id, uint64_t q0_id, uint64_t q1_id,
                                   size_t len, uint64_t suffix_id, size_t suffix_offset, const vz_fp2* r,
                                   uint64_t ladder0_id, uint64_t ladder1_id, uint64_t ladder2_id,
                                   uint64_t ladder3_id, uint64_t out_id, size_t out_offset);

/*
 * Blind LogUp corrections (rust/volta-proto/src/logup.rs:1903-2000
 * BlindSink::root / round / splits; cuda/p7_logup_blind_rounds.cu:180-214):
 * per job, one fraction-tree layer whose raw round output is resident in the
 * layout above (4 accumulators per round, then the four split values).
 * Output, in proof order, each value minus the mask at the same index:
 *   [root p, root q]       only when root_id != 0
 *   h0_j, h2_j per round   h = cpref (lambda pq + qq), cpref *= 2 pt r + 1 - pt - r
 *   p0, p1, q0, q1         the split values
 *   p0 q1, p1 q0, q0 q1    the layer-end products
 * sched holds the rounds claim-point coordinates and then the rounds
 * challenges.  Any number of jobs (rounds <= 64 each); one launch per 64.
 */
typedef struct vzb_blind_job {
    uint64_t raw_id;
    size_t raw_offset;
    uint64_t root_id;
    size_t root_offset;
    uint64_t sched_id;
    size_t sched_offset;
    uint64_t mask_id;
    size_t mask_offset;
    uint64_t out_id;
    size_t out_offset;
    vz_fp2 lambda;
    size_t rounds;
} vzb_blind_job;
int volta_b200_logup_blind_corrections_device(void* ctx, const vzb_blind_job* jobs, size_t count);

/*
 * LogUp layer rounds read straight from a fraction-tree level: the layer's
 * vectors p0, p1, q0, q1 (vector_len entries each) are the even/odd children
 * p[child_offset + 2k], p[child_offset + 2k + 1], q[...] of the level.
 * round_il: round 0 (as volta_cuda_logup_general_round_into_device on the
 * deinterleaved vectors); fold_round_il: fold with r into the four resident
 * half-length vectors o0..o3 and the next round's message (as
 * volta_b200_logup_fold_round_into_device), suffix table at
 * (suffix_id, suffix_offset).
 */
int volta_b200_logup_round_il_into_device(void* ctx, uint64_t p_id, uint64_t q_id, size_t child_offset,
                                          size_t vector_len, uint64_t suffix_id, size_t suffix_offset,
                                          uint64_t out_id, size_t out_offset);
int volta_b200_logup_fold_round_il_into_device(void* ctx, uint64_t p_id, uint64_t q_id, size_t child_offset,
                                               size_t vector_len, vz_fp2 r, uint64_t o0_id, uint64_t o1_id,
                                               uint64_t o2_id, uint64_t o3_id, uint64_t suffix_id,
                                               size_t suffix_offset, uint64_t out_id, size_t out_offset);

/*
 * Column commitments of row-sharded matrices (one Ligero commitment over
 * several GPUs).  A column's BLAKE3 tree over rows = 128 * 2^k is a perfect
 * binary tree of 1 KiB chunks, so a slab of 128 * 2^j aligned rows is one of
 * its subtrees.
 * hash_fp_column_cvs: per column of a rows x cols Fp slab, the non-root
 *   chaining value of that subtree (first chunk's global index chunk_base),
 *   32 bytes per column.
 * merkle_from_cvs: column leaves from the `shards` subtree values per column
 *   ([shards][cols] x 32 B, top-to-bottom slab order) merged left to right
 *   with ROOT on the final merge, then the Merkle tree over them (layout of
 *   volta_cuda_hash_fp_tree_device).
 * merkle_levels: the levels above `leaves` leaves already stored at level 0.
 */
int volta_b200_hash_fp_column_cvs_device(void* ctx, uint64_t matrix_id, size_t matrix_offset, size_t rows,
                                         size_t cols, uint64_t chunk_base, uint64_t out_id,
                                         size_t out_offset_bytes);
int volta_b200_merkle_from_cvs_device(void* ctx, uint64_t cvs_id, size_t cvs_offset_bytes, size_t shards,
                                      size_t cols, uint64_t tree_id, size_t tree_offset_bytes);
int volta_b200_merkle_levels_device(void* ctx, uint64_t tree_id, size_t tree_offset_bytes, size_t leaves);

/*
 * Whole small sumchecks in one CTA each, with the challenges in device memory
 * (known in advance in the clear sink / private transcript).
 *
 * A LogUp layer job runs all `rounds` (<= 11) rounds of a layer sumcheck on
 * vectors of 2^rounds entries: either four resident vectors (v_id[k] at
 * v_offset[k]) or, when il_p_id != 0, the interleaved children
 * (p, q)[il_offset .. il_offset + 2^(rounds+1)) of a fraction-tree level.
 * Its suffix-eq tables come from the `rounds` claim-point coordinates at
 * (point_id, point_offset); round j folds with the challenge at
 * (r_id, r_offset + j).  Output at (out_id, out_offset): per round the four
 * raw accumulators of volta_cuda_logup_general_round_device, then the four
 * final values (p0, p1, q0, q1).  Jobs are independent (one CTA each).
 */
typedef struct vzb_layer_job {
    uint64_t v_id[4];
    size_t v_offset[4];
    uint64_t il_p_id, il_q_id;
    size_t il_offset;
    size_t rounds;
    uint64_t point_id;
    size_t point_offset;
    uint64_t r_id;
    size_t r_offset;
    uint64_t out_id;
    size_t out_offset;
} vzb_layer_job;
int volta_b200_logup_layers_device(void* ctx, const vzb_layer_job* jobs, size_t count);

/*
 * Batched LogUp layer rounds.  In the clear sink / private transcript every
 * layer's claim point and challenges are known in advance, so the round
 * steps of different fraction-tree layers are independent; this call runs
 * `count` (<= 24) of them in one launch, each exactly one of these calls:
 *   kind 0: volta_b200_logup_round_il_into_device (in_id[0] = P, in_id[1] = Q,
 *           the interleaved children at in_offset[0]; len = vector length);
 *   kind 1: volta_b200_logup_fold_round_il_into_device (the same inputs, fold
 *           with r into out_id[k] at out_offset[k], len / 2 entries each);
 *   kind 2: volta_b200_logup_fold_round_into_device (the four vectors in_id[k]
 *           at in_offset[k], len entries each, folded into out_id[k]);
 *   kind 3: volta_cuda_logup_fold4_device (the fold of kind 2, no round).
 * Kinds 0-2 read the suffix-eq table at (s_id, s_offset) and write the four
 * raw accumulators at (msg_id, msg_offset).  r = (c0, c1) of the challenge.
 * flags bit 0 (VZB_ROUND_P_ONE): every numerator entry (P, or the p0 and p1
 * vectors) equals 1, as in the leaf layer of a side without multiplicities
 * (logup materialize_leaves).  The numerators are then neither read nor
 * written, except that kind 3 writes ones into out_id[0] and out_id[1]; the
 * results equal those of the same job on all-one numerators.
 * flags bit 1 (VZB_ROUND_Q_COLUMN, kinds 0 and 1 with P_ONE): the children
 * are the leaves themselves, read from a query column: in_id[1] is that
 * column (u64 Fp values f_j from in_offset[0]) and child j's denominator is
 * (q_alpha[0] - f_j, q_alpha[1]) (materialize_leaves of the packed leaf
 * alpha0 - f_j), so neither the leaves nor their denominators are stored.
 * flags bit 2 (VZB_ROUND_PARENTS, kind 0 without P_ONE): out_id[0] and
 * out_id[1] (from out_offset[0], len entries each) hold the layer's own tree
 * level, the parents of the children: for pair i, a0 d0 + b0 c0 and c0 d0 are
 * the parent p and q at index 2 i (p = pa qb + pb qa, q = qa qb), so they are
 * read instead of recomputed.  Correct only when they are those parents.
 * Outputs of different jobs must not overlap each other or any input.
 */
#define VZB_ROUND_P_ONE 1u
#define VZB_ROUND_Q_COLUMN 2u
#define VZB_ROUND_PARENTS 4u
typedef struct vzb_round_job {
    uint32_t kind;
    uint32_t flags;
    uint64_t in_id[4];
    size_t in_offset[4];
    size_t len;
    uint64_t r[2];
    uint64_t out_id[4];
    size_t out_offset[4];
    uint64_t s_id;
    size_t s_offset;
    uint64_t msg_id;
    size_t msg_offset;
    uint64_t q_alpha[2];
} vzb_round_job;
int volta_b200_logup_round_batch_device(void* ctx, const vzb_round_job* jobs, size_t count);

/*
 * volta_cuda_logup_tree_device for a side without multiplicities whose leaves
 * are alpha0 - f_j for a single query column f (pack_lookup_leaf_device with
 * one column at shift 0): the same tree, without the packed leaf column.
 */
int volta_b200_logup_tree_column_device(void* ctx, uint64_t col_id, size_t col_offset, uint64_t alpha0, size_t n,
                                        uint64_t alpha1, uint64_t p_id, size_t p_offset, uint64_t q_id,
                                        size_t q_offset);

/*
 * Suffix-eq tables of several layers at once: job j writes exactly what
 * volta_cuda_logup_suffix_eq_device(ctx, points_id, points_offset, point_len,
 * out_id, out_offset) writes (table k = eq over the last k of the point_len
 * coordinates, at offset 2^k - 1).  Any number of jobs; 2 + ceil(max(L - 12,
 * 0) / 11) launches in all.  Outputs must not overlap.
 */
typedef struct vzb_suffix_job {
    uint64_t points_id;
    size_t points_offset;
    size_t point_len;
    uint64_t out_id;
    size_t out_offset;
} vzb_suffix_job;
int volta_b200_logup_suffix_eq_batch_device(void* ctx, const vzb_suffix_job* jobs, size_t count);

/* All rounds of a triple-product sumcheck on three resident tables of len
 * (<= 2^11, a power of two) entries; challenges at (r_id, r_offset).  Output:
 * 3 messages per round, then the 3 final values. */
int volta_b200_triple_tail_device(void* ctx, uint64_t a_id, uint64_t b_id, uint64_t c_id, size_t len,
                                  uint64_t r_id, size_t r_offset, uint64_t out_id, size_t out_offset);

/*
 * Product sumchecks (two factors, the GEMM and LayerNorm claims of the GPT-2
 * layer proof), the counterparts of the triple-product extensions above:
 *   product_fold_round_into: fold resident a, b (len entries, a multiple of
 *     4) with r into a_out, b_out (len/2 entries) exactly as
 *     volta_cuda_fp2_fold_rows_device, and write the next round's [g(0), g(2)]
 *     (as volta_cuda_fp2_product_round_into_device on the folded vectors) to
 *     (out_id, out_offset): one pass and one launch instead of three;
 *   product_tail: all rounds on two resident vectors of len (<= 2^11, a power
 *     of two) entries in one CTA, challenges at (r_id, r_offset); output: 2
 *     messages per round, then the 2 final values.
 */
int volta_b200_product_fold_round_into_device(void* ctx, uint64_t a_id, uint64_t b_id, size_t len, vz_fp2 r,
                                              uint64_t a_out_id, uint64_t b_out_id, uint64_t out_id,
                                              size_t out_offset);
int volta_b200_product_tail_device(void* ctx, uint64_t a_id, uint64_t b_id, size_t len, uint64_t r_id,
                                   size_t r_offset, uint64_t out_id, size_t out_offset);

/*
 * Triple-product round message without any device allocation.
 *
 * No counterpart in the reference seam.  Every other entry point reserves
 * its reduction workspace through the context (cudaMalloc on first use or
 * growth).  Some callers cannot allocate: code whose HBM is owned by another
 * framework's caching allocator (a process that budgets all device memory
 * itself), and per-round paths that cannot afford the device-wide
 * synchronisation cudaMalloc/cudaFree can trigger.  This variant takes plain
 * device pointers and a stream, and keeps its reduction scratch in a fixed
 * array compiled into the library (VOLTA_B200_NOALLOC_SCRATCH_BYTES per GPU
 * that loads it, held until the process exits).
 *
 *   a, b, c  device pointers to 2*pairs Fp2 each (16-byte aligned)
 *   output   device pointer receiving [g(0), g(2), g(3)] (3 Fp2), the same
 *            values volta_cuda_fp2_triple_product_round_device returns
 *   stream   cudaStream_t to enqueue on (NULL = legacy default stream)
 * Returns 0 on success, -1 on null pointers or pairs == 0, -2
 * (VOLTA_B200_NOALLOC_TOO_LARGE) when pairs exceeds
 * VOLTA_B200_NOALLOC_MAX_PAIRS, or a cudaError_t value.
 *
 * The first call on a device resolves the scratch array's device address
 * (once per device, with that device current); make that first call before
 * any stream capture.  The address is kept per device and driver context: a
 * call after the context was re-created (cudaDeviceReset) resolves it again.  All calls share the one scratch array: calls that
 * overlap on the GPU (concurrent streams, several host threads) race and
 * must be serialised by the caller.  The result is final once `stream`
 * completes.
 */
#define VOLTA_B200_NOALLOC_MAX_PAIRS ((size_t)22369280)  /* 21845 blocks x 1024 pairs */
#define VOLTA_B200_NOALLOC_SCRATCH_BYTES ((size_t)1048576 + 256)
#define VOLTA_B200_NOALLOC_TOO_LARGE (-2)
int volta_b200_triple_product_round_noalloc(const vz_fp2* a, const vz_fp2* b, const vz_fp2* c,
                                            size_t pairs, vz_fp2* output, void* stream);

/*
 * Triple-product rounds on base-field tables: a, b, c are Fp columns (u64,
 * canonical), i.e. Fp2 tables whose c1 is 0 (such as FpStream rows).
 *   triple_round_fp: volta_cuda_fp2_triple_product_round_into_device on the
 *     2 * pairs entries of each column (the message's c1 parts are 0);
 *   triple_fold_round_fp: the fold of each column with r into Fp2 tables of
 *     len / 2 entries (ao, bo, co) and the next round's message on them, as
 *     volta_b200_triple_fold_round_into_device on the lifted tables.
 * Reading 8 bytes per entry and multiplying in Fp, they are exact drop-ins
 * for the first two rounds of a sumcheck whose tables are base-field values.
 */
int volta_b200_triple_round_fp_into_device(void* ctx, uint64_t a_id, uint64_t b_id, uint64_t c_id, size_t pairs,
                                           uint64_t out_id, size_t out_offset);
int volta_b200_triple_fold_round_fp_into_device(void* ctx, uint64_t a_id, uint64_t b_id, uint64_t c_id, size_t len,
                                                vz_fp2 r, uint64_t ao_id, uint64_t bo_id, uint64_t co_id,
                                                uint64_t out_id, size_t out_offset);

/*
 * Thirteen triple-product rounds on chip, tile by tile.
 *
 * No single counterpart in the reference seam: it computes what thirteen
 * rounds of volta_cuda_fp2_triple_product_round_into_device and
 * volta_cuda_fp2_fold_rows_device (cuda/volta_cuda_backend.cu:5106-5153,
 * 6862-6882) compute, for challenges known in advance.  The round pairs
 * entries (2i, 2i + 1), so a tile of 8192 consecutive entries folds into one
 * entry after 13 rounds; each tile runs on one CTA with its tables read once.
 *   a, b, c   len entries (a power of two, >= 8192): Fp columns (u64,
 *             canonical) when base != 0, else Fp2 tables;
 *   tiles     tile0 .. tile0 + tiles - 1 of the len / 8192 tiles (a launch per
 *             uploaded chunk is fine; all tiles must be covered before the
 *             flush);
 *   r         the 13 challenges of these rounds at (r_id, r_offset);
 *   acc       156 u64 counters, zero before the first tile: each tile adds
 *             its share of the 13 messages (3 Fp2 each) exactly (32-bit
 *             halves, integer atomics), so the order of tiles and launches
 *             does not matter;
 *   fa, fb, fc  len / 8192 Fp2 each: the folded a, b, c tables (tile t's
 *             values at entry t), i.e. the tables of round 13.
 * volta_b200_triple_flush_device writes the 39 canonical message values
 * (round-major, 3 per round) at (out_id, out_offset) and zeroes acc.
 */
int volta_b200_triple_local_device(void* ctx, int base, uint64_t a_id, uint64_t b_id, uint64_t c_id, size_t len,
                                   size_t tile0, size_t tiles, uint64_t r_id, size_t r_offset, uint64_t acc_id,
                                   uint64_t fa_id, uint64_t fb_id, uint64_t fc_id);
int volta_b200_triple_flush_device(void* ctx, uint64_t acc_id, uint64_t out_id, size_t out_offset);

/*
 * Asynchronous uploads: upload_async copies `bytes` from `src` (pinned host
 * memory for a truly asynchronous copy) into (id, offset) on the context's
 * copy stream and returns at once; wait_uploads makes the context's stream
 * (every later kernel and download) wait for all uploads issued so far.
 * Until then the destination must not be read, written or freed, and `src`
 * must stay valid.  This lets a caller upload the inputs of one protocol
 * while another protocol computes.
 */
int volta_b200_upload_async(void* ctx, uint64_t id, size_t offset_bytes, const void* src, size_t bytes);
int volta_b200_wait_uploads(void* ctx);

/*
 * Asynchronous downloads (no counterpart in the reference's ABI, which
 * downloads synchronously): download_async copies `bytes` from (id, offset)
 * to host memory `dst` (pinned for a truly asynchronous copy) on a second
 * copy stream, after every kernel enqueued on the context's stream so far,
 * and returns at once, so that the copy overlaps the kernels enqueued after
 * it.  wait_downloads blocks until every such copy has landed; `dst` must
 * stay valid until then.  A buffer freed while a copy is pending may be
 * reused at once: later work on the context's stream waits for the copies.
 */
int volta_b200_download_async(void* ctx, uint64_t id, size_t offset_bytes, void* dst, size_t bytes);
int volta_b200_wait_downloads(void* ctx);

/*
 * int16 column to canonical Fp values (v >= 0 -> v, v < 0 -> p + v), so that
 * int16 witness columns (lookup queries and tables) travel as 2 bytes per
 * entry and are embedded on the device.
 */
int volta_b200_embed_i16_device(void* ctx, uint64_t in_id, size_t in_offset, uint64_t out_id, size_t out_offset,
                                size_t n);

/*
 * Many small host-to-device uploads in one call (the counterpart of one
 * volta_cuda_resident_upload per item): item k copies bytes (1 .. 64 KiB)
 * from host memory src to (dst_id, dst_offset bytes), ordered on the
 * context's stream like any upload.  The items are packed into the pinned
 * staging ring and copied by one launch per filled staging slot.  Every
 * destination is bounds-checked before anything is staged.
 */
typedef struct vzb_upload {
    uint64_t dst_id;
    size_t dst_offset;
    const void* src;
    size_t bytes;
} vzb_upload;
int volta_b200_upload_batch(void* ctx, const vzb_upload* items, size_t count);

/*
 * Many small device-to-device copies in one call (the counterpart of one
 * volta_cuda_resident_copy_rows call per segment with rows = 1): segment k
 * copies bytes from (src_id, src_offset) to (dst_id, dst_offset), offsets in
 * bytes.  Segments must not overlap one another's destinations.  Every
 * segment is bounds-checked before anything is launched; one launch per 96
 * segments.
 */
typedef struct vzb_copy_seg {
    uint64_t src_id;
    size_t src_offset;
    uint64_t dst_id;
    size_t dst_offset;
    size_t bytes;
} vzb_copy_seg;
int volta_b200_copy_segments_device(void* ctx, const vzb_copy_seg* segs, size_t count);

/*
 * Greedy token selection of KV-cached decoding (rust/volta-gpt2/src/decode.rs:
 * 270-272 argmax): the index of the largest of n i64 values, the last one
 * among equal maxima (Iterator::max_by_key), written as a u32 token id at
 * (out_id, out_offset) so the next decode step embeds it without a host
 * round trip.
 */
int volta_b200_argmax_i64_device(void* ctx, uint64_t in_id, size_t in_offset, size_t n, uint64_t out_id,
                                 size_t out_offset);

/*
 * Softmax witness columns of the GPT-2 layer proof, from the forward's
 * causal-packed wires (scores_q, exp_out, weights: heads * rows(rows+1)/2
 * int16; row_shift, recips: heads * rows int16; denoms: heads * rows int64).
 * Writes u64 columns into the buffers out_ids[0..7] (offset 0), [0..5] of
 * n_pad >= packed entries: [0] the score gap c_row - s (the ExpGap table
 * index, rust/volta-gpt2/src/luts.rs:188-206), [1] the exp lookup's packed
 * query gap + 2^16 exp, [2] the exp value (Fp), [3] the softmax-norm requant
 * remainder exp*rc + 2^(s-1) - w*2^s (Range(s) lookup, s = norm_shift), [4]
 * the row's reciprocal (Fp), [5] a 0/1 real-entry mask, the entries past the
 * packed length holding the pads (gap 0, exp = exp_pad, 2^(s-1), 0, 0); and
 * [6..7] of h_pad * t_pad entries (index head * t_pad + row): the reciprocal
 * lookup's input denom >> recip_den_shift (table index over the 18-bit
 * domain, luts.rs:208-226) and its packed query input + 2^18 rc,
 * (recip_pad_in, recip_pad_out) outside the real heads and rows.  An
 * out-of-domain gap, remainder or reciprocal input sets *error to 1.
 * Replaces the host-side column builders of the reference's softmax sites
 * (rust/volta-proto/src/block_proof.rs: build_attn_wires, prove_range_site,
 * c62_softmax_recip_wires).
 */
int volta_b200_softmax_lookup_columns_device(void* ctx, uint64_t scores_id, size_t scores_offset,
                                            uint64_t row_shift_id, size_t row_shift_offset, uint64_t exp_id,
                                            size_t exp_offset, uint64_t denoms_id, size_t denoms_offset,
                                            uint64_t recips_id, size_t recips_offset, uint64_t weights_id,
                                            size_t weights_offset, const uint64_t* out_ids, uint64_t error_id,
                                            size_t error_offset, size_t rows, size_t heads, size_t n_pad,
                                            size_t h_pad, size_t t_pad, uint64_t exp_pad, uint32_t norm_shift,
                                            uint32_t recip_den_shift, uint64_t recip_pad_in, uint64_t recip_pad_out);

/*
 * The same columns for a band of `rows` query rows at positions t0 .. t0 +
 * rows - 1 attending over t0 + rows keys (rust/volta-proto/src/block_proof.rs
 * BandShape, build_attn_wires_band): row i of head h holds t0 + i + 1 packed
 * entries at h * caus + i * t0 + i (i + 1) / 2, caus = rows * t0 +
 * rows (rows + 1) / 2 (band.rs band packing); the row tables are heads x
 * rows and t_pad pads the rows.  t0 = 0 is the entry point above.
 */
int volta_b200_softmax_lookup_columns_band_device(
    void* ctx, uint64_t scores_id, size_t scores_offset, uint64_t row_shift_id, size_t row_shift_offset,
    uint64_t exp_id, size_t exp_offset, uint64_t denoms_id, size_t denoms_offset, uint64_t recips_id,
    size_t recips_offset, uint64_t weights_id, size_t weights_offset, const uint64_t* out_ids, uint64_t error_id,
    size_t error_offset, size_t rows, size_t t0, size_t heads, size_t n_pad, size_t h_pad, size_t t_pad,
    uint64_t exp_pad, uint32_t norm_shift, uint32_t recip_den_shift, uint64_t recip_pad_in, uint64_t recip_pad_out);

/*
 * A pair lookup's query column: out[i] = cols[i] + 2^shift cols[n + i]
 * (mod p) for the two canonical columns at cols (input, then output), as
 * the reference packs pairs (rust/volta-proto/src/block_proof.rs:2511-2520
 * pair_table).
 */
int volta_b200_pack_pair_column_device(void* ctx, uint64_t cols_id, size_t cols_offset, size_t n, uint32_t shift,
                                       uint64_t out_id, size_t out_offset);

/*
 * Factors of the A.V contraction sumcheck (the attention-value GEMM of
 * rust/volta-proto/src/block_proof.rs prove_attn_block): over index
 * h * t_pad + j, A = sum_i eq_rows[i] w[h,i,j] (causal-packed weights),
 * B = sum_c eq_dim[c] v[j, h*head_dim + c] (v: rows x heads*head_dim int16),
 * C = eq_head[h]; three Fp2 vectors of h_pad * t_pad entries into the buffers
 * out_ids[0..2] (offset 0), zero past the real heads and rows.
 */
int volta_b200_av_factors_device(void* ctx, uint64_t weights_id, size_t weights_offset, uint64_t v_id,
                                size_t v_offset, uint64_t eq_rows_id, size_t eq_rows_offset, uint64_t eq_dim_id,
                                size_t eq_dim_offset, uint64_t eq_head_id, size_t eq_head_offset,
                                const uint64_t* out_ids, size_t rows, size_t heads, size_t head_dim, size_t h_pad,
                                size_t t_pad);

/*
 * The A.V factors of a band (rows query rows at positions t0 .. t0 + rows -
 * 1, band-packed weights as above): over index h * s_pad + j for the t0 +
 * rows keys j, A = sum over the rows i with t0 + i >= j of eq_rows[i]
 * w[h,i,j] (eq_rows: q_pad entries), B = sum_c eq_dim[c] v[j, h*head_dim + c]
 * (v: the t0 + rows cached V rows), C = eq_head[h]; h_pad * s_pad entries
 * each.  t0 = 0, q_pad = s_pad = t_pad is the entry point above.
 */
int volta_b200_av_factors_band_device(void* ctx, uint64_t weights_id, size_t weights_offset, uint64_t v_id,
                                     size_t v_offset, uint64_t eq_rows_id, size_t eq_rows_offset,
                                     uint64_t eq_dim_id, size_t eq_dim_offset, uint64_t eq_head_id,
                                     size_t eq_head_offset, const uint64_t* out_ids, size_t rows, size_t t0,
                                     size_t heads, size_t head_dim, size_t h_pad, size_t q_pad, size_t s_pad);

#ifdef __cplusplus
}
#endif
#endif /* VOLTA_B200_EXT_H */
