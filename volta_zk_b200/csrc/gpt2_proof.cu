// Witness columns of the GPT-2 layer proof that no seam entry point
// produces in one pass (include/volta_b200_ext.h):
//
//   softmax_lookup_columns  one warp per causal row (head, row) reads the
//       row's packed scores, exp outputs and normalised weights once and
//       writes, per packed entry, the columns of three sub-proofs of the
//       softmax (rust/volta-proto/src/block_proof.rs layer_lookups:
//       "exp" on the ExpGap table, "softmax_norm" on Range(14); and the
//       norm product exp * recip): the score gap c_row - s
//       (luts.rs:188-206 softmax_exp_from_gap), the exp value, the requant
//       remainder rem = exp * rc + 2^(s-1) - w * 2^s (layer.rs:103-115), the
//       row's reciprocal and a 0/1 real-entry mask.  Entries past the packed
//       length up to the padded length get the pad values (gap 0, exp =
//       ExpGap[0], rem 2^(s-1), rc 0, mask 0), so every column is a
//       complete lookup / sumcheck table.  The exp lookup's query column is
//       written packed (gap + 2^16 exp) beside the gap (its table index).
//       Lane 0 of each row also writes the row's reciprocal lookup input
//       denom >> den_shift and its packed pair input + 2^18 rc at head *
//       t_pad + row (the "softmax_recip" instance over the 18-bit domain,
//       luts.rs:208-226); the other (head, row) slots hold the pad pair.
//       Band form (rows t0 .. t0 + q - 1 of a longer forward, band.rs
//       BandShape): row i's window is t0 + i + 1 keys at i t0 + i (i + 1) / 2
//       of its head's packed segment; the prefill is t0 = 0.
//   pack_pair_column  a + 2^k b of two canonical columns (a pair lookup's
//       query column).
//   av_factors  the three factors of the A.V contraction sumcheck over
//       (head, key position): A[h,j] = sum_i eq_i[i] w[h,i,j] (packed
//       causal weights, t0 + i >= j), B[h,j] = sum_c eq_c[c] v[j, h*dh + c]
//       over the t0 + q cached V rows, C[h,j] = eq_h[h]; index h * s_pad + j,
//       zero past the real heads and keys.
#include "reduce.cuh"
#include "runtime.cuh"

namespace vzb {
namespace {

struct SoftmaxCols {
    uint64_t *gap, *packed, *exp, *rem, *rc, *mask, *rin, *rpacked;
};

__global__ void softmax_columns_kernel(const int16_t* scores, const int16_t* row_shift, const int16_t* exp_out,
                                       const int64_t* denoms, const int16_t* recips, const int16_t* weights,
                                       SoftmaxCols cols, uint32_t* error, size_t rows, size_t t0,
                                       size_t heads, size_t packed, size_t n_pad, size_t h_pad, size_t t_pad,
                                       uint64_t exp_pad, uint64_t packed_pad, uint32_t norm_shift,
                                       uint32_t den_shift, uint64_t recip_pad_in, uint64_t recip_pad_packed) {
    uint64_t* gap_c = cols.gap;
    uint64_t* exp_c = cols.exp;
    uint64_t* packed_c = cols.packed;
    uint64_t* rem_c = cols.rem;
    uint64_t* rc_c = cols.rc;
    uint64_t* mask_c = cols.mask;
    const size_t warp = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const size_t warps = (static_cast<size_t>(gridDim.x) * blockDim.x) >> 5;
    const int lane = threadIdx.x & 31;
    const size_t per_head = rows * t0 + rows * (rows + 1) / 2;
    const int64_t half = int64_t{1} << (norm_shift - 1);
    bool bad = false;
    // real entries: warp per (head, row)
    for (size_t z = warp; z < heads * rows; z += warps) {
        const size_t head = z / rows, row = z - head * rows;
        const size_t start = head * per_head + row * t0 + row * (row + 1) / 2;
        const int32_t c = row_shift[head * rows + row];
        const int64_t rc = recips[head * rows + row];
        if (lane == 0) {
            const int64_t rin = denoms[head * rows + row] >> den_shift;
            if (rin < 0 || rin >= (int64_t{1} << 18)) bad = true;
            const int64_t ri = rin & ((int64_t{1} << 18) - 1);
            cols.rin[head * t_pad + row] = static_cast<uint64_t>(ri);
            cols.rpacked[head * t_pad + row] = ffrom_i64(ri + rc * (int64_t{1} << 18));
        }
        for (size_t j = lane; j <= t0 + row; j += 32) {
            const size_t e = start + j;
            const int64_t gap = static_cast<int64_t>(c) - scores[e];
            const int64_t ex = exp_out[e];
            const int64_t rem = ex * rc + half - static_cast<int64_t>(weights[e]) * (int64_t{1} << norm_shift);
            if (gap < 0 || gap > 0xFFFF || rem < 0 || rem >= (int64_t{1} << norm_shift)) bad = true;
            gap_c[e] = static_cast<uint64_t>(gap & 0xFFFF);
            exp_c[e] = ffrom_i64(ex);
            packed_c[e] = ffrom_i64((gap & 0xFFFF) + ex * 65536);
            rem_c[e] = static_cast<uint64_t>(rem & ((int64_t{1} << norm_shift) - 1));
            rc_c[e] = ffrom_i64(rc);
            mask_c[e] = 1;
        }
    }
    // pads
    for (size_t e = packed + static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < n_pad;
         e += static_cast<size_t>(gridDim.x) * blockDim.x) {
        gap_c[e] = 0;
        exp_c[e] = exp_pad;
        packed_c[e] = packed_pad;
        rem_c[e] = static_cast<uint64_t>(half);
        rc_c[e] = 0;
        mask_c[e] = 0;
    }
    // reciprocal pads: every (head, row) slot outside the real heads and rows
    for (size_t z = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; z < h_pad * t_pad;
         z += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t head = z / t_pad, row = z - head * t_pad;
        if (head < heads && row < rows) continue;
        cols.rin[z] = recip_pad_in;
        cols.rpacked[z] = recip_pad_packed;
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicExch(error, 1u);
}

// out[i] = a[i] + 2^shift b[i] (mod p) for canonical a, b: a packed lookup
// pair as one query column
__global__ void pack_pair_kernel(const uint64_t* a, const uint64_t* b, uint64_t* out, size_t n, uint64_t scale) {
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        out[i] = dadd(__ldcs(a + i), dmul(__ldcs(b + i), scale));
}

// One block per (head, tile of 32 key positions): lane j of each of the 8
// warps takes key position j0 + lane, and the warps split the band rows i
// that see key j (t0 + i >= j; row i's window t0 + i + 1 is contiguous in the
// packed layout, at i t0 + i (i + 1) / 2); the partial sums meet in shared
// memory.  B and C come from warp 0.  keys = t0 + rows.
__global__ void __launch_bounds__(256) av_factors_kernel(const int16_t* weights, const int16_t* v,
                                                         const Fp2* eq_i, const Fp2* eq_c, const Fp2* eq_h,
                                                         Fp2* out_a, Fp2* out_b, Fp2* out_c, size_t rows, size_t t0,
                                                         size_t heads, size_t head_dim, size_t h_pad,
                                                         size_t s_pad) {
    __shared__ Fp2 part[8][32];
    const size_t tiles = (s_pad + 31) / 32, keys = t0 + rows;
    const size_t h = blockIdx.x / tiles, j = (blockIdx.x % tiles) * 32 + (threadIdx.x & 31);
    const unsigned w = threadIdx.x >> 5;
    const size_t per_head = rows * t0 + rows * (rows + 1) / 2;
    Fp2 a{0, 0};
    if (h < heads && j < keys) {
        const int16_t* wh = weights + h * per_head;
        for (size_t i = (j > t0 ? j - t0 : 0) + w; i < rows; i += 8) {
            const int16_t x = wh[i * t0 + i * (i + 1) / 2 + j];
            if (x) a = f2add(a, f2mul_base(ldg2(eq_i + i), ffrom_i64(x)));
        }
    }
    part[w][threadIdx.x & 31] = a;
    __syncthreads();
    if (w == 0 && j < s_pad) {
        for (int k = 1; k < 8; ++k) a = f2add(a, part[k][threadIdx.x]);
        Fp2 b{0, 0};
        if (h < heads && j < keys) {
            const int16_t* vr = v + j * heads * head_dim + h * head_dim;
            for (size_t c = 0; c < head_dim; ++c) {
                const int16_t x = vr[c];
                if (x) b = f2add(b, f2mul_base(ldg2(eq_c + c), ffrom_i64(x)));
            }
        }
        const size_t z = h * s_pad + j;
        st2(out_a + z, a);
        st2(out_b + z, b);
        st2(out_c + z, ldg2(eq_h + h));
    }
}

}  // namespace
}  // namespace vzb

using namespace vzb;

extern "C" int volta_b200_softmax_lookup_columns_band_device(
    void* raw, uint64_t scores_id, size_t scores_offset, uint64_t row_shift_id, size_t row_shift_offset,
    uint64_t exp_id, size_t exp_offset, uint64_t denoms_id, size_t denoms_offset, uint64_t recips_id,
    size_t recips_offset, uint64_t weights_id, size_t weights_offset, const uint64_t* out_ids, uint64_t error_id,
    size_t error_offset, size_t rows, size_t t0, size_t heads, size_t n_pad, size_t h_pad, size_t t_pad,
    uint64_t exp_pad, uint32_t norm_shift, uint32_t recip_den_shift, uint64_t recip_pad_in, uint64_t recip_pad_out) {
    Context* c = static_cast<Context*>(raw);
    const size_t packed = heads * (rows * t0 + rows * (rows + 1) / 2);
    if (!c || !out_ids || !rows || !heads || n_pad < packed || h_pad < heads || t_pad < rows || !norm_shift ||
        norm_shift > 30 || !recip_den_shift || recip_den_shift > 30 || exp_pad >= kP || recip_pad_in >= (1u << 18) ||
        recip_pad_out >= kP)
        return fail_message(c, "invalid softmax lookup column geometry");
    void *sc = nullptr, *rs = nullptr, *ex = nullptr, *dn = nullptr, *rc = nullptr, *w = nullptr, *err = nullptr;
    void* outs[8] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
    if (region_elems(c, scores_id, scores_offset, packed, 2, &sc) ||
        region_elems(c, row_shift_id, row_shift_offset, heads * rows, 2, &rs) ||
        region_elems(c, exp_id, exp_offset, packed, 2, &ex) ||
        region_elems(c, denoms_id, denoms_offset, heads * rows, 8, &dn) ||
        region_elems(c, recips_id, recips_offset, heads * rows, 2, &rc) ||
        region_elems(c, weights_id, weights_offset, packed, 2, &w) ||
        region_elems(c, error_id, error_offset, 1, 4, &err))
        return -1;
    for (int k = 0; k < 8; ++k)
        if (region_elems(c, out_ids[k], 0, k < 6 ? n_pad : h_pad * t_pad, 8, &outs[k])) return -1;
    SoftmaxCols cols;
    uint64_t** dst[8] = {&cols.gap, &cols.packed, &cols.exp, &cols.rem, &cols.rc, &cols.mask, &cols.rin, &cols.rpacked};
    for (int k = 0; k < 8; ++k) *dst[k] = static_cast<uint64_t*>(outs[k]);
    // pads: gap 0 with ExpGap[0]; the reciprocal pad pair, packed
    const uint64_t packed_pad = fmul(exp_pad, uint64_t{1} << 16);
    const uint64_t recip_pad_packed = fadd(recip_pad_in, fmul(recip_pad_out, uint64_t{1} << 18));
    if (op_begin(c) || op_mark(c, 1)) return -1;
    softmax_columns_kernel<<<grid_for(c, n_pad, 256), 256, 0, c->stream>>>(
        static_cast<const int16_t*>(sc), static_cast<const int16_t*>(rs), static_cast<const int16_t*>(ex),
        static_cast<const int64_t*>(dn), static_cast<const int16_t*>(rc), static_cast<const int16_t*>(w), cols,
        static_cast<uint32_t*>(err), rows, t0, heads, packed, n_pad, h_pad, t_pad, exp_pad, packed_pad, norm_shift,
        recip_den_shift, recip_pad_in, recip_pad_packed);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpLogup, 0, 0);
}

extern "C" int volta_b200_softmax_lookup_columns_device(
    void* raw, uint64_t scores_id, size_t scores_offset, uint64_t row_shift_id, size_t row_shift_offset,
    uint64_t exp_id, size_t exp_offset, uint64_t denoms_id, size_t denoms_offset, uint64_t recips_id,
    size_t recips_offset, uint64_t weights_id, size_t weights_offset, const uint64_t* out_ids, uint64_t error_id,
    size_t error_offset, size_t rows, size_t heads, size_t n_pad, size_t h_pad, size_t t_pad, uint64_t exp_pad,
    uint32_t norm_shift, uint32_t recip_den_shift, uint64_t recip_pad_in, uint64_t recip_pad_out) {
    return volta_b200_softmax_lookup_columns_band_device(
        raw, scores_id, scores_offset, row_shift_id, row_shift_offset, exp_id, exp_offset, denoms_id, denoms_offset,
        recips_id, recips_offset, weights_id, weights_offset, out_ids, error_id, error_offset, rows, 0, heads, n_pad,
        h_pad, t_pad, exp_pad, norm_shift, recip_den_shift, recip_pad_in, recip_pad_out);
}

extern "C" int volta_b200_pack_pair_column_device(void* raw, uint64_t cols_id, size_t cols_offset, size_t n,
                                                  uint32_t shift, uint64_t out_id, size_t out_offset) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !n || shift >= 64) return fail_message(c, "invalid pair-column packing geometry");
    void *cols = nullptr, *out = nullptr;
    if (region_elems(c, cols_id, cols_offset, 2 * n, 8, &cols) || region_elems(c, out_id, out_offset, n, 8, &out))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    const uint64_t* a = static_cast<const uint64_t*>(cols);
    pack_pair_kernel<<<grid_for(c, n, 256), 256, 0, c->stream>>>(a, a + n, static_cast<uint64_t*>(out), n,
                                                                 uint64_t{1} << shift);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpLogup, 0, 0);
}

extern "C" int volta_b200_av_factors_band_device(void* raw, uint64_t weights_id, size_t weights_offset,
                                                uint64_t v_id, size_t v_offset, uint64_t eq_rows_id,
                                                size_t eq_rows_offset, uint64_t eq_dim_id, size_t eq_dim_offset,
                                                uint64_t eq_head_id, size_t eq_head_offset, const uint64_t* out_ids,
                                                size_t rows, size_t t0, size_t heads, size_t head_dim, size_t h_pad,
                                                size_t q_pad, size_t s_pad) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !out_ids || !rows || !heads || !head_dim || h_pad < heads || q_pad < rows || s_pad < t0 + rows)
        return fail_message(c, "invalid A.V factor geometry");
    const size_t packed = heads * (rows * t0 + rows * (rows + 1) / 2);
    void *w = nullptr, *v = nullptr, *ei = nullptr, *ec = nullptr, *eh = nullptr;
    void* outs[3] = {nullptr, nullptr, nullptr};
    if (region_elems(c, weights_id, weights_offset, packed, 2, &w) ||
        region_elems(c, v_id, v_offset, (t0 + rows) * heads * head_dim, 2, &v) ||
        region_elems(c, eq_rows_id, eq_rows_offset, q_pad, sizeof(Fp2), &ei) ||
        region_elems(c, eq_dim_id, eq_dim_offset, head_dim, sizeof(Fp2), &ec) ||
        region_elems(c, eq_head_id, eq_head_offset, h_pad, sizeof(Fp2), &eh))
        return -1;
    for (int k = 0; k < 3; ++k)
        if (region_elems(c, out_ids[k], 0, h_pad * s_pad, sizeof(Fp2), &outs[k])) return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    av_factors_kernel<<<static_cast<unsigned>(h_pad * ((s_pad + 31) / 32)), 256, 0, c->stream>>>(
        static_cast<const int16_t*>(w), static_cast<const int16_t*>(v), static_cast<const Fp2*>(ei),
        static_cast<const Fp2*>(ec), static_cast<const Fp2*>(eh), static_cast<Fp2*>(outs[0]),
        static_cast<Fp2*>(outs[1]), static_cast<Fp2*>(outs[2]), rows, t0, heads, head_dim, h_pad, s_pad);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpGemm, 0, 0);
}

extern "C" int volta_b200_av_factors_device(void* raw, uint64_t weights_id, size_t weights_offset, uint64_t v_id,
                                           size_t v_offset, uint64_t eq_rows_id, size_t eq_rows_offset,
                                           uint64_t eq_dim_id, size_t eq_dim_offset, uint64_t eq_head_id,
                                           size_t eq_head_offset, const uint64_t* out_ids, size_t rows, size_t heads,
                                           size_t head_dim, size_t h_pad, size_t t_pad) {
    return volta_b200_av_factors_band_device(raw, weights_id, weights_offset, v_id, v_offset, eq_rows_id,
                                             eq_rows_offset, eq_dim_id, eq_dim_offset, eq_head_id, eq_head_offset,
                                             out_ids, rows, 0, heads, head_dim, h_pad, t_pad, t_pad);
}
