// Attention proof wires (seam entry point cuda/volta_cuda_backend.cu:5278-5375,
// kernels 2202-2470): the column witnesses the attention sub-proof commits
// to, built from the forward's own tensors, with every consistency check of
// the reference folded into the sticky error word:
//   rect  9 columns over head_pad x query_pad x seq_pad (normalisation and
//         score remainders, weights, score values / indices, exp inputs and
//         outputs, row-max markers, full scores)
//   rows  13 columns over head_pad x query_pad (denominators, reciprocal
//         inputs / outputs / shifts and the limbs of the reciprocal's
//         division relation)
//   above the full scores strictly above the causal diagonal
//   qkv   2 columns over query_pad x 4 d_pad (QKV requant remainders, outputs)
#include "runtime.cuh"

namespace vzb {
namespace {

__device__ __forceinline__ void flag(uint32_t* error) { atomicExch(error, 1u); }

__device__ __forceinline__ int64_t requant_rounded(int64_t acc, uint32_t shift) {
    int64_t stage = acc;
    uint32_t fin = shift;
    if (shift > 16) {
        const uint32_t first = shift - 16;
        stage = (stage + (int64_t{1} << (first - 1))) >> first;
        fin = 16;
    }
    return (stage + (int64_t{1} << (fin - 1))) >> fin;
}

__device__ __forceinline__ size_t packed_prefix(size_t row, size_t pos0) { return row * pos0 + row * (row + 1) / 2; }

__device__ __forceinline__ int16_t recip_value(int64_t input, const int16_t* lut, uint32_t den_shift,
                                               uint32_t recip_log2, int use_row_shift, bool& bad) {
    const int64_t limit = use_row_shift ? (int64_t{1} << 18) : (int64_t{1} << 16);
    if (input < 0 || input >= limit) {
        bad = true;
        return lut[0];
    }
    if (input < (int64_t{1} << 16)) return lut[static_cast<size_t>(input)];
    const uint64_t den_back = (static_cast<uint64_t>(input) << den_shift) + (uint64_t{1} << (den_shift - 1));
    uint64_t v = ((uint64_t{1} << recip_log2) + den_back / 2) / den_back;
    if (v > static_cast<uint64_t>(INT16_MAX)) v = INT16_MAX;
    return static_cast<int16_t>(v);
}

struct Wires {
    const int16_t *q, *k_cache, *own_k, *v, *scores_q, *row_shifts, *exp_outputs, *recips, *weights, *recip_lut;
    const int64_t *scores_acc, *denoms, *qkv_acc;
    uint64_t *rect, *rows, *above, *qkv;
    uint32_t* error;
    vz_attention_wires_args a;
};

__global__ void rect_kernel(Wires w) {
    const vz_attention_wires_args& a = w.a;
    const size_t sp2 = a.query_pad * a.seq_pad, entries = a.head_pad * sp2;
    const size_t qr = a.query_rows, d = a.heads * a.head_dim;
    const size_t per_head = qr * a.pos0 + qr * (qr + 1) / 2;
    const int rs = a.use_row_shift;
    const int64_t half_s = int64_t{1} << (a.shift_scores - 1), half_n = int64_t{1} << (a.shift_softmax_norm - 1);
    for (size_t z = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; z < entries;
         z += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t head = z / sp2, rem = z - head * sp2, row = rem / a.seq_pad, col = rem - row * a.seq_pad;
        int64_t norm_rem = half_n, weight = 0, score_rem = half_s;
        int64_t score_value = rs ? -static_cast<int64_t>(a.exp_pad_input) : static_cast<int64_t>(a.exp_pad_input);
        int64_t score_index = score_value + (int64_t{1} << 16);
        int64_t exp_input = a.exp_pad_input, exp_value = 0, is_max = 0, full = 0;
        bool bad = false;
        if (head < a.heads && row < qr && col < a.seq) {
            const int16_t* qrow = w.q + row * d + head * a.head_dim;
            const int16_t* krow = w.k_cache + col * d + head * a.head_dim;
            for (size_t l = 0; l < a.head_dim; ++l) full += static_cast<int64_t>(qrow[l]) * krow[l];
            const size_t width = a.pos0 + row + 1;
            if (col < width) {
                const size_t start = head * per_head + packed_prefix(row, a.pos0), pk = start + col;
                const int64_t acc = w.scores_acc[pk];
                const int64_t score = w.scores_q[pk];
                const int64_t raw = requant_rounded(acc, a.shift_scores);
                const int64_t clamped = raw < INT16_MIN ? INT16_MIN : (raw > INT16_MAX ? INT16_MAX : raw);
                bad |= raw < -(int64_t{1} << 16) || raw >= (int64_t{1} << 16) || score != clamped;
                const int64_t shift_v = rs ? w.row_shifts[head * qr + row] : 0;
                score_value = score;
                score_index = raw + (int64_t{1} << 16);
                exp_input = rs ? shift_v - score : score;
                bad |= rs ? (exp_input < 0 || exp_input > UINT16_MAX) : (exp_input < INT16_MIN || exp_input > INT16_MAX);
                score_rem = acc + half_s - raw * (int64_t{1} << a.shift_scores);
                bad |= score_rem < 0 || score_rem >= (int64_t{1} << a.shift_scores);
                bad |= acc != full;
                exp_value = w.exp_outputs[pk];
                weight = w.weights[pk];
                const int64_t rc = w.recips[head * qr + row];
                norm_rem = exp_value * rc + half_n - weight * (int64_t{1} << a.shift_softmax_norm);
                bad |= norm_rem < 0 || norm_rem >= (int64_t{1} << a.shift_softmax_norm);
                if (rs && exp_input == 0) {  // first occurrence of the row maximum
                    bool first = true;
                    for (size_t prior = 0; prior < col && first; ++prior)
                        first = static_cast<int64_t>(w.scores_q[start + prior]) != shift_v;
                    is_max = first ? 1 : 0;
                }
            } else {
                const size_t local = col - width;
                const size_t row_prefix = row * (qr - 1) - row * (row - 1) / 2;
                w.above[head * (qr * (qr - 1) / 2) + row_prefix + local] = ffrom_i64(full);
            }
        }
        if (bad) flag(w.error);
        w.rect[z] = static_cast<uint64_t>(norm_rem);
        w.rect[entries + z] = ffrom_i64(weight);
        w.rect[2 * entries + z] = static_cast<uint64_t>(score_rem);
        w.rect[3 * entries + z] = rs ? static_cast<uint64_t>(score_index) : ffrom_i64(score_value);
        w.rect[4 * entries + z] = ffrom_i64(score_value);
        w.rect[5 * entries + z] = rs ? static_cast<uint64_t>(exp_input) : ffrom_i64(exp_input);
        w.rect[6 * entries + z] = ffrom_i64(exp_value);
        w.rect[7 * entries + z] = static_cast<uint64_t>(is_max);
        w.rect[8 * entries + z] = ffrom_i64(full);
    }
}

__global__ void row_kernel(Wires w) {
    const vz_attention_wires_args& a = w.a;
    const size_t entries = a.head_pad * a.query_pad, qr = a.query_rows;
    const size_t per_head = qr * a.pos0 + qr * (qr + 1) / 2;
    const uint32_t ds = a.recip_den_shift;
    for (size_t z = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; z < entries;
         z += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t head = z / a.query_pad, row = z - head * a.query_pad;
        int64_t denom = 0, rin = 0, rc = a.recip_pad_output, shift_v = 0;
        bool real = false, bad = false;
        if (head < a.heads && row < qr) {
            real = true;
            denom = w.denoms[head * qr + row];
            rin = denom >> ds;
            rc = w.recips[head * qr + row];
            shift_v = a.use_row_shift ? w.row_shifts[head * qr + row] : 0;
            const int16_t expect = recip_value(rin, w.recip_lut, ds, a.recip_log2, a.use_row_shift, bad);
            bad |= expect != rc;
            if (a.use_row_shift) {
                const size_t start = head * per_head + packed_prefix(row, a.pos0), width = a.pos0 + row + 1;
                bool found = false;
                for (size_t c = 0; c < width && !found; ++c) found = w.scores_q[start + c] == shift_v;
                bad |= !found || width > a.seq;
            }
        }
        w.rows[z] = ffrom_i64(denom);
        w.rows[entries + z] = static_cast<uint64_t>(rin);
        w.rows[2 * entries + z] = ffrom_i64(rc);
        w.rows[3 * entries + z] = ffrom_i64(shift_v);
        // the reciprocal's division relation (padding rows use input 256)
        const int64_t r_in = real ? rin : 256;
        const int64_t r_den = real ? denom : (int64_t{256} << ds);
        const int64_t r_q = real ? rc : recip_value(256, w.recip_lut, ds, a.recip_log2, 1, bad);
        const int64_t denom_low = r_den - (r_in << ds);
        const int64_t divisor = (r_in << ds) + (int64_t{1} << (ds - 1));
        const int64_t remainder = (int64_t{1} << a.recip_log2) + divisor / 2 - r_q * divisor;
        const int64_t slack = divisor - 1 - remainder;
        bad |= denom_low < 0 || denom_low >= (int64_t{1} << ds) || r_in < 0 || r_in >= (int64_t{1} << 18) ||
               r_q < 0 || r_q >= (int64_t{1} << 15) || remainder < 0 || remainder >= divisor ||
               remainder >= (int64_t{1} << 24) || slack < 0 || slack >= (int64_t{1} << 24);
        if (bad) flag(w.error);
        w.rows[4 * entries + z] = static_cast<uint64_t>(denom_low);
        w.rows[5 * entries + z] = static_cast<uint64_t>(r_in & 0xffff);
        w.rows[6 * entries + z] = static_cast<uint64_t>(r_in >> 16);
        w.rows[7 * entries + z] = static_cast<uint64_t>(r_q);
        w.rows[8 * entries + z] = static_cast<uint64_t>(remainder & 0xffff);
        w.rows[9 * entries + z] = static_cast<uint64_t>(remainder >> 16);
        w.rows[10 * entries + z] = static_cast<uint64_t>(slack & 0xffff);
        w.rows[11 * entries + z] = static_cast<uint64_t>(slack >> 16);
        w.rows[12 * entries + z] = static_cast<uint64_t>(divisor);
    }
}

__global__ void qkv_kernel(Wires w) {
    const vz_attention_wires_args& a = w.a;
    const size_t d = a.heads * a.head_dim, width = 4 * a.d_pad, entries = a.query_pad * width;
    const int64_t half = int64_t{1} << (a.shift_qkv - 1);
    for (size_t z = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; z < entries;
         z += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t row = z / width, col = z - row * width, third = col / a.d_pad, rest = col - third * a.d_pad;
        int64_t rem = half, out = 0;
        if (row < a.query_rows && third < 3 && rest < d) {
            out = third == 0 ? w.q[row * d + rest] : (third == 1 ? w.own_k[row * d + rest] : w.v[row * d + rest]);
            rem = w.qkv_acc[row * 3 * d + third * d + rest] + half - out * (int64_t{1} << a.shift_qkv);
            if (rem < 0 || rem >= (int64_t{1} << a.shift_qkv)) flag(w.error);
        }
        w.qkv[z] = static_cast<uint64_t>(rem);
        w.qkv[entries + z] = ffrom_i64(out);
    }
}

bool pow2(size_t n) { return n && !(n & (n - 1)); }

template <class P>
int typed_region(Context* c, uint64_t id, size_t off, size_t count, P*& out) {
    void* p = nullptr;
    if (region_elems(c, id, off, count, sizeof(P), &p)) return -1;
    out = static_cast<P*>(p);
    return 0;
}

}  // namespace
}  // namespace vzb

using namespace vzb;

extern "C" int volta_cuda_attention_proof_wires_device(void* raw, const vz_attention_wires_args* args) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !args) return fail_message(c, "invalid resident attention-proof geometry");
    const vz_attention_wires_args& a = *args;
    if (a.query_rows < 2 || !a.seq || !a.heads || !a.head_dim || a.head_pad < a.heads || !pow2(a.head_pad) ||
        a.pos0 + a.query_rows != a.seq || a.query_pad < a.query_rows || !pow2(a.query_pad) || a.seq_pad < a.seq ||
        !pow2(a.seq_pad) || a.d_pad < a.heads * a.head_dim || !pow2(a.d_pad) || !a.shift_scores ||
        a.shift_scores > 16 || !a.shift_softmax_norm || a.shift_softmax_norm > 16 || !a.shift_qkv ||
        a.shift_qkv > 16 || !a.recip_den_shift || a.recip_den_shift >= 63 || a.recip_log2 >= 63 ||
        a.exp_pad_input < INT16_MIN || a.exp_pad_input > INT16_MAX || a.recip_pad_output < INT16_MIN ||
        a.recip_pad_output > INT16_MAX || (a.use_row_shift != 0 && a.use_row_shift != 1))
        return fail_message(c, "invalid resident attention-proof geometry");
    const size_t d = a.heads * a.head_dim;
    const size_t packed = a.heads * (a.query_rows * a.pos0 + a.query_rows * (a.query_rows + 1) / 2);
    const size_t real_rows = a.heads * a.query_rows;
    const size_t rect_entries = a.head_pad * a.query_pad * a.seq_pad, row_entries = a.head_pad * a.query_pad;
    const size_t above_entries = a.heads * a.query_rows * (a.query_rows - 1) / 2;
    const size_t qkv_entries = a.query_pad * 4 * a.d_pad;
    Wires w{};
    w.a = a;
    if (typed_region(c, a.q_id, a.q_offset, a.query_rows * d, w.q) ||
        typed_region(c, a.k_cache_id, a.k_cache_offset, a.seq * d, w.k_cache) ||
        typed_region(c, a.own_k_id, a.own_k_offset, a.query_rows * d, w.own_k) ||
        typed_region(c, a.v_id, a.v_offset, a.query_rows * d, w.v) ||
        typed_region(c, a.scores_acc_id, a.scores_acc_offset, packed, w.scores_acc) ||
        typed_region(c, a.scores_q_id, a.scores_q_offset, packed, w.scores_q) ||
        typed_region(c, a.row_shifts_id, a.row_shifts_offset, real_rows, w.row_shifts) ||
        typed_region(c, a.exp_outputs_id, a.exp_outputs_offset, packed, w.exp_outputs) ||
        typed_region(c, a.denoms_id, a.denoms_offset, real_rows, w.denoms) ||
        typed_region(c, a.recips_id, a.recips_offset, real_rows, w.recips) ||
        typed_region(c, a.softmax_weights_id, a.softmax_weights_offset, packed, w.weights) ||
        typed_region(c, a.recip_lut_id, a.recip_lut_offset, size_t{1} << 16, w.recip_lut) ||
        typed_region(c, a.qkv_acc_id, a.qkv_acc_offset, a.query_rows * 3 * d, w.qkv_acc) ||
        typed_region(c, a.error_id, a.error_offset, 1, w.error) ||
        typed_region(c, a.rect_id, a.rect_offset, 9 * rect_entries, w.rect) ||
        typed_region(c, a.rows_id, a.rows_offset, 13 * row_entries, w.rows) ||
        typed_region(c, a.above_id, a.above_offset, above_entries, w.above) ||
        typed_region(c, a.qkv_id, a.qkv_offset, 2 * qkv_entries, w.qkv))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    rect_kernel<<<grid_for(c, rect_entries, 256), 256, 0, c->stream>>>(w);
    VZB_LAUNCHED(c);
    row_kernel<<<grid_for(c, row_entries, 256), 256, 0, c->stream>>>(w);
    VZB_LAUNCHED(c);
    qkv_kernel<<<grid_for(c, qkv_entries, 256), 256, 0, c->stream>>>(w);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpLogup, 0, 0);
}
